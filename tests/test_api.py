"""CPU: the drop-in Python API (names, modes, errors, no fallback)."""
from __future__ import annotations

from pathlib import Path

import pytest
import torch

import tensorcore_gemm as tg
import importlib

gemm_mod = importlib.import_module("tensorcore_gemm.gemm")

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "ampere-gemm_b200" / "tensorcore_gemm"

REFERENCE_MODES = (
    "wmma", "mma", "reg_pingpong_256", "reg_pingpong_256_mma",
    "reg_pingpong_256_colb", "reg_pingpong_256_colb_mma",
)


def test_public_names():
    assert tg.__all__ == ["KERNEL_MODES", "gemm", "gemm_pretransposed", "is_supported"]
    assert tg.KERNEL_MODES == REFERENCE_MODES


def test_unknown_mode_is_value_error():
    with pytest.raises(ValueError, match="Unsupported mode"):
        gemm_mod._normalize_mode("wgmma")
    A = torch.zeros(8, 8, dtype=torch.float16)
    with pytest.raises(ValueError):
        tg.gemm(A, A, mode="nope")
    with pytest.raises(ValueError):
        tg.gemm_pretransposed(A, A, mode="nope")


def test_cpu_tensors_raise_instead_of_falling_back():
    A = torch.ones(16, 16, dtype=torch.float16)
    assert not tg.is_supported(A, A)
    with pytest.raises(RuntimeError, match="CUDA"):
        tg.gemm(A, A)
    with pytest.raises(RuntimeError, match="CUDA"):
        tg.gemm_pretransposed(A, A, mode="reg_pingpong_256_colb")
    with pytest.raises(RuntimeError, match="CUDA"):
        gemm_mod.root_gemm_cuda(A, A, 2)


def test_is_supported_shape_rules():
    # CPU tensors are never supported; the shape rule itself is checked here.
    A = torch.zeros(3, 8, dtype=torch.float16)
    B = torch.zeros(9, 8, dtype=torch.float16)
    assert not tg.is_supported(A, B)      # inner mismatch
    assert not tg.is_supported(A.float(), A.float().t())


def test_mode_ids_and_operand_conventions():
    assert [gemm_mod._normalize_mode(m) for m in REFERENCE_MODES] == [0, 1, 2, 3, 4, 5]
    # gemm_pretransposed reads its operand as K x N for ids 2/3 (reference quirk).
    assert gemm_mod._PRETRANSPOSED_ROW_MAJOR_IDS == {2, 3}


def test_product_path_never_touches_oracle_or_fallbacks():
    import ast

    for src in PKG.glob("*.py"):
        tree = ast.parse(src.read_text())
        for node in ast.walk(tree):
            if isinstance(node, (ast.Import, ast.ImportFrom)):
                mods = [a.name for a in node.names] + [getattr(node, "module", None) or ""]
                assert not any("oracle" in m for m in mods), f"{src.name} imports the oracle"
            if isinstance(node, ast.Call) and isinstance(node.func, ast.Attribute) and src.name != "cublas_gemm.py":
                f = node.func
                if isinstance(f.value, ast.Name) and f.value.id == "torch":
                    assert f.attr not in ("matmul", "mm", "bmm", "addmm"), f"{src.name} calls torch.{f.attr}"
