"""Generate the golden GEMM fixtures from the reference implementation.

Run in a container where the reference package is importable (it is NOT
needed at test time; the fixtures are committed):

    python tests/golden/make_golden.py --ref-src /path/to/reference/src

For each case it builds seeded fp16 inputs on the CPU, calls the reference's
public ``tensorcore_gemm.gemm(A, B, mode)`` on CPU tensors, which is the
reference's CPU path (``is_supported`` is False for CPU tensors, so it returns
``torch.matmul(A, B)`` in fp16: tensorcore_gemm/gemm.py:219-221), and stores
A, B and that output in ``gemm_golden.npz``.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

# (name, M, N, K, distribution, seed_a, seed_b)
CASES = [
    ("tiny_1x8x8", 1, 8, 8, "uniform", 10, 11),
    ("odd_37x24x40", 37, 24, 40, "uniform", 12, 13),
    ("aligned_256x128x64", 256, 128, 64, "uniform", 14, 15),
    ("skinny_64x256x256", 64, 256, 256, "normal", 16, 17),
    ("deep_48x64x1000", 48, 64, 1000, "uniform", 18, 19),
    ("ragged_130x72x136", 130, 72, 136, "normal", 20, 21),
]


def make(M, N, K, dist, sa, sb):
    ga = torch.Generator().manual_seed(sa)
    gb = torch.Generator().manual_seed(sb)
    if dist == "uniform":
        A = torch.rand((M, K), generator=ga) * 2 - 1
        B = torch.rand((K, N), generator=gb) * 2 - 1
    else:
        A = torch.randn((M, K), generator=ga)
        B = torch.randn((K, N), generator=gb)
    return A.half(), B.half()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-src", default="/root/reference/src")
    args = ap.parse_args()
    sys.path.insert(0, args.ref_src)
    import tensorcore_gemm as ref  # the unmodified reference package

    arrays = {}
    meta = []
    for name, M, N, K, dist, sa, sb in CASES:
        A, B = make(M, N, K, dist, sa, sb)
        C = ref.gemm(A, B, mode="reg_pingpong_256")
        assert C.dtype == torch.float16 and tuple(C.shape) == (M, N)
        arrays[f"{name}__A"] = A.numpy()
        arrays[f"{name}__B"] = B.numpy()
        arrays[f"{name}__C"] = C.numpy()
        meta.append({"name": name, "M": M, "N": N, "K": K, "dist": dist, "seed_a": sa, "seed_b": sb})
    np.savez_compressed(HERE / "gemm_golden.npz", **arrays)
    (HERE / "gemm_golden.json").write_text(json.dumps({
        "generator": "tests/golden/make_golden.py",
        "reference_call": "tensorcore_gemm.gemm(A_cpu, B_cpu, mode='reg_pingpong_256') -> torch.matmul fallback",
        "torch": torch.__version__,
        "cases": meta,
    }, indent=1) + "\n")
    print(f"wrote {len(meta)} cases")


if __name__ == "__main__":
    main()
