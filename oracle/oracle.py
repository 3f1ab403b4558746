"""Python front of the CPU oracle (gemm_oracle.c) and of the reference kernels.

TEST INFRASTRUCTURE ONLY.  Imported by tests/, __graft_entry__.smoke() and
bench.py's cpu_baseline leg, always as the checker; the product path
(ampere-gemm_b200/tensorcore_gemm) never imports it.

* ``gemm_f16``     oracle GEMM on numpy fp16 arrays: fp32 sum of fp16
                   products, one round-to-nearest-even to fp16.  Restates the
                   reference kernels' arithmetic (tensorcore_gemm/gemm.cu
                   :1208-1290 loop, :1360-1361 epilogue).
* ``parity_ok``    the acceptance bound of the hot path:
                   max|C - C_ref| <= 2e-3 * sqrt(K) * RMS(C_ref), C_ref the
                   fp32 product of the same fp16 inputs.
* ``ref_kernels``  ctypes handle of oracle/_ref/libref_gemm.so: the reference's
                   own reg_pingpong_256* CUDA kernels, for GPU cross-checks.
"""
from __future__ import annotations

import ctypes
import math
import shutil
import subprocess
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
LIB = ORACLE_DIR / "liboracle.so"
REF_LIB = ORACLE_DIR / "_ref" / "libref_gemm.so"

PARITY_COEFF = 2e-3  # 2e-3 * sqrt(K) * RMS(C_ref)

_lib = None


def build(force: bool = False) -> Path:
    """Compile liboracle.so with gcc (make)."""
    if force or not LIB.exists() or LIB.stat().st_mtime < (ORACLE_DIR / "gemm_oracle.c").stat().st_mtime:
        if shutil.which("make") is None:
            raise RuntimeError("make not found; cannot build the oracle")
        subprocess.run(["make", "-s", "-C", str(ORACLE_DIR), "liboracle.so"], check=True)
    return LIB


def build_ref(ref_src: str | None = None) -> Path | None:
    """Compile the reference kernels into _ref/ when their sources exist."""
    src = Path(ref_src or "/root/reference/src/tensorcore_gemm")
    if not (src / "gemm.cu").exists() or shutil.which("nvcc") is None and not Path("/usr/local/cuda/bin/nvcc").exists():
        return REF_LIB if REF_LIB.exists() else None
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    subprocess.run(["make", "-s", "-C", str(ORACLE_DIR), "ref", f"REF_SRC={src}", f"NVCC={nvcc}"], check=True)
    return REF_LIB


def _load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(str(LIB))
        lib.oracle_gemm_f16.restype = ctypes.c_int
        lib.oracle_gemm_f16.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                        ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                        ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                        ctypes.c_int, ctypes.c_int]
        lib.oracle_f16_to_f32_array.restype = None
        lib.oracle_f16_to_f32_array.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64]
        lib.oracle_f32_to_f16_array.restype = None
        lib.oracle_f32_to_f16_array.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64]
        _lib = lib
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def f16_to_f32(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.float16).view(np.uint16)
    out = np.empty(h.shape, dtype=np.float32)
    _load().oracle_f16_to_f32_array(_ptr(h), _ptr(out), h.size)
    return out


def f32_to_f16(f: np.ndarray) -> np.ndarray:
    f = np.ascontiguousarray(f, dtype=np.float32)
    out = np.empty(f.shape, dtype=np.uint16)
    _load().oracle_f32_to_f16_array(_ptr(f), _ptr(out), f.size)
    return out.view(np.float16)


def gemm_f16(A: np.ndarray, B: np.ndarray, b_col_major: bool = False, threads: int = 1,
             want_acc: bool = True) -> tuple[np.ndarray, np.ndarray | None]:
    """Oracle C = A @ B (or A @ B.T when b_col_major) -> (C fp16, fp32 accumulator)."""
    A = np.ascontiguousarray(A, dtype=np.float16)
    B = np.ascontiguousarray(B, dtype=np.float16)
    M, K = A.shape
    if b_col_major:
        N, Kb = B.shape
    else:
        Kb, N = B.shape
    if Kb != K:
        raise ValueError(f"inner dimensions differ: {K} vs {Kb}")
    C = np.zeros((M, N), dtype=np.float16)
    acc = np.zeros((M, N), dtype=np.float32) if want_acc else None
    rc = _load().oracle_gemm_f16(_ptr(A), _ptr(B), _ptr(C), _ptr(acc) if acc is not None else None,
                                 M, N, K, max(K, 1), B.shape[1] if B.ndim == 2 else 1, max(N, 1),
                                 1 if b_col_major else 0, int(threads))
    if rc != 0:
        raise RuntimeError("oracle_gemm_f16 failed")
    return C, acc


def parity_bound(ref: np.ndarray, K: int) -> float:
    """Allowed max |C - C_ref| for a K-deep product whose fp32 result is ref."""
    ref = np.asarray(ref, dtype=np.float64)
    rms = float(np.sqrt(np.mean(ref * ref))) if ref.size else 0.0
    return PARITY_COEFF * math.sqrt(max(K, 1)) * rms


def parity_report(C: np.ndarray, ref: np.ndarray, K: int) -> dict:
    C = np.asarray(C, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    err = float(np.max(np.abs(C - ref))) if C.size else 0.0
    bound = parity_bound(ref, K)
    return {"max_abs_err": err, "bound": bound, "ok": bool(err <= bound or (C.size and err == 0.0)),
            "finite": bool(np.all(np.isfinite(C)))}


def parity_ok(C: np.ndarray, ref: np.ndarray, K: int) -> bool:
    r = parity_report(C, ref, K)
    return r["ok"] and r["finite"]


def ref_kernels():
    """ctypes handle of the reference's CUDA kernels, or None if not built."""
    if not REF_LIB.exists():
        return None
    lib = ctypes.CDLL(str(REF_LIB))
    lib.ref_gemm_launch.restype = ctypes.c_int
    lib.ref_gemm_launch.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                    ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    return lib


# ---------------------------------------------------------------------------
# Seeded synthetic inputs of the hot path's configurations.  Generated on the
# CPU from torch.Generator seeds so every machine sees the same operands.
# ---------------------------------------------------------------------------
def make_inputs(M: int, N: int, K: int, dist: str = "uniform", seed_a: int = 0, seed_b: int = 1,
                std: float = 1.0):
    """Return (A, B) fp16 CPU torch tensors, A M x K and B K x N.

    dist "uniform": iid U[-1, 1); "normal": iid N(0, std^2).
    """
    import torch

    ga = torch.Generator().manual_seed(seed_a)
    gb = torch.Generator().manual_seed(seed_b)
    if dist == "uniform":
        A = torch.rand((M, K), generator=ga, dtype=torch.float32) * 2 - 1
        B = torch.rand((K, N), generator=gb, dtype=torch.float32) * 2 - 1
    elif dist == "normal":
        A = torch.randn((M, K), generator=ga, dtype=torch.float32) * std
        B = torch.randn((K, N), generator=gb, dtype=torch.float32) * std
    else:
        raise ValueError(dist)
    return A.half(), B.half()
