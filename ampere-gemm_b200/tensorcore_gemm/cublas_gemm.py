"""cuBLAS comparator, mirroring the reference's ``tensorcore_gemm.cublas_gemm``.

The reference wrapped ``cublasGemmEx`` (fp16 in/out, fp32 compute) in its own
extension (tensorcore_gemm/cublas_gemm.py:29-43, cublas_gemm.cu:7-62).  Here
the same library GEMM is reached through ``torch.mm`` on fp16 CUDA tensors,
which calls cuBLAS with fp32 accumulation.  This module is a measurement
comparator only; nothing on the product path imports it.
"""
from __future__ import annotations

import torch


def gemm(A: torch.Tensor, B: torch.Tensor) -> torch.Tensor:
    if A.ndim != 2 or B.ndim != 2:
        raise RuntimeError("A and B must be 2D")
    if A.shape[1] != B.shape[0]:
        raise ValueError("Inner dimensions must match.")
    if not (A.is_cuda and B.is_cuda) or A.dtype != torch.float16 or B.dtype != torch.float16:
        raise RuntimeError("cublas comparator expects float16 CUDA tensors")
    return torch.mm(A, B)
