"""K-means assignment step on the B200 skinny GEMM, with the argmin fused.

The reference benchmarks its K = 256 shapes as "K-means-like" (points x
centroids^T, README.md:44) but stops at the fp16 product; a K-means step then
needs an argmin over that M x N product.  `assign` computes it inside the
GEMM's epilogue, so the M x N matrix is never written to HBM.
"""
from __future__ import annotations

import torch

from . import _native


def _pitched(t: torch.Tensor) -> torch.Tensor:
    """`t` with unit column stride and a 16-byte aligned base and row pitch
    (TMA's rule), copied into such a buffer only when it is not already."""
    if t.stride(1) == 1 and t.stride(0) % 8 == 0 and t.data_ptr() % 16 == 0 and t.stride(0) >= t.shape[1]:
        return t
    rows, cols = t.shape
    buf = torch.empty((rows, -(-cols // 8) * 8), dtype=t.dtype, device=t.device)
    buf[:, :cols].copy_(t)
    return buf[:, :cols]


def assign(X: torch.Tensor, centroids: torch.Tensor, centroids_kn: bool = False,
           return_scores: bool = False):
    """Nearest centroid for every point.

    X: M x K fp16 CUDA (points).  centroids: N x K fp16 CUDA (one centroid
    per row), or K x N when `centroids_kn`.  1 <= K <= 256.  Returns int32
    indices (M,), and with `return_scores` also the fp32 scores
    ||c||^2 - 2 x.c of the winners (add ||x||^2 for squared distances).
    Ties go to the smaller index.
    """
    for name, t in (("X", X), ("centroids", centroids)):
        if not (isinstance(t, torch.Tensor) and t.is_cuda and t.dtype == torch.float16 and t.dim() == 2):
            raise RuntimeError(f"{name} must be a 2-D float16 CUDA tensor")
    M, K = X.shape
    if centroids_kn:
        Kc, N = centroids.shape
        layout = _native.B200_B_ROW_MAJOR
    else:
        N, Kc = centroids.shape
        layout = _native.B200_B_COL_MAJOR
    if Kc != K:
        raise RuntimeError("Inner dimensions must match")
    X = _pitched(X)
    centroids = _pitched(centroids)
    idx = torch.empty(M, dtype=torch.int32, device=X.device)
    scores = torch.empty(M, dtype=torch.float32, device=X.device) if return_scores else None
    lib = _native.load()
    ws_bytes = lib.b200_kmeans_workspace_size(M, N)
    if ws_bytes < 0:
        _native.check(-ws_bytes, "b200_kmeans_workspace_size")
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=X.device)
    with torch.cuda.device(X.device):
        code = lib.b200_kmeans_assign_f16(
            X.data_ptr(), centroids.data_ptr(), M, N, K, X.stride(0), centroids.stride(0), layout,
            ws.data_ptr(), ws_bytes, idx.data_ptr(), scores.data_ptr() if scores is not None else None,
            torch.cuda.current_stream(X.device).cuda_stream)
    _native.check(code, "b200_kmeans_assign_f16")
    return (idx, scores) if return_scores else idx
