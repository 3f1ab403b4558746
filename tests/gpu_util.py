"""Helpers shared by the GPU tests: oracle references and parity asserts."""
from __future__ import annotations

import numpy as np
import torch

from oracle import oracle


def fp32_ref(A: torch.Tensor, B: torch.Tensor, b_col_major: bool = False) -> torch.Tensor:
    """fp32 product of the fp16 operands, computed on the GPU without TF32."""
    Bf = B.float().t() if b_col_major else B.float()
    return A.float() @ Bf


def assert_parity(C: torch.Tensor, ref: torch.Tensor, K: int, what: str = "") -> None:
    """max|C - ref| <= 2e-3 * sqrt(K) * RMS(ref); ref is fp32."""
    assert C.dtype == torch.float16
    Cf = C.float()
    assert torch.isfinite(Cf).all(), f"{what}: non-finite output"
    err = (Cf - ref).abs().max().item() if C.numel() else 0.0
    rms = ref.double().pow(2).mean().sqrt().item() if ref.numel() else 0.0
    bound = oracle.PARITY_COEFF * max(K, 1) ** 0.5 * rms
    assert err <= bound, f"{what}: max|err| {err:.4g} > bound {bound:.4g} (K={K}, rms={rms:.4g})"


def oracle_check(C: torch.Tensor, A: torch.Tensor, B: torch.Tensor, b_col_major: bool = False) -> None:
    """Compare a GPU result with the C oracle (small sizes only)."""
    Co, acc = oracle.gemm_f16(A.cpu().numpy(), B.cpu().numpy(), b_col_major=b_col_major, threads=8)
    K = A.shape[1]
    rep = oracle.parity_report(C.cpu().numpy(), acc, K)
    assert rep["finite"] and rep["ok"], f"oracle parity failed: {rep}"
