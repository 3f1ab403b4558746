"""B200-native drop-in for the reference ``tensorcore_gemm`` package.

Public surface identical to the reference (tensorcore_gemm/__init__.py:1-3).
"""
from .gemm import KERNEL_MODES, gemm, gemm_pretransposed, is_supported

__all__ = ["KERNEL_MODES", "gemm", "gemm_pretransposed", "is_supported"]
