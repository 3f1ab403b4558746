"""B200-native drop-in for the reference ``tensorcore_gemm`` package.

Public surface identical to the reference (tensorcore_gemm/__init__.py:1-3).
Importing the package also registers ``torch.ops.tensorcore_gemm.mm`` (the
same GEMM as a dispatcher operator with autograd, see ``ops``).
"""
from . import ops as _ops  # noqa: F401  (registers torch.ops.tensorcore_gemm.mm)
from .gemm import KERNEL_MODES, gemm, gemm_pretransposed, is_supported

__all__ = ["KERNEL_MODES", "gemm", "gemm_pretransposed", "is_supported"]
