"""The B200 GEMM as a registered PyTorch operator with autograd.

`torch.ops.tensorcore_gemm.mm(A, B)` is C = A @ B (fp16 in, fp32 accumulate,
fp16 out) on the same sm_100a kernels as `tensorcore_gemm.gemm`.  Registering
it through `torch.library` makes it visible to the dispatcher: it has a fake
(meta) implementation, so `torch.compile` and other tracers see its output
shape without running it, and a backward formula, so it can sit inside a
model that is trained:

    dA = dC @ B^T      dB = A^T @ dC

Both gradients run on the same kernels; the transposes are views that the
launcher reads in place (B^T as a column-major second operand, A^T as a
column-major first operand), so the backward pass copies nothing.

The reference bound its kernels as a plain pybind function (load_inline in
tensorcore_gemm/cuda_compile.py:235-245, called from gemm.py:202-228), which
autograd and the tracers cannot see.  Like every entry of this package the
operator raises for inputs the kernels do not take (CPU tensors, other
dtypes); nothing falls back to another implementation.
"""
from __future__ import annotations

import torch

from .gemm import _check_operands, _launch


def _check(A: torch.Tensor, B: torch.Tensor) -> None:
    _check_operands(A, B)
    if A.shape[1] != B.shape[0]:
        raise RuntimeError("Inner dimensions must match")


@torch.library.custom_op("tensorcore_gemm::mm", mutates_args=())
def mm(A: torch.Tensor, B: torch.Tensor) -> torch.Tensor:
    """C = A @ B on the B200 kernels (A M x K, B K x N, both fp16 CUDA)."""
    _check(A, B)
    return _launch(A, B, False)


@mm.register_fake
def _mm_fake(A: torch.Tensor, B: torch.Tensor) -> torch.Tensor:
    _check(A, B)
    return A.new_empty((A.shape[0], B.shape[1]))


def _setup_context(ctx, inputs, output) -> None:
    A, B = inputs
    ctx.save_for_backward(A if ctx.needs_input_grad[1] else None, B if ctx.needs_input_grad[0] else None)


def _backward(ctx, grad: torch.Tensor):
    A, B = ctx.saved_tensors
    dA = mm(grad, B.t()) if ctx.needs_input_grad[0] else None
    dB = mm(A.t(), grad) if ctx.needs_input_grad[1] else None
    return dA, dB


mm.register_autograd(_backward, setup_context=_setup_context)
