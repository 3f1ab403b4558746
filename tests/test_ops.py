"""The registered operator torch.ops.tensorcore_gemm.mm: shape propagation
without a GPU (fake tensors), loud failure on CPU tensors, and on the GPU
forward and backward parity with the fp32 products."""
from __future__ import annotations

import pytest
import torch

import tensorcore_gemm  # noqa: F401  (registers the operator)
from oracle import oracle


def test_operator_is_registered():
    assert hasattr(torch.ops.tensorcore_gemm, "mm")


def test_fake_tensor_shapes_without_gpu():
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode(allow_non_fake_inputs=False) as mode:
        A = torch.empty((300, 136), dtype=torch.float16, device="cuda")
        B = torch.empty((136, 72), dtype=torch.float16, device="cuda")
        C = torch.ops.tensorcore_gemm.mm(A, B)
        assert tuple(C.shape) == (300, 72) and C.dtype == torch.float16
        with pytest.raises(RuntimeError, match="Inner dimensions"):
            torch.ops.tensorcore_gemm.mm(A, B.t())
    del mode


def test_cpu_tensors_raise():
    A = torch.zeros((8, 8), dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        torch.ops.tensorcore_gemm.mm(A, A)


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(256, 512, 320), (300, 136, 1000), (2048, 2048, 2048)])
def test_forward_and_backward_parity(cuda_device, native_lib, M, N, K):
    A0, B0 = oracle.make_inputs(M, N, K, dist="normal", seed_a=M, seed_b=N, std=0.1)
    A = A0.to(cuda_device).requires_grad_()
    B = B0.to(cuda_device).requires_grad_()
    G = (torch.randn((M, N), generator=torch.Generator().manual_seed(K)) * 0.1).half().to(cuda_device)
    C = torch.ops.tensorcore_gemm.mm(A, B)
    C.backward(G)
    torch.cuda.synchronize()
    Af, Bf, Gf = A.detach().float(), B.detach().float(), G.float()
    for got, ref, depth, what in ((C, Af @ Bf, K, "C"), (A.grad, Gf @ Bf.t(), N, "dA"), (B.grad, Af.t() @ Gf, M, "dB")):
        err = (got.float() - ref).abs().max().item()
        bound = oracle.PARITY_COEFF * depth ** 0.5 * ref.pow(2).mean().sqrt().item()
        assert err <= bound, f"{what}: {err} > {bound}"


@pytest.mark.gpu
def test_opcheck(cuda_device, native_lib):
    A0, B0 = oracle.make_inputs(128, 256, 64, dist="normal", seed_a=1, seed_b=2)
    A, B = A0.to(cuda_device).requires_grad_(), B0.to(cuda_device).requires_grad_()
    torch.library.opcheck(torch.ops.tensorcore_gemm.mm, (A, B),
                          test_utils=("test_schema", "test_faketensor", "test_aot_dispatch_static"))
