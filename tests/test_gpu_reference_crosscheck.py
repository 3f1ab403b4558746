"""GPU cross-checks against the reference's own kernels and cuBLAS.

The reference's reg_pingpong_256* kernels are built from its sources into
oracle/_ref/libref_gemm.so (oracle/Makefile) and run on the same inputs; both
they and the B200 kernels must meet the acceptance bound against the fp32
product, and must agree with each other within twice that bound.
"""
from __future__ import annotations

import pytest
import torch

import tensorcore_gemm as tg
from gpu_util import assert_parity, fp32_ref
from oracle import oracle
from tensorcore_gemm import cublas_gemm

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref_lib():
    lib = oracle.ref_kernels()
    if lib is None:
        pytest.fail("oracle/_ref/libref_gemm.so is missing: build it with `make -C oracle ref`")
    return lib


def _run_ref(lib, A, Bop, M, N, K, mode):
    C = torch.empty((M, N), dtype=torch.float16, device=A.device)
    rc = lib.ref_gemm_launch(A.data_ptr(), Bop.data_ptr(), C.data_ptr(), M, N, K, mode,
                             torch.cuda.current_stream().cuda_stream)
    assert rc == 0, f"reference launch failed ({rc})"
    torch.cuda.synchronize()
    return C


@pytest.mark.parametrize("M,N,K", [(2048, 2048, 2048), (4096, 4096, 4096), (16384, 1024, 256), (512, 256, 64)])
def test_against_reference_kernels(cuda_device, native_lib, ref_lib, M, N, K):
    A, B = oracle.make_inputs(M, N, K, dist="normal", seed_a=1, seed_b=2)
    A, B = A.to(cuda_device), B.to(cuda_device)
    Bc = B.t().contiguous()
    ref = fp32_ref(A, B)
    ours_row = tg.gemm(A, B, mode="reg_pingpong_256")
    ours_col = tg.gemm_pretransposed(A, Bc, mode="reg_pingpong_256_colb")
    assert_parity(ours_row, ref, K, "b200 rowB")
    assert_parity(ours_col, ref, K, "b200 colb")
    bound = oracle.PARITY_COEFF * K ** 0.5 * ref.pow(2).mean().sqrt().item()
    for mode, Bop in ((2, B), (3, B), (4, Bc), (5, Bc)):
        C_ref_kernel = _run_ref(ref_lib, A, Bop, M, N, K, mode)
        assert_parity(C_ref_kernel, ref, K, f"reference mode {mode}")
        diff = (C_ref_kernel.float() - ours_row.float()).abs().max().item()
        assert diff <= 2 * bound, f"b200 vs reference mode {mode}: {diff} > {2 * bound}"


@pytest.mark.parametrize("M,N,K", [(2048, 2048, 2048), (8192, 8192, 8192), (32768, 1024, 256), (4000, 6000, 3000)])
def test_against_cublas(cuda_device, native_lib, M, N, K):
    torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
    A, B = oracle.make_inputs(M, N, K, dist="uniform", seed_a=3, seed_b=4)
    A, B = A.to(cuda_device), B.to(cuda_device)
    ref = fp32_ref(A, B)
    ours = tg.gemm(A, B)
    lib = cublas_gemm.gemm(A, B)
    assert_parity(ours, ref, K, "b200")
    assert_parity(lib, ref, K, "cublas")


@pytest.fixture(scope="module")
def reference_cublas():
    """The reference's own cuBLAS mode from the unmodified package in
    baseline/_ref (cublas_gemm.py:29-43 over cublas_gemm.cu:7-62), built by
    the reference's own JIT path on first use."""
    from baseline import reference

    mod = reference.cublas_module()
    if mod is None:
        pytest.fail("baseline/_ref is not installed: run `python baseline/install_reference.py`")
    return mod


@pytest.mark.parametrize("M,N,K", [(2048, 2048, 2048), (8192, 8192, 8192), (32768, 1024, 256), (4096, 8192, 4096)])
def test_against_reference_cublas_mode(cuda_device, native_lib, reference_cublas, M, N, K):
    A, B = oracle.make_inputs(M, N, K, dist="uniform", seed_a=5, seed_b=6)
    A, B = A.to(cuda_device), B.to(cuda_device)
    ref = fp32_ref(A, B)
    ours = tg.gemm(A, B)
    theirs = reference_cublas.gemm(A, B)
    torch.cuda.synchronize()
    assert_parity(ours, ref, K, "b200")
    assert_parity(theirs, ref, K, "reference cublas_gemm")
    bound = oracle.PARITY_COEFF * K ** 0.5 * ref.pow(2).mean().sqrt().item()
    diff = (theirs.float() - ours.float()).abs().max().item()
    assert diff <= 2 * bound, f"b200 vs reference cublas_gemm: {diff} > {2 * bound}"
