"""GPU: the bounded-wait failure path, exercised without faulting the GPU.

A one-thread kernel waits on an mbarrier that nothing arrives at, with a
10 ms limit; it must give up, leave cause 5 in the device error word and
return, after which the context still runs GEMMs correctly.
"""
from __future__ import annotations

import pytest
import torch

import tensorcore_gemm as tg
from gpu_util import assert_parity, fp32_ref
from oracle import oracle
from tensorcore_gemm import _native

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_and_recovers(cuda_device, native_lib):
    assert _native.selftest_bounded_wait(10_000_000) == 5
    assert _native.last_device_error() == 0          # the self-test cleared the word
    A, B = oracle.make_inputs(256, 512, 320, seed_a=41, seed_b=42)
    A, B = A.to(cuda_device), B.to(cuda_device)
    C = tg.gemm(A, B)
    torch.cuda.synchronize()
    assert _native.last_device_error() == 0
    assert_parity(C, fp32_ref(A, B), 320)


def test_selftest_rejects_bad_limits(native_lib):
    assert _native.selftest_bounded_wait(0) < 0
    assert _native.selftest_bounded_wait(5_000_000_000) < 0


def test_split_fixup_timeout_leaves_tail_tiles_unstored(cuda_device, native_lib):
    """The last K range of a split tile gives up on a part that never arrives:
    the tile is not stored, cause 6 is reported, and the next GEMM is right."""
    M, N, K = 2560, 2048, 8192           # 80 tiles of 256 x 256: 74 whole, 6 split 4 ways
    A, B = oracle.make_inputs(M, N, K, seed_a=51, seed_b=52)
    A, B = A.to(cuda_device), B.to(cuda_device)
    C = torch.full((M, N), float("nan"), dtype=torch.float16, device=cuda_device)
    word = _native.selftest_split_fixup(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, 2_000_000,
                                        torch.cuda.current_stream().cuda_stream)
    assert word == 6
    assert _native.last_device_error() == 0          # the self-test cleared the word
    unstored = torch.isnan(C)
    assert int(unstored.sum()) == 6 * 256 * 256      # exactly the six split tiles
    ref = fp32_ref(A, B)
    stored = ~unstored
    assert_parity(C[stored].view(1, -1), ref[stored].view(1, -1), K, "tiles stored before the timeout")
    # The tail counters were reset: the same split launch now completes.
    _native.set_variant("pair")
    try:
        C2 = tg.gemm(A, B)
        torch.cuda.synchronize()
    finally:
        _native.set_variant("auto")
    assert _native.last_device_error() == 0
    assert_parity(C2, ref, K, "split launch after the fixup timeout")


def test_split_fixup_selftest_rejects_unsplit_shapes(cuda_device, native_lib):
    A = torch.zeros((256, 512), dtype=torch.float16, device=cuda_device)
    B = torch.zeros((512, 256), dtype=torch.float16, device=cuda_device)
    C = torch.empty((256, 256), dtype=torch.float16, device=cuda_device)
    assert _native.selftest_split_fixup(A.data_ptr(), B.data_ptr(), C.data_ptr(), 256, 256, 512) \
        == -_native.B200_ERR_INVALID_ARGUMENT
