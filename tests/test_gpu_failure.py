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
