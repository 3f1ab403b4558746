"""GPU, one device: the gathered-output GEMM (b200_gemm_f16_gather).

On one GPU the "peers" are further buffers on the same device; the epilogue
writes them exactly as it writes another GPU's copy (plain 16-byte stores),
so every store path, edge clip and variant is covered without a second GPU.
Each copy must hold the shard's rows bit-identical to the local output, the
local output must meet the parity bar, and every byte outside the shard must
keep its guard value.
"""
from __future__ import annotations

import pytest
import torch

from gpu_util import assert_parity, fp32_ref

pytestmark = pytest.mark.gpu

GUARD = 0x7BFF  # fp16 65504: never produced by these products


@pytest.fixture(params=["auto", "cta1", "pair", "skinny", "pair2m", "pair2m_224", "pair2m_192"])
def variant(request, native_lib):
    from tensorcore_gemm import _native

    _native.set_variant(request.param)
    yield request.param
    _native.set_variant("auto")


def _gathered(M_total, row0, M, N, K, n_peers, b_col_major, seed):
    from tensorcore_gemm import _native

    g = torch.Generator(device="cuda").manual_seed(seed)
    A = (torch.randn((M, K), device="cuda", generator=g) * 0.5).half()
    B = (torch.randn((N, K) if b_col_major else (K, N), device="cuda", generator=g) * 0.5).half()
    ldc = -(-N // 8) * 8
    bufs = [torch.full((M_total, ldc), GUARD, dtype=torch.int16, device="cuda") for _ in range(n_peers + 1)]
    ptrs = [b.data_ptr() + row0 * ldc * 2 for b in bufs]
    stream = torch.cuda.current_stream().cuda_stream
    code = _native.gemm_gather_raw(A.data_ptr(), B.data_ptr(), ptrs[0], M, N, K, K,
                                   K if b_col_major else N, ldc,
                                   _native.B200_B_COL_MAJOR if b_col_major else _native.B200_B_ROW_MAJOR,
                                   ptrs[1:], stream)
    torch.cuda.synchronize()
    return code, A, B, bufs, ldc


def _check(bufs, A, B, row0, M, N, K, b_col_major):
    from tensorcore_gemm import _native

    local = bufs[0]
    C = local[row0:row0 + M, :N].view(torch.float16)
    assert_parity(C, fp32_ref(A, B, b_col_major), K, "gathered local")
    for i, b in enumerate(bufs[1:]):
        assert torch.equal(b, local), f"peer copy {i} differs from the local output"
    outside = torch.ones_like(local, dtype=torch.bool)
    outside[row0:row0 + M, :N] = False
    assert (local[outside] == GUARD).all(), "a store landed outside the shard"
    assert _native.last_device_error() == 0


@pytest.mark.parametrize("M,N,K,b_col_major", [
    (1000, 264, 512, False),       # ragged rows, pair kernels' partial waves
    (517, 1000, 1024, True),
    (4096, 1024, 256, False),      # skinny-kernel shape under auto
    (300, 136, 64, True),
    (256, 2048, 2048, False),
])
def test_gather_matches_local_and_parity(variant, M, N, K, b_col_major):
    row0 = 256
    code, A, B, bufs, _ = _gathered(M + 2 * row0, row0, M, N, K, 3, b_col_major, seed=M + N + K)
    assert code == 0
    _check(bufs, A, B, row0, M, N, K, b_col_major)


def test_gather_ragged_columns(native_lib):
    """N not a multiple of 8: the last 16-byte segment of each row is written element-wise."""
    from tensorcore_gemm import _native

    M, N, K, row0 = 333, 1001, 264, 128
    g = torch.Generator(device="cuda").manual_seed(5)
    A = (torch.randn((M, K), device="cuda", generator=g) * 0.5).half()
    Bbuf = torch.zeros((K, 1008), dtype=torch.float16, device="cuda")
    Bbuf[:, :N] = (torch.randn((K, N), device="cuda", generator=g) * 0.5).half()
    B = Bbuf[:, :N]
    ldc = 1008
    bufs = [torch.full((M + 2 * row0, ldc), GUARD, dtype=torch.int16, device="cuda") for _ in range(8)]
    ptrs = [b.data_ptr() + row0 * ldc * 2 for b in bufs]
    code = _native.gemm_gather_raw(A.data_ptr(), B.data_ptr(), ptrs[0], M, N, K, K, 1008, ldc, 0, ptrs[1:],
                                   torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert code == 0
    _check(bufs, A, B, row0, M, N, K, False)


def test_gather_empty_reduction_zeros_every_copy(native_lib):
    from tensorcore_gemm import _native

    M, N, row0 = 77, 40, 16
    bufs = [torch.full((M + 2 * row0, N), GUARD, dtype=torch.int16, device="cuda") for _ in range(3)]
    ptrs = [b.data_ptr() + row0 * N * 2 for b in bufs]
    code = _native.gemm_gather_raw(0, 0, ptrs[0], M, N, 0, 8, N, N, 0, ptrs[1:],
                                   torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert code == 0
    for b in bufs:
        assert (b[row0:row0 + M] == 0).all()
        assert (b[:row0] == GUARD).all() and (b[row0 + M:] == GUARD).all()


def test_gather_rejects_repitch_and_bad_peers(native_lib):
    from tensorcore_gemm import _native

    A = torch.zeros((64, 36), dtype=torch.float16, device="cuda")     # K = 36: pitch not a multiple of 8
    B = torch.zeros((36, 64), dtype=torch.float16, device="cuda")
    C = torch.zeros((64, 64), dtype=torch.float16, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert _native.gemm_gather_raw(A.data_ptr(), B.data_ptr(), C.data_ptr(), 64, 64, 36, 36, 64, 64, 0, [],
                                   s) == _native.B200_ERR_MISALIGNED
    assert _native.gemm_gather_raw(A.data_ptr(), B.data_ptr(), C.data_ptr(), 64, 64, 32, 32, 64, 64, 0,
                                   [C.data_ptr() + 2], s) == _native.B200_ERR_MISALIGNED


def test_ipc_alloc_roundtrip_in_process(native_lib):
    """Allocation and handle export work; the buffer is usable as a torch tensor through the wrapper."""
    from tensorcore_gemm import _native, sharded

    ptr, handle = _native.ipc_alloc(4096 * 2)
    assert len(handle) == _native.load().b200_ipc_handle_size() and ptr % 256 == 0
    t = torch.as_tensor(sharded._DeviceBuffer(ptr, 64, 64), device="cuda")
    t.fill_(1.5)
    assert t.float().sum().item() == 1.5 * 4096
    del t
    torch.cuda.synchronize()
    _native.ipc_free(ptr)
