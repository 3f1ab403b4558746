"""GPU: the allocation-free entry point b200_gemm_f16_noalloc.

Some callers cannot allocate device memory: their memory belongs to a host
framework's pool that forbids side allocations, or they sit on a latency
path that cannot afford cudaMalloc's implicit synchronisation.  For them the
library keeps a fixed scratch array and b200_gemm_f16_noalloc re-pitches odd
operands into it instead of into a caller workspace.  This file checks it
through the C ABI against the workspace entry point b200_gemm_f16_ws on two
calls in a row (different shapes, so the second call runs over the first
call's leftovers in the shared array), plus its size limit.  It is named so
pytest collects it last.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from gpu_util import assert_parity, fp32_ref
from oracle import oracle
from tensorcore_gemm import _native

pytestmark = pytest.mark.gpu

SCRATCH_LIMIT = 32 << 20


def _noalloc(lib):
    fn = lib.b200_gemm_f16_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int64] * 6 + [ctypes.c_int, ctypes.c_void_p]
    return fn


def _case(dev, M, N, K, ld_extra, colb, seed):
    """A with an odd row pitch (lda = K + ld_extra) and B row-major or col-major."""
    A0, B0 = oracle.make_inputs(M, N, K, dist="normal", seed_a=seed, seed_b=seed + 1)
    lda = K + ld_extra
    Abuf = torch.zeros((M, lda), dtype=torch.float16, device=dev)
    Abuf[:, :K] = A0.to(dev)
    Bop = (B0.t().contiguous() if colb else B0).to(dev)
    ldb = Bop.shape[1]
    return A0.to(dev), B0.to(dev), Abuf, lda, Bop, ldb


def _run_both(lib, dev, M, N, K, ld_extra, colb, seed):
    A, B, Abuf, lda, Bop, ldb = _case(dev, M, N, K, ld_extra, colb, seed)
    layout = _native.B200_B_COL_MAJOR if colb else _native.B200_B_ROW_MAJOR
    stream = torch.cuda.current_stream().cuda_stream
    C_ref = torch.empty((M, N), dtype=torch.float16, device=dev)
    args = (Abuf.data_ptr(), Bop.data_ptr(), C_ref.data_ptr(), M, N, K, lda, ldb, N, layout)
    need = _native.workspace_size(*args)
    assert 0 < need <= SCRATCH_LIMIT
    ws = torch.empty(need, dtype=torch.uint8, device=dev)
    assert _native.gemm_f16_ws_raw(*args, ws.data_ptr(), need, stream) == 0
    C = torch.full((M, N), float("nan"), dtype=torch.float16, device=dev)
    rc = _noalloc(lib)(Abuf.data_ptr(), Bop.data_ptr(), C.data_ptr(), M, N, K, lda, ldb, N, layout, stream)
    assert rc == 0, _native.strerror(rc)
    torch.cuda.synchronize()
    assert _native.last_device_error() == 0
    ref = fp32_ref(A, B)
    assert_parity(C_ref, ref, K, "workspace entry")
    assert_parity(C, ref, K, "no-alloc entry")
    # Same kernels, same inputs: within the tests' tolerance of each other.
    bound = oracle.PARITY_COEFF * K ** 0.5 * ref.pow(2).mean().sqrt().item()
    assert (C.float() - C_ref.float()).abs().max().item() <= bound


def test_noalloc_matches_workspace_entry_two_calls(cuda_device, native_lib):
    _run_both(native_lib, cuda_device, 300, 197, 131, 3, False, seed=61)
    _run_both(native_lib, cuda_device, 1000, 136, 77, 1, True, seed=71)


def test_noalloc_rejects_operands_beyond_scratch(cuda_device, native_lib):
    M, K = 17000, 1001                      # A re-pitched: 17000 x 1008 x 2 B = 34.3 MB > 32 MiB
    Abuf = torch.zeros((M, K), dtype=torch.float16, device=cuda_device)
    B = torch.zeros((K, 64), dtype=torch.float16, device=cuda_device)
    C = torch.empty((M, 64), dtype=torch.float16, device=cuda_device)
    rc = _noalloc(native_lib)(Abuf.data_ptr(), B.data_ptr(), C.data_ptr(), M, 64, K, K, 64, 64,
                              _native.B200_B_ROW_MAJOR, torch.cuda.current_stream().cuda_stream)
    assert rc == _native.B200_ERR_SCRATCH_LIMIT
    assert "32 MiB" in _native.strerror(rc)


@pytest.mark.parametrize("M,N,K,ld_extra", [
    (2560, 2048, 8192, 0),      # operands used in place; the pair kernel's last wave would split 4 ways
    (1024, 19200, 12288, 1),    # A re-pitched into the scratch (odd lda); last wave would split 6 ways
])
def test_noalloc_split_shapes_allocate_nothing(cuda_device, native_lib, M, N, K, ld_extra):
    """Shapes whose b200_gemm_f16 launch splits its last wave along K (that split
    keeps partial sums in a per-stream workspace allocated on first use) run
    whole through the no-alloc entry: device free memory does not move across
    calls on a stream that has never run a GEMM."""
    variant, ranges = _native.plan(M, N, K, torch.cuda.get_device_properties(cuda_device).multi_processor_count)
    assert variant == "pair" and ranges > 1, (variant, ranges)
    fn = _noalloc(native_lib)
    A0, B0 = oracle.make_inputs(M, N, K, dist="uniform", seed_a=M, seed_b=N)
    lda = K + ld_extra
    Abuf = torch.zeros((M, lda), dtype=torch.float16, device=cuda_device)
    Abuf[:, :K] = A0.to(cuda_device)
    B = B0.to(cuda_device)
    C = torch.empty((M, N), dtype=torch.float16, device=cuda_device)
    args = (Abuf.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, lda, N, N, _native.B200_B_ROW_MAJOR)
    # Warm-up on the current stream: the first launch of a kernel may load its code.
    assert fn(*args, torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    fresh = torch.cuda.Stream()
    free_before = torch.cuda.mem_get_info(cuda_device)[0]
    for _ in range(2):
        assert fn(*args, fresh.cuda_stream) == 0
    torch.cuda.synchronize()
    free_after = torch.cuda.mem_get_info(cuda_device)[0]
    assert free_after == free_before, f"device free memory moved by {free_before - free_after} bytes"
    assert _native.last_device_error() == 0
    A, Bd = A0.to(cuda_device), B0.to(cuda_device)
    assert_parity(C, fp32_ref(A, Bd), K, f"no-alloc {M}x{N}x{K}")
