"""CPU: the C-ABI library loads, exports every declared symbol, and rejects
bad arguments before touching the GPU."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
HEADERS = sorted((REPO / "include").glob("*.h"))


def _declared_symbols():
    names = []
    for h in HEADERS:
        text = h.read_text()
        names += re.findall(r"B200_API\s+[\w\s\*]+?\b(\w+)\s*\(", text)
    return names


def test_header_declares_entry_points():
    names = _declared_symbols()
    assert "b200_gemm_f16" in names and "b200_gemm_strerror" in names
    assert len(names) == len(set(names))


def test_library_exports_every_declared_symbol(native_lib):
    for name in _declared_symbols():
        assert hasattr(native_lib, name), f"{name} declared in include/ but not exported"


def test_version_and_strerror(native_lib):
    from tensorcore_gemm import _native

    assert _native.version() >= 100
    for code in range(0, 8):
        assert _native.strerror(code)
    assert "unknown" in _native.strerror(999)


@pytest.mark.parametrize("args,code", [
    # (M, N, K, lda, ldb, ldc, layout)
    ((-1, 8, 8, 8, 8, 8, 0), 1),
    ((8, -1, 8, 8, 8, 8, 0), 1),
    ((8, 8, -1, 8, 8, 8, 0), 1),
    ((8, 8, 8, 8, 8, 8, 2), 1),
    ((1 << 31, 8, 8, 8, 8, 8, 0), 3),
    ((0, 8, 8, 8, 8, 8, 0), 0),   # empty output: nothing to do
    ((8, 0, 8, 8, 8, 8, 1), 0),
])
def test_argument_validation_without_gpu(native_lib, args, code):
    from tensorcore_gemm import _native

    M, N, K, lda, ldb, ldc, layout = args
    got = _native.gemm_f16_raw(0, 0, 0, M, N, K, lda, ldb, ldc, layout, 0)
    assert got == code


def test_null_output_rejected(native_lib):
    from tensorcore_gemm import _native

    assert _native.gemm_f16_raw(16, 16, 0, 8, 8, 8, 8, 8, 8, 0, 0) == _native.B200_ERR_INVALID_ARGUMENT


def test_misaligned_output_rejected(native_lib):
    from tensorcore_gemm import _native

    buf = ctypes.create_string_buffer(4096)
    base = (ctypes.addressof(buf) + 15) & ~15
    assert _native.gemm_f16_raw(base, base, base + 2, 8, 8, 8, 8, 8, 8, 0, 0) == _native.B200_ERR_MISALIGNED
    assert _native.gemm_f16_raw(base, base, base, 8, 8, 8, 8, 8, 12, 0, 0) == _native.B200_ERR_MISALIGNED
    assert _native.gemm_f16_raw(base, base, base, 8, 12, 8, 8, 8, 8, 0, 0) == _native.B200_ERR_INVALID_ARGUMENT


def test_set_variant_validation(native_lib):
    from tensorcore_gemm import _native

    assert native_lib.b200_gemm_set_variant(99) == _native.B200_ERR_INVALID_ARGUMENT
    assert native_lib.b200_gemm_set_variant(-1) == _native.B200_ERR_INVALID_ARGUMENT
    for v in ("pair", "cta1", "auto"):
        _native.set_variant(v)


def test_workspace_size_plan(native_lib):
    """Host-side workspace arithmetic: 16-byte pitches, 256-byte aligned parts."""
    from tensorcore_gemm import _native

    A, B, C = 0x10000, 0x20000, 0x30000          # aligned fake addresses (never dereferenced)
    ws = lambda *a: native_lib.b200_gemm_workspace_size(*a)
    assert ws(A, B, C, 64, 64, 64, 64, 64, 64, 0) == 0                 # nothing to re-pitch
    assert ws(A, B, C, 10, 16, 7, 7, 16, 16, 0) == 256                  # A: 10 x 8 x 2 = 160 -> 256
    assert ws(A, B, C, 10, 17, 16, 16, 17, 17, 0) == 768 + 512          # B 16x24x2=768; C 10x24x2=480 -> 512
    # B col-major N x K with odd K: both A and B re-pitched
    assert ws(A, B, C, 4, 8, 9, 9, 9, 8, 1) == 256 + 256
    assert ws(A + 2, B, C, 4, 8, 8, 8, 8, 8, 0) == 256                  # misaligned base only
    assert ws(A, B, C, 0, 8, 8, 8, 8, 8, 0) == 0                        # empty output
    assert ws(A, B, C, 4, 8, 8, 4, 8, 8, 0) == -_native.B200_ERR_INVALID_ARGUMENT   # lda < K


def test_gather_argument_validation_without_gpu(native_lib):
    """Checks of b200_gemm_f16_gather that come before any CUDA call."""
    from tensorcore_gemm import _native

    buf = ctypes.create_string_buffer(4096)
    base = (ctypes.addressof(buf) + 15) & ~15
    assert _native.gemm_gather_raw(base, base, base, 8, 8, 8, 8, 8, 8, 0, [base] * 8, 0) == \
        _native.B200_ERR_INVALID_ARGUMENT                                   # more than 7 peers
    assert _native.gemm_gather_raw(base, base, base, 8, 8, 8, 8, 8, 8, 0, [0], 0) == \
        _native.B200_ERR_INVALID_ARGUMENT                                   # null peer
    assert _native.gemm_gather_raw(base, base, base, 8, 8, 8, 8, 8, 8, 0, [base + 8], 0) == \
        _native.B200_ERR_MISALIGNED                                         # peer not 16-byte aligned
    assert _native.gemm_gather_raw(base, base, base, 0, 8, 8, 8, 8, 8, 0, [base], 0) == _native.B200_OK
    lib = _native.load()
    assert lib.b200_ipc_handle_size() == 64
    ptr = ctypes.c_void_p()
    assert lib.b200_ipc_alloc(0, ctypes.byref(ptr), buf) == _native.B200_ERR_INVALID_ARGUMENT
    assert lib.b200_ipc_open(None, ctypes.byref(ptr)) == _native.B200_ERR_INVALID_ARGUMENT
    assert lib.b200_ipc_close(None) == _native.B200_OK and lib.b200_ipc_free(None) == _native.B200_OK


@pytest.mark.parametrize("shape,variant,ranges", [
    ((65536, 8192, 8192), "pair2m", 1),   # bench workload, 1 GPU
    ((8192, 8192, 8192), "pair2m", 1),    # its shard at 8 GPUs
    ((32768, 1024, 256), "skinny", 1),    # K = 256, many tiles per SM
    ((16384, 256, 256), "cta1", 1),       # K = 256, too few tiles for the B-stationary kernel
    ((2048, 2048, 2048), "cta1", 1),      # one wave of 1-CTA tiles
    ((200, 264, 136), "cta1", 1),         # K < 512
    ((2560, 2048, 8192), "pair", 4),      # partial last wave, deep K: split 4 ways
    ((4096, 4096, 16384), "pair", 2),     # partial last wave, deep K: split 2 ways
    ((2560, 2048, 2048), "pair2m_192", 1),  # one wave of 55 tiles 192 wide (256 wide: 40 tiles on 80 SMs)
    ((4000, 6000, 3000), "pair2m", 1),    # narrower wide-pair tiles would not save a wave
    ((4096, 8192, 4096), "pair", 1),
    ((3072, 3072, 3072), "pair2m", 1),    # one wave of wide tiles against two of the pair kernel
    ((1536, 1280, 8192), "pair", 1),      # one wave, deep K: the pair kernel, not the 1-CTA one
])
def test_launch_plan(native_lib, shape, variant, ranges):
    """The kernel choice (wave model) and last-wave split, computed on the host."""
    from tensorcore_gemm import _native

    assert _native.plan(*shape, sm_count=148) == (variant, ranges)


def test_launch_plan_forced_variant_and_errors(native_lib):
    from tensorcore_gemm import _native

    _native.set_variant("pair")
    try:
        assert _native.plan(4096, 4096, 16384) == ("pair", 2)
        assert _native.plan(4096, 4096, 4096)[0] == "pair"
    finally:
        _native.set_variant("auto")
    _native.set_variant("skinny")
    try:
        assert _native.plan(4096, 4096, 4096) == ("cta1", 1)    # outside the skinny kernel's K range
    finally:
        _native.set_variant("auto")
    with pytest.raises(RuntimeError):
        _native.plan(0, 8, 8)
