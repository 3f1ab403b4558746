"""Drop-in ``tensorcore_gemm`` API on B200 tcgen05 kernels.

Same public names, arguments and mode strings as the reference package
(tensorcore_gemm/__init__.py:1-3, gemm.py:9-29, 166-228):

    gemm(A, B, mode="wmma")                       C = A @ B, B row-major K x N
    gemm_pretransposed(A, B_col_major, mode=...)  C = A @ B_col_major.T
    is_supported(A, B)                            can `gemm` run A, B natively?
    KERNEL_MODES                                  the six mode strings

Every mode runs the same sm_100a kernel family through the C ABI
(include/b200_gemm.h); the mode only selects how the second operand is laid
out, exactly as the reference's mode ids did (row-major B for ids 0-3 via
`gemm`, col-major B for 4/5 and for everything that goes through
`gemm_pretransposed` except ids 2/3, see below).  Numerics are fp16 inputs,
fp32 accumulation, one round-to-nearest-even to fp16.

Differences from the reference, all deliberate:
  * No silent fallback.  The reference returned ``torch.matmul(A, B)`` for any
    input it could not run (gemm.py:219-221), on CPU too.  Here unsupported
    inputs raise ``RuntimeError``; nothing computes on the CPU.
  * Any M, N, K is accepted (TMA zero fill / clipped stores; operands whose
    row pitch is not 16-byte aligned are re-pitched through a workspace on
    the GPU), not only M % 256 == N % 128 == K % 32 == 0 with K >= 64
    (gemm.py:185-192).
  * ``gemm`` in a colb mode does not transpose B first (gemm.py:227-228): the
    kernel reads row-major B with an MN-major shared-memory descriptor, which
    gives the same product without the extra HBM pass.
  * Modes "wmma" and "mma" work (the reference's build of them failed, since
    gemm.cu has no ``gemm_cuda`` launcher, gemm.py:195-199).
  * Kernels run on the current torch CUDA stream, not the legacy default
    stream (reference launches at gemm.py:82, 103, 122, 141).
"""
from __future__ import annotations

import torch

from . import _native

KERNEL_MODES = (
    "wmma",
    "mma",
    "reg_pingpong_256",
    "reg_pingpong_256_mma",
    "reg_pingpong_256_colb",
    "reg_pingpong_256_colb_mma",
)

_MODE_TO_ID = {name: i for i, name in enumerate(KERNEL_MODES)}
_F16 = torch.float16

# Mode ids whose `gemm_pretransposed` operand is read as row-major K x N.  In
# the reference, gemm_pretransposed(A, X, mode) with ids 2/3 called
# root_gemm_cuda(A, X, id) with use_colb = false (gemm.py:43, 215-216), so X is
# a row-major K x N B despite the function's name; ids 0/1/4/5 read X as the
# N x K (col-major) B that `gemm` builds for them (gemm.py:227-228).
_PRETRANSPOSED_ROW_MAJOR_IDS = frozenset({2, 3})

# TMA needs 16-byte aligned bases and row pitches: 8 fp16 elements.
_ALIGN_ELEMS = 8


def _normalize_mode(mode: str) -> int:
    """Mode string -> id; same error as the reference (gemm.py:166-170)."""
    try:
        return _MODE_TO_ID[mode]
    except (KeyError, TypeError) as exc:
        raise ValueError(f"Unsupported mode {mode!r}. Expected one of {KERNEL_MODES}.") from exc


def _row_view(t: torch.Tensor) -> tuple[torch.Tensor, int]:
    """Return (tensor, leading dimension) with unit inner stride.

    Row-strided views (e.g. a column slice) are used in place; anything else
    is made contiguous first, as the reference always did (gemm.py:213-225).
    """
    if t.stride(1) == 1 and t.stride(0) >= max(1, t.size(1)):
        return t, t.stride(0)
    t = t.contiguous()
    return t, max(1, t.size(1))


def is_supported(A: torch.Tensor, B: torch.Tensor) -> bool:
    """True when ``gemm(A, B)`` runs on the B200 kernels.

    Reference predicate: gemm.py:173-192.  The tile-multiple and contiguity
    conditions are gone (TMA zero fill, clipped stores, strided views, and a
    re-pitching workspace for odd K/N); what remains is CUDA, fp16, 2-D, one
    device and a matching inner dimension.
    """
    if not (isinstance(A, torch.Tensor) and isinstance(B, torch.Tensor)):
        return False
    if not (A.is_cuda and B.is_cuda):
        return False
    if A.ndim != 2 or B.ndim != 2:
        return False
    if A.shape[1] != B.shape[0]:
        return False
    if A.dtype != _F16 or B.dtype != _F16:
        return False
    return A.get_device() == B.get_device()


def _check_operands(A: torch.Tensor, B: torch.Tensor) -> None:
    # Same checks and messages as the reference launcher (gemm.py:33-40).
    if not (isinstance(A, torch.Tensor) and A.is_cuda):
        raise RuntimeError("A must be a CUDA tensor")
    if not (isinstance(B, torch.Tensor) and B.is_cuda):
        raise RuntimeError("B must be a CUDA tensor")
    if A.dtype != torch.float16:
        raise RuntimeError("A must be float16")
    if B.dtype != torch.float16:
        raise RuntimeError("B must be float16")
    if A.dim() != 2:
        raise RuntimeError("A must be 2D")
    if B.dim() != 2:
        raise RuntimeError("B must be 2D")
    if A.device != B.device:
        raise RuntimeError("A and B must be on the same CUDA device")


_RAW_STREAM = getattr(torch._C, "_cuda_getCurrentRawStream", None)
_GET_DEVICE = getattr(torch._C, "_cuda_getDevice", None) or torch.cuda.current_device


def _current_stream(dev: int) -> int:
    """Raw cudaStream_t of torch's current stream on `dev`."""
    if _RAW_STREAM is not None:
        return _RAW_STREAM(dev)
    return torch.cuda.current_stream(dev).cuda_stream


def _call(A, B, C, M, N, K, lda, ldb, ldc, layout, dev, a_layout=0, alpha=1.0, beta=0.0) -> int:
    stream = _current_stream(dev)
    a, b, c = A.data_ptr(), B.data_ptr(), C.data_ptr()
    aligned = (K == 0 or (a % 16 == 0 and b % 16 == 0 and lda % 8 == 0 and ldb % 8 == 0)) and \
        c % 16 == 0 and ldc % 8 == 0
    if aligned and a_layout == 0 and alpha == 1.0 and beta == 0.0:
        return _native.gemm_f16_raw(a, b, c, M, N, K, lda, ldb, ldc, layout, stream)
    ws_bytes = 0
    ws_ptr = None
    if not aligned:
        # An operand TMA cannot address (odd K or N, or storage not 16-byte
        # aligned): the library re-pitches it through a workspace on the GPU.
        ws_bytes = _native.workspace_size_ex(a, b, c, M, N, K, lda, ldb, ldc, a_layout, layout)
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=A.device)
        ws_ptr = ws.data_ptr()
    return _native.gemm_ex_raw(a, b, c, M, N, K, lda, ldb, ldc, a_layout, layout, alpha, beta, ws_ptr, ws_bytes,
                               stream)


def _launch(A: torch.Tensor, B: torch.Tensor, b_col_major: bool, out: torch.Tensor | None = None,
            alpha: float = 1.0, beta: float = 0.0) -> torch.Tensor:
    """C = alpha * A @ B + beta * out (B given as K x N, or as N x K when b_col_major)."""
    M, K = A.shape
    N = B.shape[0] if b_col_major else B.shape[1]
    if not b_col_major and B.stride(0) == 1 and B.stride(1) >= max(1, K) and B.size(0) > 1:
        # B is the transpose view of an N x K row-major buffer: read it as colb.
        B = B.t()
        b_col_major = True
    a_layout = _native.B200_A_ROW_MAJOR
    if A.stride(0) == 1 and A.stride(1) >= max(1, M) and A.size(1) > 1 and A.size(0) > 1:
        # A is the transpose view of a K x M row-major buffer: read it in place.
        a_layout = _native.B200_A_COL_MAJOR
        lda = A.stride(1)
    else:
        A, lda = _row_view(A)
    B, ldb = _row_view(B)
    if out is None:
        C = torch.empty((M, N), dtype=torch.float16, device=A.device)
        beta = 0.0
    else:
        C = out
    if M == 0 or N == 0:
        return C
    ldc = C.stride(0) if N > 1 else max(1, N)
    dev = A.get_device()
    layout = _native.B200_B_COL_MAJOR if b_col_major else _native.B200_B_ROW_MAJOR
    if dev != _GET_DEVICE():
        with torch.cuda.device(dev):
            code = _call(A, B, C, M, N, K, lda, ldb, ldc, layout, dev, a_layout, alpha, beta)
    else:
        code = _call(A, B, C, M, N, K, lda, ldb, ldc, layout, dev, a_layout, alpha, beta)
    _native.check(code, "root_gemm launch")
    return C


def root_gemm_cuda(A: torch.Tensor, B: torch.Tensor, mode: int) -> torch.Tensor:
    """Counterpart of the reference's native launcher (gemm.py:32-153).

    Same argument meaning: ids 4/5 read B as N x K (`use_colb`, gemm.py:43),
    the others as K x N.  Ids 0-5 are all accepted (the reference allowed
    2-5 only, gemm.py:41, because 0/1 had no launcher).
    """
    _check_operands(A, B)
    if not (0 <= int(mode) <= 5):
        raise RuntimeError("mode must be one of the KERNEL_MODES ids 0-5")
    use_colb = int(mode) in (4, 5)
    if use_colb:
        if A.size(1) != B.size(1):
            raise RuntimeError("Inner dimensions must match for pre-transposed B")
    elif A.size(1) != B.size(0):
        raise RuntimeError("Inner dimensions must match")
    return _launch(A, B, use_colb)


def gemm_pretransposed(A: torch.Tensor, B_col_major: torch.Tensor, mode: str = "wmma") -> torch.Tensor:
    """C = A @ B where B is passed pre-transposed (N x K contiguous).

    Reference: gemm.py:209-216, including its operand convention for mode
    ids 2/3 (the second argument is read as a row-major K x N matrix).
    """
    mode_id = _normalize_mode(mode)
    _check_operands(A, B_col_major)
    if mode_id in _PRETRANSPOSED_ROW_MAJOR_IDS:
        if A.size(1) != B_col_major.size(0):
            raise RuntimeError("Inner dimensions must match")
        return _launch(A, B_col_major, False)
    if A.size(1) != B_col_major.size(1):
        raise RuntimeError("Inner dimensions must match for pre-transposed B")
    return _launch(A, B_col_major, True)


def gemm(A: torch.Tensor, B: torch.Tensor, mode: str = "wmma", out: torch.Tensor | None = None) -> torch.Tensor:
    """C = A @ B with A M x K and B K x N (reference: gemm.py:219-228).

    Raises instead of falling back when ``is_supported`` is False.  ``out``
    (optional, M x N fp16 CUDA tensor with unit column stride) receives the
    result without a new allocation.
    """
    if mode not in _MODE_TO_ID:
        _normalize_mode(mode)
    if not is_supported(A, B):
        _check_operands(A, B)
        if A.shape[1] != B.shape[0]:
            raise RuntimeError("Inner dimensions must match")
        raise RuntimeError("unsupported operands for the B200 GEMM")
    if out is not None:
        if (out.dtype != torch.float16 or out.device != A.device or tuple(out.shape) != (A.shape[0], B.shape[1])
                or (out.shape[1] > 1 and out.stride(1) != 1)):
            raise RuntimeError("out must be an M x N float16 tensor on A's device with unit column stride")
    return _launch(A, B, False, out)


def gemm_ex(A: torch.Tensor, B: torch.Tensor, out: torch.Tensor | None = None, alpha: float = 1.0,
            beta: float = 0.0) -> torch.Tensor:
    """C = alpha * A @ B + beta * out, the reference kernels' alpha / beta
    epilogue (gemm.cu:1360-1364), which the reference launcher fixed to 1 / 0.

    A and B may be row-major or transpose views (read in place).  With
    beta != 0, `out` must be given and holds the old C on entry.
    """
    if not is_supported(A, B):
        _check_operands(A, B)
        raise RuntimeError("Inner dimensions must match")
    if beta != 0.0 and out is None:
        raise RuntimeError("beta != 0 needs `out` holding the old C")
    if out is not None:
        if (out.dtype != torch.float16 or out.device != A.device or tuple(out.shape) != (A.shape[0], B.shape[1])
                or (out.shape[1] > 1 and out.stride(1) != 1)):
            raise RuntimeError("out must be an M x N float16 tensor on A's device with unit column stride")
    return _launch(A, B, False, out, float(alpha), float(beta))
