"""Row-sharded multi-GPU GEMM: one process per GPU, A split by rows, B replicated.

The reference is single-GPU only; this is the multi-GPU form of the same
product.  Output rows are independent, so the GEMM itself needs no
collective: rank r computes C[r-th row block] = A[r-th row block] @ B on its
own GPU.  The only collective is the optional all-gather of the C shards into
a full C on every rank (NCCL over NVLink/NVSwitch), kept separate so it can
be timed on its own.
"""
from __future__ import annotations

import torch

from .gemm import gemm

# Shards start on multiples of the kernel's 128-row tile so no tile straddles
# two ranks.
SHARD_ALIGN_ROWS = 128


def row_shard_bounds(M: int, world: int, rank: int, align: int = SHARD_ALIGN_ROWS) -> tuple[int, int]:
    """[start, end) rows of A / C owned by `rank` of `world`.

    Blocks of `align` rows are dealt out as evenly as possible; lower ranks get
    the extra blocks, the last rank gets the ragged tail.
    """
    if world < 1 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} of world {world}")
    if M < 0:
        raise ValueError("M must be >= 0")
    blocks = -(-M // align)
    base, extra = divmod(blocks, world)
    b0 = rank * base + min(rank, extra)
    b1 = b0 + base + (1 if rank < extra else 0)
    return min(b0 * align, M), min(b1 * align, M)


def all_shard_bounds(M: int, world: int, align: int = SHARD_ALIGN_ROWS) -> list[tuple[int, int]]:
    return [row_shard_bounds(M, world, r, align) for r in range(world)]


def sharded_gemm(A_shard: torch.Tensor, B: torch.Tensor, mode: str = "reg_pingpong_256",
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """This rank's C rows: A_shard @ B on the local GPU (no communication)."""
    return gemm(A_shard, B, mode=mode, out=out)


def all_gather_rows(C_shard: torch.Tensor, M: int, group=None, align: int = SHARD_ALIGN_ROWS) -> torch.Tensor:
    """Gather every rank's C rows into a full M x N tensor on every rank.

    Shards may differ in length (ragged last shard); each is padded to the
    largest shard for one all_gather_into_tensor and the padding is dropped.
    """
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    bounds = all_shard_bounds(M, world, align)
    lo, hi = bounds[rank]
    if C_shard.shape[0] != hi - lo:
        raise ValueError(f"rank {rank} shard has {C_shard.shape[0]} rows, expected {hi - lo}")
    rows = max(b - a for a, b in bounds)
    N = C_shard.shape[1]
    if all(b - a == rows for a, b in bounds):
        full = torch.empty((rows * world, N), dtype=C_shard.dtype, device=C_shard.device)
        dist.all_gather_into_tensor(full, C_shard.contiguous(), group=group)
        return full[:M]
    padded = torch.zeros((rows, N), dtype=C_shard.dtype, device=C_shard.device)
    padded[: hi - lo] = C_shard
    full = torch.empty((rows * world, N), dtype=C_shard.dtype, device=C_shard.device)
    dist.all_gather_into_tensor(full, padded, group=group)
    return torch.cat([full[r * rows: r * rows + (b - a)] for r, (a, b) in enumerate(bounds)], dim=0)


def peer_shard_ptrs(peer_bases: list[int], row0: int, ldc: int, elem_bytes: int = 2) -> list[int]:
    """Addresses of this shard's first row in every peer's copy of the gathered C."""
    return [int(b) + int(row0) * int(ldc) * elem_bytes for b in peer_bases]


def agree_on_failure(failure: str | None, group, flag: torch.Tensor) -> None:
    """Collective: raise on every rank of `group` if `failure` is set on any.

    `flag` is a one-element float32 tensor on the device the collective runs
    on; it is overwritten.  On a CUDA device the all-reduce is enqueued on the
    current stream, so it is also a device-side barrier: it completes on a rank
    only once every rank's stream has reached it.  Reading the result back
    synchronises this rank's current stream.
    """
    import torch.distributed as dist

    flag.fill_(1.0 if failure else 0.0)
    dist.all_reduce(flag, group=group)
    if flag.item() > 0:
        raise RuntimeError(f"gathered GEMM not run: {failure or 'failed on another rank'}")


def exchange_and_open(handle: bytes, group, open_fn, close_fn, flag_device) -> list:
    """Collective: share this rank's buffer handle, map every other rank's.

    Returns the peers' mappings in rank order (own rank skipped).  Every rank
    learns whether all of them succeeded, so a failure anywhere (an empty
    handle: the rank could not allocate; or `open_fn` raising) makes every
    rank close what it opened and raise together, instead of leaving some
    rank waiting in a later collective.
    """
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    handles = [None] * world
    dist.all_gather_object(handles, handle, group=group)
    peers, failure = [], None
    if not all(handles):
        failure = "a rank could not allocate its IPC buffer"
    else:
        try:
            for r, h in enumerate(handles):
                if r != rank:
                    peers.append(open_fn(h))
        except RuntimeError as exc:
            failure = str(exc)
    flag = torch.tensor([1.0 if failure else 0.0], device=flag_device)
    dist.all_reduce(flag, group=group)
    if flag.item() > 0:
        for p in peers:
            close_fn(p)
        dist.barrier(group=group)
        raise RuntimeError(f"gathered output unavailable: {failure or 'failed on another rank'}")
    return peers


class _DeviceBuffer:
    """A raw device allocation exposed to torch (__cuda_array_interface__)."""

    def __init__(self, ptr: int, rows: int, cols: int):
        self.__cuda_array_interface__ = {"shape": (rows, cols), "typestr": "<f2", "data": (int(ptr), False),
                                         "version": 3, "strides": None}


class GatheredOutput:
    """The full M x N C on every rank, filled by the fused gathered-output GEMM.

    Every rank allocates its copy of C as one IPC-shareable buffer (legacy
    CUDA IPC, no multicast object) and maps every peer's copy.  `gemm` then
    runs this rank's row shard with b200_gemm_f16_gather: each finished C
    block goes to the local copy with a TMA store and to every peer's copy
    with plain 16-byte stores over NVLink, so the all-gather rides under the
    GEMM.  A one-element all-reduce on the current stream afterwards is the
    device-side barrier after which every rank's copy holds all rows.
    Collective: every rank of `group` constructs it, calls `gemm` and
    `close` in the same order.
    """

    def __init__(self, M: int, N: int, group=None, device: torch.device | None = None,
                 align: int = SHARD_ALIGN_ROWS):
        import torch.distributed as dist

        from . import _native

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world - 1 > 7:
            raise ValueError("the gathered output supports at most 8 ranks")
        self.M, self.N, self.align = int(M), int(N), align
        self.ldc = max(8, -(-self.N // 8) * 8)
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        with torch.cuda.device(self.device):
            try:
                self._ptr, handle = _native.ipc_alloc(max(1, self.M) * self.ldc * 2)
            except RuntimeError:
                self._ptr, handle = 0, b""
            try:
                self._peers = exchange_and_open(handle, group, _native.ipc_open, _native.ipc_close, self.device)
            except RuntimeError:
                if self._ptr:
                    _native.ipc_free(self._ptr)
                raise
            self._buf = _DeviceBuffer(self._ptr, max(1, self.M), self.ldc)
            self._full = torch.as_tensor(self._buf, device=self.device)
            self._flag = torch.zeros(1, dtype=torch.float32, device=self.device)
        self._closed = False

    @property
    def full(self) -> torch.Tensor:
        """This rank's copy of the gathered C (M x N view of the M x ldc buffer)."""
        return self._full[: self.M, : self.N]

    def bounds(self) -> tuple[int, int]:
        return row_shard_bounds(self.M, self.world, self.rank, self.align)

    def gemm(self, A_shard: torch.Tensor, B: torch.Tensor, b_col_major: bool = False) -> torch.Tensor:
        """Fill `full` with [A_0; A_1; ...] @ B, A_r being rank r's rows (B as K x N, or N x K if b_col_major).

        Collective.  Before the launch the ranks agree on their argument checks
        with a one-element all-reduce on the current stream (a rank whose
        operands are wrong makes every rank raise, so none is left waiting in
        a collective); that all-reduce is also the barrier that keeps this
        call's peer stores out of `full` until every rank's stream has passed
        its work queued before the call.  Work that reads `full` on another
        stream must be ordered before the next call's current stream by the
        caller.  A second all-reduce after the launch marks every copy
        complete; a failed launch still joins it, then raises on every rank.
        """
        from . import _native
        from .gemm import _check_operands, _current_stream
        from .kmeans import _pitched

        if self._closed:
            raise RuntimeError("GatheredOutput is closed")
        lo, hi = self.bounds()
        failure = None
        try:
            Bk = B.t() if b_col_major else B
            _check_operands(A_shard, Bk)
            if A_shard.shape[0] != hi - lo:
                raise RuntimeError(f"rank {self.rank} shard has {A_shard.shape[0]} rows, expected {hi - lo}")
            if Bk.shape[1] != self.N:
                raise RuntimeError(f"B has {Bk.shape[1]} columns, the gathered output {self.N}")
            if not b_col_major and B.stride(0) == 1 and B.stride(1) >= max(1, B.shape[0]) and B.size(0) > 1:
                B, b_col_major = B.t(), True   # transposed view of an N x K buffer
            A = _pitched(A_shard)
            B = _pitched(B)
        except (RuntimeError, ValueError) as exc:
            failure = f"rank {self.rank}: {exc}"
        with torch.cuda.device(self.device):
            agree_on_failure(failure, self.group, self._flag)
            layout = _native.B200_B_COL_MAJOR if b_col_major else _native.B200_B_ROW_MAJOR
            K = A.shape[1]
            c_ptr = self._ptr + lo * self.ldc * 2
            code = _native.gemm_gather_raw(A.data_ptr(), B.data_ptr(), c_ptr, hi - lo, self.N, K,
                                           A.stride(0), B.stride(0),
                                           self.ldc, layout, peer_shard_ptrs(self._peers, lo, self.ldc),
                                           _current_stream(self.device.index))
            launch_failure = None if code == _native.B200_OK else (
                f"rank {self.rank}: b200_gemm_f16_gather failed: {_native.strerror(code)} (code {code})")
            agree_on_failure(launch_failure, self.group, self._flag)
        return self.full

    def close(self) -> None:
        """Unmap the peers' copies, then free this rank's (collective)."""
        import torch.distributed as dist

        from . import _native

        if self._closed:
            return
        self._closed = True
        with torch.cuda.device(self.device):
            torch.cuda.synchronize()
            dist.barrier(group=self.group)
            for p in self._peers:
                _native.ipc_close(p)
            dist.barrier(group=self.group)
            self._full = None
            _native.ipc_free(self._ptr)
