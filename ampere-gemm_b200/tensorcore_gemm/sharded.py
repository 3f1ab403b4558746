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
