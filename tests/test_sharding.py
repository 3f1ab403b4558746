"""CPU: row-shard bookkeeping and the C all-gather with two gloo ranks."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tensorcore_gemm import sharded


@pytest.mark.parametrize("M,world", [(65536, 1), (65536, 2), (65536, 8), (1000, 3), (5, 4), (0, 2), (129, 2)])
def test_shards_cover_rows_exactly_once(M, world):
    b = sharded.all_shard_bounds(M, world)
    assert b[0][0] == 0 and b[-1][1] == M
    for (a0, a1), (b0, b1) in zip(b, b[1:]):
        assert a1 == b0 and a0 <= a1
    for lo, _ in b:
        assert lo % sharded.SHARD_ALIGN_ROWS == 0 or lo == M


def test_even_split_of_config_shape():
    assert sharded.all_shard_bounds(65536, 8) == [(r * 8192, (r + 1) * 8192) for r in range(8)]


def test_bad_rank():
    with pytest.raises(ValueError):
        sharded.row_shard_bounds(10, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, M, N, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lo, hi = sharded.row_shard_bounds(M, world, rank)
        # Stand-in for this rank's GEMM output: row index encoded in the values.
        shard = torch.arange(lo, hi, dtype=torch.float32).unsqueeze(1).repeat(1, N).half()
        full = sharded.all_gather_rows(shard, M)
        want = torch.arange(M, dtype=torch.float32).unsqueeze(1).repeat(1, N).half()
        q.put((rank, bool(torch.equal(full, want))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("M", [512, 300])
def test_all_gather_two_gloo_ranks(M):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, M, 8, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    results = dict(q.get(timeout=10) for _ in procs)
    assert all(p.exitcode == 0 for p in procs)
    assert results == {0: True, 1: True}


def test_peer_shard_pointers():
    """Each peer pointer is that peer's buffer base plus the shard's first row (fp16, pitch ldc)."""
    bases = [0x7f0000000000, 0x7f1000000000, 0x7f2000000000]
    lo, _ = sharded.row_shard_bounds(65536, 8, 5)
    ptrs = sharded.peer_shard_ptrs(bases, lo, 8192)
    assert ptrs == [b + lo * 8192 * 2 for b in bases]
    assert all(p % 16 == 0 for p in ptrs)


def _exchange_worker(rank, world, port, scenario, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    closed = []
    try:
        handle = b"" if (scenario == "alloc_fails" and rank == 0) else bytes([rank + 1]) * 64

        def open_fn(h):
            if scenario == "open_fails" and rank == world - 1 and h[0] == 1:
                raise RuntimeError("cannot map rank 0")
            return 1000 + h[0] - 1       # "address" of the peer's buffer: 1000 + its rank

        try:
            peers = sharded.exchange_and_open(handle, None, open_fn, closed.append, "cpu")
            q.put((rank, "ok", peers, closed))
        except RuntimeError as exc:
            q.put((rank, "raised", str(exc), closed))
    finally:
        dist.destroy_process_group()


def _run_exchange(scenario, world=3):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, world, port, scenario, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    results = {r: rest for r, *rest in (q.get(timeout=10) for _ in procs)}
    assert all(p.exitcode == 0 for p in procs)
    return results


def test_gathered_output_handshake_maps_every_peer():
    """Each rank maps every other rank's buffer, in rank order, and closes nothing."""
    res = _run_exchange("ok")
    for r, (outcome, peers, closed) in res.items():
        assert outcome == "ok"
        assert peers == [1000 + p for p in range(3) if p != r]
        assert closed == []


@pytest.mark.parametrize("scenario", ["open_fails", "alloc_fails"])
def test_gathered_output_handshake_fails_on_every_rank(scenario):
    """One rank failing (a peer it cannot map, or no buffer of its own) makes
    every rank raise, each after closing the mappings it had opened."""
    res = _run_exchange(scenario)
    for r, (outcome, detail, closed) in res.items():
        assert outcome == "raised", (r, detail)
        assert "gathered output unavailable" in detail
    if scenario == "open_fails":
        assert res[0][2] == [1001, 1002] and res[1][2] == [1000, 1002]   # opened both, closed both
        assert res[2][2] == []                                          # failed on its first open
    else:
        assert all(closed == [] for _, _, closed in res.values())       # nothing was opened


def _agree_worker(rank, world, port, bad_rank, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        flag = torch.zeros(1)
        failure = "shard has 100 rows, expected 128" if rank == bad_rank else None
        try:
            sharded.agree_on_failure(failure, None, flag)
            outcome = "ok"
        except RuntimeError as exc:
            outcome = str(exc)
        # The group is still usable afterwards: nobody was left inside a collective.
        t = torch.tensor([float(rank)])
        dist.all_reduce(t)
        q.put((rank, outcome, t.item()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("bad_rank", [None, 1])
def test_gathered_gemm_agrees_on_argument_failures(bad_rank):
    """One rank with a wrong shard makes both ranks raise before any launch
    (GatheredOutput.gemm's pre-launch agreement); with no failure both go on."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_agree_worker, args=(r, 2, port, bad_rank, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    res = {r: (o, s) for r, o, s in (q.get(timeout=10) for _ in procs)}
    assert all(p.exitcode == 0 for p in procs)
    for r, (outcome, total) in res.items():
        assert total == 1.0
        if bad_rank is None:
            assert outcome == "ok"
        else:
            assert "gathered GEMM not run" in outcome
            assert ("shard has 100 rows" in outcome) == (r == bad_rank)
