"""GPU, 2+ devices: row-sharded GEMM on each rank plus the NCCL all-gather of
C, and the fused gathered-output GEMM (peer stores from the epilogue).

Skipped when fewer than two GPUs are visible.  Each rank is its own process
(one process per GPU); no kernel waits on another GPU.
"""
from __future__ import annotations

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parent.parent
    for p in (str(repo), str(repo / "ampere-gemm_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist

    from oracle import oracle
    from tensorcore_gemm import _native, sharded

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        M, N, K = 1000, 264, 512          # ragged: the last shard is short
        A, B = oracle.make_inputs(M, N, K, dist="normal", seed_a=31, seed_b=32, std=0.02)
        lo, hi = sharded.row_shard_bounds(M, world, rank)
        Cs = sharded.sharded_gemm(A[lo:hi].to(dev), B.to(dev))
        full = sharded.all_gather_rows(Cs, M)
        torch.cuda.synchronize()
        ref = A.float() @ B.float()
        err = (full.float().cpu() - ref).abs().max().item()
        bound = 2e-3 * K ** 0.5 * ref.pow(2).mean().sqrt().item()
        q.put((rank, err <= bound and _native.last_device_error() == 0, err, bound))
    finally:
        dist.destroy_process_group()


def test_two_rank_sharded_gemm_and_all_gather(native_lib):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    res = [q.get(timeout=30) for _ in procs]
    assert all(p.exitcode == 0 for p in procs)
    assert all(ok for _, ok, _, _ in res), res


def _gather_worker(rank, world, port, q):
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parent.parent
    for p in (str(repo), str(repo / "ampere-gemm_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist

    from oracle import oracle
    from tensorcore_gemm import _native, sharded

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    out = None
    try:
        results = []
        for (M, N, K, colb) in [(1000, 264, 512, False), (3000, 1001, 256, True), (2048, 2048, 2048, False)]:
            A, B = oracle.make_inputs(M, N, K, dist="normal", seed_a=41 + M, seed_b=42 + N, std=0.02)
            out = sharded.GatheredOutput(M, N, device=dev)
            lo, hi = out.bounds()
            Bd = B.to(dev)
            full = out.gemm(A[lo:hi].to(dev), Bd.t().contiguous() if colb else Bd, b_col_major=colb)
            torch.cuda.synchronize()
            ref = A.float() @ B.float()
            err = (full.float().cpu() - ref).abs().max().item()
            bound = 2e-3 * K ** 0.5 * ref.pow(2).mean().sqrt().item()
            # Rows written by the peers must equal what the plain path computes there.
            results.append(err <= bound)
            out.close()
            out = None
        q.put((rank, all(results) and _native.last_device_error() == 0, results))
    finally:
        if out is not None:
            out.close()
        dist.destroy_process_group()


def test_two_rank_gathered_output(native_lib):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    res = [q.get(timeout=30) for _ in procs]
    assert all(p.exitcode == 0 for p in procs)
    assert all(ok for _, ok, _ in res), res


def _b2b_worker(rank, world, port, q):
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parent.parent
    for p in (str(repo), str(repo / "ampere-gemm_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist

    from oracle import oracle
    from tensorcore_gemm import _native, sharded

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    out = None
    try:
        M, N, K = 4096, 2048, 1024
        A, B1 = oracle.make_inputs(M, N, K, dist="normal", seed_a=7, seed_b=8, std=0.02)
        _, B2 = oracle.make_inputs(M, N, K, dist="normal", seed_a=7, seed_b=9, std=0.02)
        out = sharded.GatheredOutput(M, N, device=dev)
        lo, hi = out.bounds()
        Ad = A[lo:hi].to(dev)
        oks = []
        for _ in range(3):
            full = out.gemm(Ad, B1.to(dev))
            if rank == world - 1:
                torch.cuda._sleep(100_000_000)   # a slow consumer: reads call 1's result late
            snap = full.clone()                  # same stream as the next call
            full2 = out.gemm(Ad, B2.to(dev))
            torch.cuda.synchronize()
            for got, Bx in ((snap, B1), (full2, B2)):
                ref = A.float() @ Bx.float()
                err = (got.float().cpu() - ref).abs().max().item()
                oks.append(err <= 2e-3 * K ** 0.5 * ref.pow(2).mean().sqrt().item())
        q.put((rank, all(oks) and _native.last_device_error() == 0, oks))
    finally:
        if out is not None:
            out.close()
        dist.destroy_process_group()


def test_two_rank_gathered_output_back_to_back_with_slow_reader(native_lib):
    """A rank's next gathered call must not store into a peer's copy while that
    peer is still reading the previous result (the pre-launch barrier)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_b2b_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    res = [q.get(timeout=30) for _ in procs]
    assert all(p.exitcode == 0 for p in procs)
    assert all(ok for _, ok, _ in res), res
