"""GEMM on operands that live in host memory, with the PCIe traffic overlapped.

`gemm_streamed(A_host, B, out_host)` computes C = A @ B on the current GPU for
A (and optionally B and C) in pinned host memory.  A's rows are cut into
chunks; three CUDA streams run in a pipeline -- host-to-device copy of chunk
i+1, the B200 kernel on chunk i, device-to-host copy of chunk i-1 -- through
two device buffers per operand, so the copies in both directions and the
tensor-core work overlap instead of running back to back.  Every chunk is
multiplied by the same sm_100a kernels as `gemm`; nothing runs on the CPU.

The reference has no host-operand path (its `gemm` on CPU tensors ran
torch.matmul on the CPU, tensorcore_gemm/gemm.py:219-221); this is the B200
answer for callers whose matrices start and end in host memory.
"""
from __future__ import annotations

import threading

import torch

from .gemm import gemm


class _Pipeline:
    """Device buffers, side streams and events of one (device, chunk shape),
    kept across calls: fresh buffers per call would be held back by the
    caching allocator until the side streams pass them, so every call would
    allocate (and synchronise) anew.  Successive calls are ordered through the
    same buffer-free events, so a buffer is never refilled before the previous
    call's kernel and copy-out have finished with it."""

    def __init__(self, dev: torch.device, rows: int, K: int, N: int):
        self.h2d, self.comp, self.d2h = (torch.cuda.Stream(dev) for _ in range(3))
        self.a_buf = [torch.empty((rows, K), dtype=torch.float16, device=dev) for _ in range(2)]
        self.c_buf = [torch.empty((rows, N), dtype=torch.float16, device=dev) for _ in range(2)]
        self.a_ready = [torch.cuda.Event() for _ in range(2)]
        self.a_free = [torch.cuda.Event() for _ in range(2)]
        self.c_ready = [torch.cuda.Event() for _ in range(2)]
        self.c_free = [torch.cuda.Event() for _ in range(2)]
        self.used = [False, False]       # buffer pair j has been used by an earlier chunk
        self.b_dev = None
        self.b_ready = torch.cuda.Event()
        self.b_free = torch.cuda.Event()  # the last kernel that read b_dev
        self.lock = threading.Lock()


_PIPELINES: dict[tuple, _Pipeline] = {}
_PIPELINES_LOCK = threading.Lock()


def _pipeline(dev: torch.device, rows: int, K: int, N: int) -> _Pipeline:
    key = (dev.index, rows, K, N)
    with _PIPELINES_LOCK:
        p = _PIPELINES.get(key)
        if p is None:
            p = _PIPELINES[key] = _Pipeline(dev, rows, K, N)
        return p


def gemm_streamed(A_host: torch.Tensor, B: torch.Tensor, out: torch.Tensor | None = None,
                  chunk_rows: int | None = None, mode: str = "reg_pingpong_256") -> torch.Tensor:
    """C = A_host @ B with A (M x K fp16) in host memory, pipelined over row chunks.

    B (K x N fp16) may be in host memory (copied in every call) or already on
    the GPU.  `out` (M x N fp16) may be a host tensor (pinned for overlap) or
    a CUDA tensor; by default a pinned host tensor is allocated and returned.
    `chunk_rows` defaults to about a sixteenth of M (a multiple of 256).  The
    call returns once all work is queued; it is ordered after the current
    stream's earlier work and the current stream waits for it, so read a host
    result after torch.cuda.synchronize().  Device buffers are kept per
    (device, chunk shape) for the next call.
    """
    if A_host.is_cuda:
        raise RuntimeError("gemm_streamed expects A in host memory; use gemm() for device operands")
    if A_host.dtype != torch.float16 or B.dtype != torch.float16:
        raise RuntimeError("A and B must be float16")
    if A_host.dim() != 2 or B.dim() != 2 or A_host.shape[1] != B.shape[0]:
        raise RuntimeError("Inner dimensions must match")
    if chunk_rows is None:
        chunk_rows = max(256, -(-A_host.shape[0] // 16 // 256) * 256)
    if chunk_rows <= 0:
        raise ValueError("chunk_rows must be positive")
    dev = torch.device("cuda", torch.cuda.current_device())
    M, K = A_host.shape
    N = B.shape[1]
    if out is None:
        out = torch.empty((M, N), dtype=torch.float16, pin_memory=True)
    if tuple(out.shape) != (M, N) or out.dtype != torch.float16:
        raise RuntimeError("out must be an M x N float16 tensor")
    if M == 0 or N == 0:
        return out
    A_host = A_host.contiguous()
    rows = min(chunk_rows, M)
    p = _pipeline(dev, rows, K, N)
    main = torch.cuda.current_stream(dev)
    with p.lock:
        for s in (p.h2d, p.comp, p.d2h):
            s.wait_stream(main)
        if B.is_cuda:
            B_dev = B
        else:
            with torch.cuda.stream(p.h2d):
                if p.b_dev is None or tuple(p.b_dev.shape) != (K, N):
                    p.b_dev = torch.empty((K, N), dtype=torch.float16, device=dev)
                else:
                    p.h2d.wait_event(p.b_free)    # the previous call's kernels are done with it
                p.b_dev.copy_(B, non_blocking=True)
                p.b_ready.record(p.h2d)
            p.comp.wait_event(p.b_ready)
            B_dev = p.b_dev

        for i, r0 in enumerate(range(0, M, rows)):
            r1 = min(r0 + rows, M)
            n = r1 - r0
            j = i & 1
            with torch.cuda.stream(p.h2d):
                if p.used[j]:
                    p.h2d.wait_event(p.a_free[j])      # the kernel that last read this buffer is done
                p.a_buf[j][:n].copy_(A_host[r0:r1], non_blocking=True)
                p.a_ready[j].record(p.h2d)
            with torch.cuda.stream(p.comp):
                p.comp.wait_event(p.a_ready[j])
                if p.used[j]:
                    p.comp.wait_event(p.c_free[j])     # the last result in this buffer has left
                gemm(p.a_buf[j][:n], B_dev, mode=mode, out=p.c_buf[j][:n])
                p.a_free[j].record(p.comp)
                p.c_ready[j].record(p.comp)
            with torch.cuda.stream(p.d2h):
                p.d2h.wait_event(p.c_ready[j])
                out[r0:r1].copy_(p.c_buf[j][:n], non_blocking=True)
                p.c_free[j].record(p.d2h)
            p.used[j] = True
        p.b_free.record(p.comp)
        if B.is_cuda:
            B.record_stream(p.comp)
        main.wait_stream(p.d2h)
        main.wait_stream(p.comp)
    return out


def release_pipelines() -> None:
    """Drop the device buffers kept for earlier gemm_streamed calls (after their
    work has finished: synchronize first)."""
    with _PIPELINES_LOCK:
        _PIPELINES.clear()
