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

import torch

from .gemm import gemm


def gemm_streamed(A_host: torch.Tensor, B: torch.Tensor, out: torch.Tensor | None = None,
                  chunk_rows: int | None = None, mode: str = "reg_pingpong_256") -> torch.Tensor:
    """C = A_host @ B with A (M x K fp16) in host memory, pipelined over row chunks.

    B (K x N fp16) may be in host memory (copied once) or already on the GPU.
    `out` (M x N fp16) may be a host tensor (pinned for overlap) or a CUDA
    tensor; by default a pinned host tensor is allocated and returned.
    `chunk_rows` defaults to about an eighth of M (a multiple of 256).  The
    call returns once all work is queued on the current stream's device;
    synchronize (or read `out` after torch.cuda.synchronize()) before using a
    host result.
    """
    if A_host.is_cuda:
        raise RuntimeError("gemm_streamed expects A in host memory; use gemm() for device operands")
    if A_host.dtype != torch.float16 or B.dtype != torch.float16:
        raise RuntimeError("A and B must be float16")
    if A_host.dim() != 2 or B.dim() != 2 or A_host.shape[1] != B.shape[0]:
        raise RuntimeError("Inner dimensions must match")
    if chunk_rows is None:
        chunk_rows = max(256, -(-A_host.shape[0] // 8 // 256) * 256)
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

    main = torch.cuda.current_stream(dev)
    h2d = torch.cuda.Stream(dev)
    comp = torch.cuda.Stream(dev)
    d2h = torch.cuda.Stream(dev)
    for s in (h2d, comp, d2h):
        s.wait_stream(main)

    rows = min(chunk_rows, M)
    with torch.cuda.stream(h2d):
        B_dev = B if B.is_cuda else B.to(dev, non_blocking=True)
        b_ready = torch.cuda.Event()
        b_ready.record(h2d)
    a_buf = [torch.empty((rows, K), dtype=torch.float16, device=dev) for _ in range(2)]
    c_buf = [torch.empty((rows, N), dtype=torch.float16, device=dev) for _ in range(2)]
    a_ready = [torch.cuda.Event() for _ in range(2)]
    a_free = [torch.cuda.Event() for _ in range(2)]
    c_ready = [torch.cuda.Event() for _ in range(2)]
    c_free = [torch.cuda.Event() for _ in range(2)]
    comp.wait_event(b_ready)

    for i, r0 in enumerate(range(0, M, rows)):
        r1 = min(r0 + rows, M)
        n = r1 - r0
        j = i & 1
        with torch.cuda.stream(h2d):
            if i >= 2:
                h2d.wait_event(a_free[j])          # the kernel two chunks back has read this buffer
            a_buf[j][:n].copy_(A_host[r0:r1], non_blocking=True)
            a_ready[j].record(h2d)
        with torch.cuda.stream(comp):
            comp.wait_event(a_ready[j])
            if i >= 2:
                comp.wait_event(c_free[j])         # chunk i-2's result has left this buffer
            gemm(a_buf[j][:n], B_dev, mode=mode, out=c_buf[j][:n])
            a_free[j].record(comp)
            c_ready[j].record(comp)
        with torch.cuda.stream(d2h):
            d2h.wait_event(c_ready[j])
            out[r0:r1].copy_(c_buf[j][:n], non_blocking=True)
            c_free[j].record(d2h)

    # Device buffers were used on the side streams: keep the allocator from
    # handing them out again before that work is done, and order the caller's
    # stream after the whole pipeline.
    for t in a_buf + c_buf:
        for s in (h2d, comp, d2h):
            t.record_stream(s)
    if not B.is_cuda:
        for s in (h2d, comp):
            B_dev.record_stream(s)
    main.wait_stream(d2h)
    main.wait_stream(comp)
    return out
