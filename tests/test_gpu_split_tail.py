"""GPU: the pair kernel's K-split of a partial last wave.

When a 256 x 256-tile launch ends with a partial wave (tiles % pairs != 0)
and K is deep enough, the tail tiles are cut into S K-ranges whose fp32
parts are summed by the last range to arrive.  These shapes all take that
path under the "pair" variant (148 SMs: 74 pairs); each is checked against
the fp32 product, for bit-determinism, through alpha / beta, under CUDA-graph
replay on a stream that already owns a workspace (the per-tile counters
reset themselves) and from two streams at once (each stream has its own
workspace).
"""
from __future__ import annotations

import pytest
import torch

import tensorcore_gemm as tg
from gpu_util import assert_parity, fp32_ref

pytestmark = pytest.mark.gpu

# (M, N, K): tiles = ceil(M/256) * ceil(N/256) > 74 with a partial last wave,
# K deep enough for the split to pay (the launcher's cost model).
SPLIT_SHAPES = [
    (2560, 2048, 8192),    # 80 tiles: 1 full wave + 6 tail tiles, 4 K ranges
    (2500, 2000, 7000),    # ragged M, N and K (K not a multiple of the 128-deep stage)
    (4096, 4096, 16384),   # 256 tiles: 3 waves + 34 tail tiles, 2 K ranges
    (1024, 19200, 12288),  # 300 tiles: 4 waves + 4 tail tiles, 6 K ranges
]


@pytest.fixture
def pair_variant(native_lib):
    from tensorcore_gemm import _native

    _native.set_variant("pair")
    yield
    _native.set_variant("auto")


def _operands(M, N, K, seed, colb=False):
    g = torch.Generator(device="cuda").manual_seed(seed)
    A = (torch.rand((M, K), device="cuda", generator=g) * 2 - 1).half()
    B = (torch.rand((N, K) if colb else (K, N), device="cuda", generator=g) * 2 - 1).half()
    return A, B


@pytest.mark.parametrize("M,N,K", SPLIT_SHAPES)
@pytest.mark.parametrize("colb", [False, True])
def test_split_tail_parity_and_determinism(pair_variant, M, N, K, colb):
    from tensorcore_gemm import _native

    A, B = _operands(M, N, K, seed=M + N + K, colb=colb)
    run = (lambda: tg.gemm_pretransposed(A, B, mode="reg_pingpong_256_colb")) if colb else (lambda: tg.gemm(A, B))
    C1 = run()
    C2 = run()
    torch.cuda.synchronize()
    assert_parity(C1, fp32_ref(A, B, b_col_major=colb), K, f"{M}x{N}x{K} split tail")
    assert torch.equal(C1, C2), "split-tail result differs between runs"
    assert _native.last_device_error() == 0


def test_split_tail_alpha_beta(pair_variant):
    from tensorcore_gemm.gemm import gemm_ex

    M, N, K = 2560, 2048, 8192
    A, B = _operands(M, N, K, seed=11)
    C = (torch.randn((M, N), device="cuda") * 4).half()
    ref = 0.75 * fp32_ref(A, B) - 0.5 * C.float()
    out = gemm_ex(A, B, out=C.clone(), alpha=0.75, beta=-0.5)
    torch.cuda.synchronize()
    assert_parity(out, ref, K, "split tail alpha/beta")


def test_split_tail_graph_replay(pair_variant):
    """The tail counters reset after each use, so a captured launch replays correctly."""
    M, N, K = 2560, 2048, 8192
    A, B = _operands(M, N, K, seed=3)
    C = torch.empty((M, N), dtype=torch.float16, device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        tg.gemm(A, B, out=C)             # allocates this stream's split workspace before capture
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    ref = C.clone()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        tg.gemm(A, B, out=C)
    for _ in range(3):
        C.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(C, ref), "graph replay of a split-tail launch changed the result"


def test_split_tail_two_streams(pair_variant):
    M, N, K = 2560, 2048, 8192
    ops = [_operands(M, N, K, seed=20 + i) for i in range(2)]
    outs = [torch.empty((M, N), dtype=torch.float16, device="cuda") for _ in range(2)]
    streams = [torch.cuda.Stream() for _ in range(2)]
    torch.cuda.synchronize()
    for _ in range(5):
        for (A, B), C, st in zip(ops, outs, streams):
            with torch.cuda.stream(st):
                tg.gemm(A, B, out=C)
    torch.cuda.synchronize()
    for (A, B), C in zip(ops, outs):
        assert_parity(C, fp32_ref(A, B), K, "split tail, concurrent streams")
