"""GPU parity of the B200 kernels through the public API and the C ABI.

Bar (north star): max|C - C_ref| <= 2e-3 * sqrt(K) * RMS(C_ref), C_ref the fp32
product of the same fp16 inputs; small cases are also checked against the C
oracle and the committed golden vectors of the reference's output.
"""
from __future__ import annotations

import importlib
import json
from pathlib import Path

import numpy as np
import pytest
import torch

import tensorcore_gemm as tg
from gpu_util import assert_parity, fp32_ref, oracle_check
from oracle import oracle
from tensorcore_gemm import _native

pytestmark = pytest.mark.gpu
gemm_mod = importlib.import_module("tensorcore_gemm.gemm")
GOLDEN = Path(__file__).resolve().parent / "golden"


def _inputs(M, N, K, dev, dist="uniform", seed=0, std=1.0):
    A, B = oracle.make_inputs(M, N, K, dist=dist, seed_a=seed, seed_b=seed + 1, std=std)
    return A.to(dev), B.to(dev)


@pytest.fixture(params=["auto", "cta1", "pair", "skinny", "pair2m", "pair2m_224", "pair2m_192"])
def variant(request, native_lib):
    _native.set_variant(request.param)
    yield request.param
    _native.set_variant("auto")


def _no_device_error():
    assert _native.last_device_error() == 0


def test_golden_vectors_on_gpu(cuda_device, variant):
    meta = json.loads((GOLDEN / "gemm_golden.json").read_text())
    data = np.load(GOLDEN / "gemm_golden.npz")
    for c in meta["cases"]:
        n = c["name"]
        A = torch.from_numpy(data[n + "__A"]).to(cuda_device)
        B = torch.from_numpy(data[n + "__B"]).to(cuda_device)
        C_ref = data[n + "__C"].astype(np.float32)
        for C in (tg.gemm(A, B), tg.gemm_pretransposed(A, B.t().contiguous(), mode="reg_pingpong_256_colb")):
            got = C.float().cpu().numpy()
            assert_parity(C, fp32_ref(A, B), c["K"], n)
            ulp = np.abs(np.spacing(data[n + "__C"])).astype(np.float32).max()
            assert np.abs(got - C_ref).max() <= 2 * ulp, f"{n}: differs from the reference output by > 2 ulp"
    _no_device_error()


SMALL = [(1, 8, 8), (8, 8, 8), (37, 24, 40), (128, 256, 64), (129, 264, 72), (255, 136, 200),
         (64, 1024, 16), (300, 8, 1000), (1000, 1000, 1000), (513, 520, 8)]


@pytest.mark.parametrize("M,N,K", SMALL)
@pytest.mark.parametrize("colb", [False, True])
def test_small_shapes_vs_oracle(cuda_device, variant, M, N, K, colb):
    A, B = _inputs(M, N, K, cuda_device, seed=M + N + K)
    if colb:
        C = tg.gemm_pretransposed(A, B.t().contiguous(), mode="reg_pingpong_256_colb_mma")
    else:
        C = tg.gemm(A, B, mode="reg_pingpong_256_mma")
    torch.cuda.synchronize()
    oracle_check(C, A, B)
    _no_device_error()


BASELINE_SHAPES = [
    (2048, 2048, 2048, "uniform"),
    (16384, 256, 256, "normal"), (16384, 512, 256, "normal"), (16384, 1024, 256, "normal"),
    (32768, 256, 256, "normal"), (32768, 512, 256, "normal"), (32768, 1024, 256, "normal"),
    (4096, 4096, 4096, "uniform"), (8192, 8192, 8192, "uniform"),
    (4096, 8192, 4096, "uniform"), (8192, 4096, 4096, "uniform"), (4000, 6000, 3000, "uniform"),
]


@pytest.mark.parametrize("M,N,K,dist", BASELINE_SHAPES)
def test_baseline_configs(cuda_device, variant, M, N, K, dist):
    A, B = _inputs(M, N, K, cuda_device, dist=dist)
    ref = fp32_ref(A, B)
    assert_parity(tg.gemm(A, B, mode="reg_pingpong_256"), ref, K, f"{M}x{N}x{K} rowB")
    Bc = B.t().contiguous()
    assert_parity(tg.gemm_pretransposed(A, Bc, mode="reg_pingpong_256_colb"), ref, K, f"{M}x{N}x{K} colb")
    _no_device_error()


def test_multi_gpu_shard_shape(cuda_device, native_lib):
    # One rank's shard of the 65536 x 8192 x 8192 config at 8 GPUs (8192 rows),
    # N(0, 0.02) operands.
    A, B = _inputs(8192, 8192, 8192, cuda_device, dist="normal", std=0.02)
    assert_parity(tg.gemm(A, B), fp32_ref(A, B), 8192, "shard")
    _no_device_error()


@pytest.mark.parametrize("rows,rank", [(65536, 0), (32768, 0), (32768, 1), (16384, 3)])
def test_bench_workload_shapes(cuda_device, native_lib, rows, rank):
    """The bench's own launches: the 65536 x 8192 x 8192 workload on one GPU
    (wide pair kernel, column-band raster) and its 2- and 4-rank shards, on the
    operands bench.py generates (device generator seeded 1000 + rank for A, 1
    for B, N(0, 0.02)), through the same call, under `auto`."""
    N = K = 8192
    gA = torch.Generator(device=cuda_device).manual_seed(1000 + rank)
    gB = torch.Generator(device=cuda_device).manual_seed(1)
    A = torch.randn((rows, K), generator=gA, device=cuda_device, dtype=torch.float16) * 0.02
    B = torch.randn((K, N), generator=gB, device=cuda_device, dtype=torch.float16) * 0.02
    assert _native.plan(rows, N, K)[0] == "pair2m"
    C = torch.empty((rows, N), dtype=torch.float16, device=cuda_device)
    tg.gemm(A, B, out=C)
    torch.cuda.synchronize()
    _no_device_error()
    ref = fp32_ref(A, B)
    assert_parity(C, ref, K, f"bench workload {rows}x{N}x{K}")
    del ref
    # Run to run the launch is bit-identical.
    C2 = tg.gemm(A, B)
    torch.cuda.synchronize()
    assert torch.equal(C, C2)


def test_all_modes_agree(cuda_device, variant):
    A, B = _inputs(384, 264, 320, cuda_device)
    Bc = B.t().contiguous()
    outs = [tg.gemm(A, B, mode=m) for m in tg.KERNEL_MODES]
    outs += [tg.gemm_pretransposed(A, Bc, mode=m) for m in ("wmma", "mma", "reg_pingpong_256_colb",
                                                            "reg_pingpong_256_colb_mma")]
    # Reference quirk: ids 2/3 read the pretransposed operand as K x N.
    outs += [tg.gemm_pretransposed(A, B, mode=m) for m in ("reg_pingpong_256", "reg_pingpong_256_mma")]
    outs += [gemm_mod.root_gemm_cuda(A, B, 2), gemm_mod.root_gemm_cuda(A, Bc, 4)]
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    assert_parity(outs[0], fp32_ref(A, B), 320)


def test_deterministic(cuda_device, native_lib):
    A, B = _inputs(2048, 2048, 2048, cuda_device)
    C1 = tg.gemm(A, B)
    C2 = tg.gemm(A, B)
    assert torch.equal(C1, C2)


def test_k_zero_gives_zeros(cuda_device, native_lib):
    A = torch.empty((64, 0), dtype=torch.float16, device=cuda_device)
    B = torch.empty((0, 72), dtype=torch.float16, device=cuda_device)
    C = tg.gemm(A, B)
    assert C.shape == (64, 72) and not C.any()


def test_empty_output(cuda_device, native_lib):
    A = torch.ones((0, 64), dtype=torch.float16, device=cuda_device)
    B = torch.ones((64, 16), dtype=torch.float16, device=cuda_device)
    assert tg.gemm(A, B).shape == (0, 16)


def test_output_guard_bands_untouched(cuda_device, variant):
    """Canary: a C view inside a larger buffer; nothing outside it is written."""
    M, N, K = 200, 136, 96
    A, B = _inputs(M, N, K, cuda_device)
    ld = 256
    buf = torch.full((M + 64, ld), 7.0, dtype=torch.float16, device=cuda_device)
    view = buf[32:32 + M, 64:64 + N]
    code = _native.gemm_f16_raw(A.data_ptr(), B.data_ptr(), view.data_ptr(), M, N, K, K, N, ld,
                                _native.B200_B_ROW_MAJOR, torch.cuda.current_stream().cuda_stream)
    assert code == 0
    torch.cuda.synchronize()
    assert_parity(view, fp32_ref(A, B), K)
    mask = torch.ones_like(buf, dtype=torch.bool)
    mask[32:32 + M, 64:64 + N] = False
    assert (buf[mask] == 7.0).all(), "kernel wrote outside the output view"


@pytest.mark.parametrize("N,alpha,beta", [(1001, 1.0, 0.0), (1001, 0.5, -1.25), (5, 1.0, 0.0), (5, 2.0, 0.5),
                                           (263, 1.0, 0.0)])
def test_output_guard_columns_ragged_n(cuda_device, variant, N, alpha, beta):
    """N not a multiple of 8 inside a wider buffer: the columns right after the
    view (inside the same 16-byte piece) keep their values; alpha / beta are
    applied to the ragged last piece as to every other column."""
    M, K = 300, 192
    A, B = _inputs(M, N, K, cuda_device)
    ld = 1024
    buf = torch.full((M + 16, ld), 7.0, dtype=torch.float16, device=cuda_device)
    off = 8
    view = buf[8:8 + M, off:off + N]
    old = (torch.randn((M, N), device=cuda_device) * 0.5).half()
    view.copy_(old)
    from tensorcore_gemm.kmeans import _pitched

    Bp = _pitched(B)                            # row pitch a multiple of 8: no workspace needed
    code = _native.gemm_ex_raw(A.data_ptr(), Bp.data_ptr(), view.data_ptr(), M, N, K, K, Bp.stride(0), ld,
                               _native.B200_A_ROW_MAJOR, _native.B200_B_ROW_MAJOR, alpha, beta,
                               0, 0, torch.cuda.current_stream().cuda_stream)
    assert code == 0
    torch.cuda.synchronize()
    ref = alpha * fp32_ref(A, B) + beta * old.float()
    assert_parity(view, ref, K)
    mask = torch.ones_like(buf, dtype=torch.bool)
    mask[8:8 + M, off:off + N] = False
    assert (buf[mask] == 7.0).all(), "kernel wrote outside the output view"


def test_strided_views_without_copies(cuda_device, variant):
    """Row-strided A, and B given as a transposed view, run in place."""
    big = torch.randn((300, 512), device=cuda_device).half()
    A = big[:, 64:64 + 256]                    # lda = 512
    Bt = torch.randn((200, 256), device=cuda_device).half()
    B = Bt.t()                                 # K x N view of an N x K buffer
    C = tg.gemm(A, B)
    assert_parity(C, A.float() @ B.float(), 256)


ODD = [(1, 1, 1), (3, 5, 7), (37, 23, 41), (130, 257, 100), (257, 300, 513), (64, 9, 1000), (2049, 129, 255)]


@pytest.mark.parametrize("M,N,K", ODD)
@pytest.mark.parametrize("colb", [False, True])
def test_odd_pitches_through_workspace(cuda_device, variant, M, N, K, colb):
    """K or N not a multiple of 8: operands are re-pitched on the GPU."""
    A, B = _inputs(M, N, K, cuda_device, seed=M * 3 + N + K)
    assert tg.is_supported(A, B)
    if colb:
        C = tg.gemm_pretransposed(A, B.t().contiguous(), mode="reg_pingpong_256_colb")
    else:
        C = tg.gemm(A, B)
    torch.cuda.synchronize()
    assert C.shape == (M, N) and C.is_contiguous()
    oracle_check(C, A, B)
    _no_device_error()


def test_misaligned_storage_and_strided_output(cuda_device, variant):
    """Bases off the 16-byte grid and an output view with an odd row pitch."""
    M, N, K = 300, 200, 264
    A0, B0 = _inputs(M, N, K, cuda_device, seed=77)
    abuf = torch.empty(M * K + 1, dtype=torch.float16, device=cuda_device)
    A = abuf[1:].view(M, K)
    A.copy_(A0)
    bbuf = torch.empty(K * N + 3, dtype=torch.float16, device=cuda_device)
    B = bbuf[3:].view(K, N)
    B.copy_(B0)
    cbuf = torch.full((M, N + 5), 9.0, dtype=torch.float16, device=cuda_device)
    C = cbuf[:, 1:1 + N]
    tg.gemm(A, B, out=C)
    torch.cuda.synchronize()
    assert_parity(C, fp32_ref(A0, B0), K)
    assert (cbuf[:, 0] == 9.0).all() and (cbuf[:, 1 + N:] == 9.0).all()
    _no_device_error()


def test_workspace_abi(cuda_device, native_lib):
    """b200_gemm_f16 refuses odd pitches; the _ws entry takes them with enough workspace."""
    M, N, K = 40, 24, 36
    A, B = _inputs(M, N, K, cuda_device, seed=5)
    Abig = torch.zeros((M, 37), dtype=torch.float16, device=cuda_device)
    Abig[:, :K] = A
    C = torch.empty((M, N), dtype=torch.float16, device=cuda_device)
    s = torch.cuda.current_stream().cuda_stream
    args = (Abig.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, 37, N, N, _native.B200_B_ROW_MAJOR)
    assert _native.gemm_f16_raw(*args, s) == _native.B200_ERR_MISALIGNED
    need = _native.workspace_size(*args)
    assert need >= M * 40 * 2
    ws = torch.empty(need, dtype=torch.uint8, device=cuda_device)
    assert _native.gemm_f16_ws_raw(*args, ws.data_ptr(), need - 256, s) == _native.B200_ERR_WORKSPACE
    assert _native.gemm_f16_ws_raw(*args, ws.data_ptr(), need, s) == 0
    torch.cuda.synchronize()
    assert_parity(C, fp32_ref(A, B), K)


def test_current_stream_is_used(cuda_device, native_lib):
    A, B = _inputs(512, 512, 512, cuda_device)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        C = tg.gemm(A, B)
    s.synchronize()
    assert_parity(C, fp32_ref(A, B), 512)


def test_variants_deterministic_and_within_bound(cuda_device, native_lib):
    A, B = _inputs(1024, 1536, 2048, cuda_device)
    ref = fp32_ref(A, B)
    for v in ("cta1", "pair"):
        _native.set_variant(v)
        try:
            C1 = tg.gemm(A, B)
            C2 = tg.gemm(A, B)
        finally:
            _native.set_variant("auto")
        assert torch.equal(C1, C2)
        assert_parity(C1, ref, 2048, v)


@pytest.mark.parametrize("M,N,K,chunk", [(1000, 264, 320, 256), (4096, 512, 1024, None), (300, 24, 40, 64)])
def test_streamed_host_operands(cuda_device, native_lib, M, N, K, chunk):
    from tensorcore_gemm.streamed import gemm_streamed

    A, B = oracle.make_inputs(M, N, K, seed_a=91, seed_b=92)
    Ah, Bh = A.pin_memory(), B.pin_memory()
    C = gemm_streamed(Ah, Bh, chunk_rows=chunk)
    torch.cuda.synchronize()
    assert not C.is_cuda and C.shape == (M, N)
    assert_parity(C, A.float() @ B.float(), K)
    # B already on the device, result into a CUDA tensor
    out = torch.empty((M, N), dtype=torch.float16, device=cuda_device)
    gemm_streamed(Ah, Bh.to(cuda_device), out=out, chunk_rows=chunk)
    torch.cuda.synchronize()
    assert torch.equal(out.cpu(), C)


def test_streamed_back_to_back_calls_reuse_buffers(cuda_device, native_lib):
    """Calls queued without a sync in between share the kept device buffers:
    each call's copies and kernels must wait for the previous call's use of
    them, whatever B, outputs and chunk counts the calls have."""
    from tensorcore_gemm.streamed import gemm_streamed

    M, N, K = 3000, 512, 768
    runs = []
    for i in range(3):
        A, B = oracle.make_inputs(M, N, K, seed_a=200 + i, seed_b=300 + i)
        runs.append((A, B, A.pin_memory(), B.pin_memory()))
    outs = [torch.empty((M, N), dtype=torch.float16).pin_memory(),
            torch.empty((M, N), dtype=torch.float16, device=cuda_device),
            torch.empty((M, N), dtype=torch.float16).pin_memory()]
    for rep in range(2):
        for (A, B, Ah, Bh), out in zip(runs, outs):
            gemm_streamed(Ah, Bh, out=out, chunk_rows=512)          # 6 chunks: both buffers reused
        torch.cuda.synchronize()
        for (A, B, Ah, Bh), out in zip(runs, outs):
            assert_parity(out.cpu() if out.is_cuda else out, A.float() @ B.float(), K, f"back-to-back call, rep {rep}")


PARTIAL_WAVES = [(2048, 2048, 4096), (4096, 4096, 4096), (4000, 6000, 3000), (8192, 6144, 2048), (1536, 1280, 8192)]


@pytest.mark.parametrize("M,N,K", PARTIAL_WAVES)
@pytest.mark.parametrize("v", ["pair", "pair2m", "pair2m_224", "pair2m_192"])
def test_pair_kernels_partial_last_wave(cuda_device, native_lib, M, N, K, v):
    """Pair kernels on tile counts that leave the last wave partly idle:
    within the bound, bit-identical run to run, equal in both B layouts."""
    A, B = _inputs(M, N, K, cuda_device, dist="normal", seed=M + N)
    _native.set_variant(v)
    try:
        C1 = tg.gemm(A, B)
        C2 = tg.gemm(A, B)
        C3 = tg.gemm_pretransposed(A, B.t().contiguous(), mode="reg_pingpong_256_colb")
    finally:
        _native.set_variant("auto")
    torch.cuda.synchronize()
    _no_device_error()
    assert torch.equal(C1, C2)
    assert torch.equal(C1, C3)
    assert_parity(C1, fp32_ref(A, B), K, f"{v} {M}x{N}x{K}")


COLA = [(300, 264, 200), (1024, 512, 2048), (4096, 4096, 1024), (32768, 1024, 256), (129, 136, 72)]


@pytest.mark.parametrize("M,N,K", COLA)
@pytest.mark.parametrize("colb", [False, True])
def test_column_major_a_in_place(cuda_device, variant, M, N, K, colb):
    """A given as the transpose view of a K x M buffer is read without a copy."""
    A, B = _inputs(M, N, K, cuda_device, dist="normal", seed=M + 2 * N + K)
    At = A.t().contiguous()           # K x M storage
    Aview = At.t()                    # M x K, column-major
    assert Aview.stride(0) == 1
    if colb:
        C = tg.gemm_pretransposed(Aview, B.t().contiguous(), mode="reg_pingpong_256_colb")
    else:
        C = tg.gemm(Aview, B)
    torch.cuda.synchronize()
    _no_device_error()
    assert torch.equal(C, tg.gemm(A, B)), "column-major A must give the row-major result bit for bit"
    assert_parity(C, fp32_ref(A, B), K)


@pytest.mark.parametrize("M,N,K", [(256, 512, 320), (4096, 4096, 4096), (32768, 1024, 256), (37, 24, 40)])
@pytest.mark.parametrize("alpha,beta", [(0.5, 0.0), (1.0, 1.0), (-2.0, 0.25), (0.0, 3.0)])
def test_alpha_beta_epilogue(cuda_device, variant, M, N, K, alpha, beta):
    gemm_ex = gemm_mod.gemm_ex
    A, B = _inputs(M, N, K, cuda_device, dist="normal", seed=M + K)
    C0 = (torch.randn((M, N), device=cuda_device) * 4).half()
    out = C0.clone()
    gemm_ex(A, B, out=out, alpha=alpha, beta=beta)
    torch.cuda.synchronize()
    _no_device_error()
    ref = alpha * fp32_ref(A, B) + beta * C0.float()
    assert_parity(out, ref, K, f"alpha={alpha} beta={beta}")


def test_alpha_beta_odd_output_pitch_and_empty_k(cuda_device, native_lib):
    gemm_ex = gemm_mod.gemm_ex
    M, N, K = 100, 37, 72                 # N odd: C goes through the re-pitch workspace
    A, B = _inputs(M, N, K, cuda_device, seed=3)
    C0 = torch.randn((M, N), device=cuda_device).half()
    out = C0.clone()
    gemm_ex(A, B, out=out, alpha=1.5, beta=-0.5)
    assert_parity(out, 1.5 * fp32_ref(A, B) + (-0.5) * C0.float(), K)
    E = torch.empty((M, 0), dtype=torch.float16, device=cuda_device)
    F = torch.empty((0, N), dtype=torch.float16, device=cuda_device)
    out2 = C0.clone()
    gemm_ex(E, F, out=out2, alpha=1.0, beta=2.0)  # K = 0: C = 2 C
    torch.cuda.synchronize()
    assert torch.equal(out2, (2.0 * C0.float()).half())


def test_column_major_a_odd_pitch_abi(cuda_device, native_lib):
    """C ABI: column-major A whose pitch is odd goes through the workspace."""
    M, N, K = 203, 64, 96
    A, B = _inputs(M, N, K, cuda_device, seed=8)
    buf = torch.zeros((K, M + 3), dtype=torch.float16, device=cuda_device)   # lda = M + 3 (odd)
    buf[:, :M] = A.t()
    C = torch.empty((M, N), dtype=torch.float16, device=cuda_device)
    args = (buf.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, M + 3, N, N,
            _native.B200_A_COL_MAJOR, _native.B200_B_ROW_MAJOR)
    need = _native.workspace_size_ex(*args)
    assert need > 0
    ws = torch.empty(need, dtype=torch.uint8, device=cuda_device)
    rc = _native.gemm_ex_raw(*args, 1.0, 0.0, ws.data_ptr(), need, torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert_parity(C, fp32_ref(A, B), K)


def test_call_from_a_fresh_host_thread(cuda_device, native_lib):
    """A thread that has made no CUDA runtime call yet (autograd's device thread
    is one) has no current context for the tensor-map encoder; the library
    makes the device's primary context current and the call succeeds."""
    import threading

    A, B = _inputs(256, 320, 512, cuda_device)
    out = {}

    def work():
        try:
            out["C"] = tg.gemm(A, B)
            torch.cuda.synchronize()
        except Exception as exc:  # noqa: BLE001 - reported below
            out["err"] = exc

    t = threading.Thread(target=work)
    t.start()
    t.join(60)
    assert "err" not in out, out.get("err")
    assert_parity(out["C"], fp32_ref(A, B), 512, "fresh thread")
    _no_device_error()


_DYN_CHILD = r"""
import sys
sys.path[:0] = [sys.argv[1], sys.argv[1] + '/ampere-gemm_b200']
import torch, tensorcore_gemm as tg
from tensorcore_gemm import _native
g = torch.Generator(device='cuda').manual_seed(9)
A = (torch.randn((8192, 2048), generator=g, device='cuda') * 0.05).half()
B = (torch.randn((2048, 4096), generator=g, device='cuda') * 0.05).half()
_native.set_variant('pair2m')
C = tg.gemm(A, B)
torch.cuda.synchronize()
assert _native.last_device_error() == 0
torch.save(C.cpu(), sys.argv[2])
"""


def test_dynamic_and_static_tile_order_agree(cuda_device, native_lib, tmp_path):
    """The wide pair kernel's dynamic tile scheduling (cluster launch control,
    the default for multi-wave launches) and its static round-robin order give
    bit-identical results: each tile is computed once, the same way."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    repo = str(Path(__file__).resolve().parent.parent)
    outs = {}
    for dyn in ("1", "0"):
        out = tmp_path / f"c{dyn}.pt"
        env = dict(os.environ, B200_GEMM_DYN=dyn)
        r = subprocess.run([sys.executable, "-c", _DYN_CHILD, repo, str(out)], env=env, capture_output=True,
                           text=True, timeout=300)
        assert r.returncode == 0, r.stderr[-2000:]
        outs[dyn] = torch.load(out)
    assert torch.equal(outs["1"], outs["0"])

