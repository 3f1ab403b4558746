"""CPU: the oracle against the reference's golden vectors and IEEE formats."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle

GOLDEN = Path(__file__).resolve().parent / "golden"


def _cases():
    meta = json.loads((GOLDEN / "gemm_golden.json").read_text())
    data = np.load(GOLDEN / "gemm_golden.npz")
    for c in meta["cases"]:
        n = c["name"]
        yield pytest.param(c, data[n + "__A"], data[n + "__B"], data[n + "__C"], id=n)


@pytest.mark.parametrize("case,A,B,C_ref", list(_cases()))
def test_oracle_matches_reference_golden(case, A, B, C_ref):
    """Oracle vs the reference's own output (its CPU path, fp16 torch.matmul)."""
    C, acc = oracle.gemm_f16(A, B, threads=4)
    same = np.mean(C.view(np.uint16) == C_ref.view(np.uint16))
    # Same fp32 accumulate + one RN rounding: bit-identical except where the
    # summation order moves a sum across a rounding boundary (long K only).
    assert same >= (1.0 if case["K"] <= 256 else 0.99), f"bit-identical fraction {same}"
    diff = np.abs(C.astype(np.float32) - C_ref.astype(np.float32)).max()
    ulp = np.abs(np.spacing(C_ref.astype(np.float16))).astype(np.float32).max()
    assert diff <= ulp, f"oracle and reference differ by more than one fp16 ulp: {diff} > {ulp}"
    # Both satisfy the hot path's acceptance bound against the fp32 product.
    assert oracle.parity_ok(C_ref, acc, case["K"])
    assert oracle.parity_ok(C, acc, case["K"])


def test_f16_to_f32_exhaustive():
    h = np.arange(65536, dtype=np.uint16).view(np.float16)
    got = oracle.f16_to_f32(h)
    want = h.astype(np.float32)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got.view(np.uint32)[~nan], want.view(np.uint32)[~nan])


def test_f32_to_f16_round_to_nearest_even():
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(400_000).astype(np.float32)
         * np.float32(2.0) ** rng.integers(-30, 18, 400_000).astype(np.float32))
    # Exact halfway cases between neighbouring fp16 values, both parities.
    h = np.arange(0x0001, 0x7BFF, 37, dtype=np.uint16).view(np.float16).astype(np.float32)
    hn = np.nextafter(h.astype(np.float16), np.float16(np.inf)).astype(np.float32)
    mids = ((h.astype(np.float64) + hn.astype(np.float64)) / 2).astype(np.float32)
    x = np.concatenate([x, mids, -mids, [0.0, -0.0, np.inf, -np.inf, 65504.0, 65520.0, 6e-8, 3e-8]]).astype(np.float32)
    with np.errstate(over="ignore"):
        want = x.astype(np.float16)
    assert np.array_equal(oracle.f32_to_f16(x).view(np.uint16), want.view(np.uint16))


def test_col_major_equals_row_major():
    A, B = oracle.make_inputs(33, 40, 72, seed_a=5, seed_b=6)
    A, B = A.numpy(), B.numpy()
    C1, _ = oracle.gemm_f16(A, B)
    C2, _ = oracle.gemm_f16(A, np.ascontiguousarray(B.T), b_col_major=True)
    assert np.array_equal(C1.view(np.uint16), C2.view(np.uint16))


def test_threads_do_not_change_result():
    A, B = oracle.make_inputs(61, 24, 100, dist="normal", seed_a=7, seed_b=8)
    C1, _ = oracle.gemm_f16(A.numpy(), B.numpy(), threads=1)
    C8, _ = oracle.gemm_f16(A.numpy(), B.numpy(), threads=8)
    assert np.array_equal(C1.view(np.uint16), C8.view(np.uint16))


def test_empty_reduction_and_empty_outputs():
    A = np.zeros((5, 0), np.float16)
    B = np.zeros((0, 7), np.float16)
    C, acc = oracle.gemm_f16(A, B)
    assert C.shape == (5, 7) and not C.any()
    C, _ = oracle.gemm_f16(np.zeros((0, 8), np.float16), np.zeros((8, 3), np.float16))
    assert C.shape == (0, 3)


def test_parity_bound_formula():
    ref = np.full((4, 4), 3.0, np.float32)
    assert oracle.parity_bound(ref, 100) == pytest.approx(2e-3 * 10 * 3.0)
    assert oracle.parity_ok(ref + 0.05, ref, 100)
    assert not oracle.parity_ok(ref + 0.07, ref, 100)
