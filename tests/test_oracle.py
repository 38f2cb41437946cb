"""CPU: pin the oracle to the reference's own functions (golden fixtures made
by tests/golden/make_golden.py from fp8_gemm_task_harness.py on CPU torch)."""

from __future__ import annotations

import numpy as np
import pytest


def test_decode_table_matches_torch(oracle):
    g = np.load(__import__("conftest").GOLDEN / "e4m3_codes.npz")
    d, t = g["decoded"], oracle.e4m3_decode_table()
    assert np.array_equal(np.isnan(d), np.isnan(t))
    ok = ~np.isnan(d)
    assert np.array_equal(d[ok].view(np.uint32), t[ok].view(np.uint32))


def test_encoder_matches_torch_bit_exact(oracle):
    g = np.load(__import__("conftest").GOLDEN / "e4m3_codes.npz")
    codes = oracle.f32_to_e4m3(g["probe"])
    assert np.array_equal(codes, g["probe_codes"])


def test_encoder_ties_to_even(oracle):
    # 17 lies between 16 (mantissa 000) and 18 (001): ties go to 16.
    # 19 lies between 18 (001) and 20 (010): ties go to 20.
    c = oracle.f32_to_e4m3(np.float32([17.0, 19.0, -17.0, 2.0 ** -10, 3 * 2.0 ** -10]))
    v = oracle.e4m3_to_f32(c)
    assert list(v) == [16.0, 20.0, -16.0, 0.0, 2.0 ** -8]


def test_encoder_rejects_out_of_range(oracle):
    with pytest.raises(ValueError):
        oracle.f32_to_e4m3(np.float32([449.0]))
    with pytest.raises(ValueError):
        oracle.f32_to_e4m3(np.float32([np.nan]))


def test_quantize_matches_reference(oracle, golden_cases):
    n = 0
    for c in golden_cases:
        if "a" not in c:
            continue
        aq, sa = oracle.quantize_per_tensor(c["a"])
        wq, sw = oracle.quantize_per_tensor(c["w"])
        assert np.array_equal(aq, c["aq"]) and np.array_equal(wq, c["wq"])
        assert sa.view(np.uint32)[0] == c["sa"].view(np.uint32)[0]
        assert sw.view(np.uint32)[0] == c["sw"].view(np.uint32)[0]
        n += 1
    assert n >= 3


def test_reference_matches_reference(oracle, golden_cases):
    for c in golden_cases:
        for fn in (oracle.reference, oracle.reference_f64):
            ref = fn(c["aq"], c["wq"], c["alpha"])
            rel = np.max(np.abs(ref - c["ref"]) / np.maximum(np.abs(c["ref"]), 1.0))
            assert rel < 1e-5, (c["m"], c["k"], c["n"], rel)


def test_bf16_rounding_matches_torch(oracle, golden_cases):
    for c in golden_cases:
        assert np.array_equal(oracle.bf16_round(c["ref"]), c["ref_bf16"])
        # and the BF16 oracle output passes the bar it defines
        assert oracle.max_rel_err(oracle.bf16_to_f32(c["ref_bf16"]), c["ref"]) <= oracle.MAX_REL_TOL


def test_bf16_round_edge_cases(oracle):
    x = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -0.0, np.inf, 3.0e38], dtype=np.float32)
    b = oracle.bf16_round(x)
    assert list(b[:4]) == [0x3F80, 0x3F80, 0x3F82, 0x8000]
    assert b[4] == 0x7F80 and b[5] == 0x7F62


def test_metrics(oracle):
    ref = np.float32([[0.5, 2.0, -100.0]])
    out = np.float32([[0.5 + 1e-3, 2.0 * (1 + 3e-3), -100.0 * (1 - 0.03)]])
    assert abs(oracle.max_rel_err(out, ref) - 0.03) < 1e-6
    assert oracle.mismatches(out, ref) == 1
    assert oracle.mismatches(np.float32([[np.nan]]), np.float32([[1.0]])) == 1
    assert oracle.harness_bar(3.9e-3, 3.9e-3) and not oracle.harness_bar(1e-2, 3.9e-3)


@pytest.mark.parametrize("dist", ["harness", "normal", "uniform", "student_t3"])
def test_make_case_distributions(oracle, dist):
    xq, wq, sx, sw, alpha = oracle.make_case(3, 4096, 64, seed=1, dist=dist)
    assert xq.dtype == np.uint8 and wq.shape == (64, 4096)
    # per-tensor scaling puts the largest magnitude exactly at 448
    assert np.max(np.abs(oracle.e4m3_to_f32(xq))) == 448.0
    assert np.max(np.abs(oracle.e4m3_to_f32(wq))) == 448.0
    assert alpha[0] == np.float32(sx[0] * sw[0])


def test_oracle_is_exact_against_float64(oracle):
    """reference_f64 is the correctly rounded sum; FP32 reference is close."""
    xq, wq, _, _, alpha = oracle.make_case(9, 6144, 96, seed=2, dist="harness")
    a = oracle.reference_f64(xq, wq, alpha)
    b = oracle.reference(xq, wq, alpha)
    # FP32 summation of the spiky harness data cancels heavily: ~2e-5 drift.
    assert oracle.max_rel_err(b, a) < 1e-4
    exp = oracle.expected_bf16(xq, wq, alpha)
    assert oracle.max_rel_err(oracle.bf16_to_f32(exp), a) <= oracle.MAX_REL_TOL
