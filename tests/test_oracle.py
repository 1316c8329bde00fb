"""CPU tests of the oracle: pinned against the reference's own code and fixtures."""
import json
import os

import numpy as np
import pytest

import oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_f16_conversion_matches_numpy_all_halves():
    # every binary16 value survives f16 -> f32 -> f16 and matches numpy's widening
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    f = O.f16_to_f32(h)
    ref = h.view(np.float16).astype(np.float32)
    nan = np.isnan(ref)
    assert np.array_equal(f.view(np.uint32)[~nan], ref.view(np.uint32)[~nan])
    assert np.all(np.isnan(f[nan]))
    back = O.f32_to_f16(f)
    assert np.array_equal(back[~nan], h[~nan])


def test_f16_rounding_matches_numpy_random():
    rng = np.random.default_rng(7)
    x = np.concatenate([rng.standard_normal(100000).astype(np.float32) * s
                        for s in (1e-7, 1e-5, 1e-3, 1.0, 3e4, 6.6e4)]).astype(np.float32)
    with np.errstate(over="ignore"):
        ref = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(O.f32_to_f16(x), ref)


def test_float2half_golden_from_reference():
    """Fixture made by the reference's host __float2half (tests/golden/gen_golden.py)."""
    pairs = np.array(json.load(open(os.path.join(GOLDEN, "float2half.json"))), np.uint64)
    f = pairs[:, 0].astype(np.uint32).view(np.float32)
    assert np.array_equal(O.f32_to_f16(f), pairs[:, 1].astype(np.uint16))


def _golden_inputs(case):
    M, N, K = case["M"], case["N"], case["K"]
    if case["init"] == "lcg":
        return O.fill_lcg(M, N, K)
    _, seed, lo, hi = case["init"].split(":")
    seed, lo, hi = int(seed), float(lo), float(hi)
    return (O.fill_uniform((M, K), seed, 0, lo, hi), O.fill_uniform((N, K), seed, 1, lo, hi),
            O.fill_uniform((N,), seed, 2, lo, hi))


@pytest.mark.parametrize("idx", range(9))
def test_spot_check_golden_from_reference(idx):
    """The restated cpu_spot_check reproduces the reference's own answers exactly."""
    case = json.load(open(os.path.join(GOLDEN, "spot_check.json")))[idx]
    A, B, bias = _golden_inputs(case)
    R = O.gemm_f64(A, B)
    if case["fused"]:
        R = np.maximum(R * case["alpha"] + O.f16_to_f32(bias)[None, :].astype(np.float64), 0.0)
    D = O.f32_to_f16(R.astype(np.float32))
    for m, n, x in case["plants"]:
        D[m, n] ^= x
    w, wm, wn = O.spot_check(A, B, D, bias, case["samples"], bool(case["fused"]), case["alpha"])
    assert (w, wm, wn) == (case["worst"], case["worst_m"], case["worst_n"])


@pytest.mark.skipif(not O.ref_available(), reason="reference library not built")
def test_spot_check_matches_reference_live():
    A, B, bias = O.fill_lcg(80, 72, 96)
    D = O.f32_to_f16(O.gemm_f64(A, B).astype(np.float32))
    D[17, 3] ^= 0x0300
    for samples in (1, 13, 100, 5760, 9000):
        for fused in (False, True):
            assert O.spot_check(A, B, D, bias, samples, fused, 0.75) == \
                O.ref_spot_check(A, B, D, bias, samples, fused, 0.75)


def test_lcg_values():
    """LCG restatement (src/gemm_bench.cu:760-765): first draws in closed form."""
    A, B, bias = O.fill_lcg(1, 2, 3)
    s = 12345
    vals = []
    for _ in range(3 + 6 + 2):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        vals.append(np.float32(((s >> 16) & 1023)) / np.float32(1023.0) - np.float32(0.5))
    expect = np.array(vals, np.float32).astype(np.float16).view(np.uint16)
    got = np.concatenate([A.reshape(-1), B.reshape(-1), bias])
    assert np.array_equal(got, expect)
    # 1024 levels in [-0.5, 0.5]
    A, B, _ = O.fill_lcg(64, 64, 64)
    v = O.f16_to_f32(A)
    assert v.min() >= -0.5 and v.max() <= 0.5 and len(np.unique(v)) > 500


def test_uniform_generator_range_and_determinism():
    a = O.fill_uniform((1000,), 3, 0, -1.0, 1.0)
    b = O.fill_uniform((1000,), 3, 0, -1.0, 1.0)
    c = O.fill_uniform((1000,), 3, 1, -1.0, 1.0)
    assert np.array_equal(a, b) and not np.array_equal(a, c)
    v = O.f16_to_f32(a)
    assert v.min() >= -1.0 and v.max() <= 1.0 and abs(v.mean()) < 0.1


def test_gemm_references_agree():
    A = O.fill_uniform((70, 50), 0, 0)
    B = O.fill_uniform((60, 50), 0, 1)
    R64 = O.gemm_f64(A, B)
    R32 = O.gemm_f32_naive(A, B)
    Rb, threads = O.gemm_f32_blocked(A, B)
    assert threads >= 1
    assert np.max(np.abs(R32 - R64)) < 1e-4
    assert np.max(np.abs(Rb - R64)) < 1e-4
    # K x N layout of the same B gives the same product
    BT = np.ascontiguousarray(B.T)
    assert np.array_equal(O.gemm_f64(A, BT, b_layout=1), R64)
    # row range
    assert np.array_equal(O.gemm_f64(A, B, 0, 10, 30), R64[10:30])


def test_metrics():
    A = O.fill_uniform((32, 32), 1, 0)
    B = O.fill_uniform((32, 32), 1, 1)
    R = O.gemm_f64(A, B)
    D = O.f32_to_f16(R.astype(np.float32))
    assert O.frobenius_rel(D, R) < 5e-4
    assert O.max_rel_diff(D, D) == 0.0
    D2 = D.copy()
    D2[0, 0] = O.f32_to_f16(np.array([O.f16_to_f32(D[0:1, 0])[0] + 2.0], np.float32))[0]
    assert O.max_rel_diff(D2, D) > 0.5


def test_tile_coord_restatement_is_a_bijection():
    for tm, tn, g in [(1, 1, 1), (7, 5, 1), (7, 5, 2), (7, 5, 3), (32, 16, 8), (33, 17, 16),
                      (3, 100, 16)]:
        seen = set()
        for t in range(tm * tn):
            m, n = O.tile_coord(t, tm, tn, g)
            assert 0 <= m < tm and 0 <= n < tn
            seen.add((m, n))
        assert len(seen) == tm * tn


def test_epilogue_and_bias_relu():
    acc = np.array([[-1.0, 0.25, 3.0], [2.0, -0.5, 0.0]], np.float32)
    bias = O.f32_to_f16(np.array([0.5, -1.0, 0.0], np.float32))
    out = O.f16_to_f32(O.epilogue(acc, bias, alpha=2.0))
    assert np.array_equal(out, np.array([[0.0, 0.0, 6.0], [4.5, 0.0, 0.0]], np.float32))
    D = O.f32_to_f16(acc)
    assert np.array_equal(O.bias_relu(D, bias, 2.0), O.epilogue(acc, bias, 2.0))
