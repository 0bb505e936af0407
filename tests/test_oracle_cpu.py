"""The oracle, pinned: against the reference's conversion library (CUTLASS +
cuda_fp6, oracle/_ref/libcutlass_pin.so), the reference's own host code and
host test binary (oracle/_ref/), its known-answer tests (tests/host_checks.cpp,
tests/cuda_checks.cu) and the committed golden vectors (tests/golden/)."""
import ctypes
import os
import subprocess

import numpy as np
import pytest

from conftest import REFERENCE_DIR, ROOT, reference_fixture_a, reference_fixture_b

GOLDEN = os.path.join(ROOT, "tests", "golden", "reference_vectors.npz")
HAVE_REF = os.path.isdir(REFERENCE_DIR)


@pytest.fixture(scope="module")
def ref_built(orc):
    if not os.path.exists(os.path.join(orc.REF_DIR, "libcutlass_pin.so")):
        if not HAVE_REF:
            pytest.skip("oracle/_ref not built and the reference checkout is absent")
        orc.build_ref()
    return orc


def _sweep():
    """Dense sample of float32: every exponent from 2^-37..2^42 with the top 12
    mantissa bits and edge low bits, both signs, plus random patterns and specials."""
    exps = np.arange(90, 170, dtype=np.uint32)
    hi = np.arange(0, 1 << 12, dtype=np.uint32) << 11
    lows = np.array([0, 1, 0x3FF, 0x400, 0x401, 0x7FF], dtype=np.uint32)
    bits = ((exps[:, None, None] << 23) | hi[None, :, None] | lows[None, None, :]).ravel()
    rnd = np.random.default_rng(0).integers(0, 2 ** 32, 1 << 20, dtype=np.uint64).astype(np.uint32)
    special = np.array([0, 0x80000000, 1, 0x80000001, 0x007FFFFF, 0x00400000, 0x00400001, 0x7F7FFFFF],
                       dtype=np.uint32)
    allb = np.concatenate([bits, bits | 0x80000000, rnd, special])
    x = allb.view(np.float32)
    return x[np.isfinite(x)]


@pytest.mark.parametrize("fmt", [0, 1, 2, 3, 4])
def test_conversions_match_cutlass(ref_built, fmt):
    orc = ref_built
    pin = orc.ref_lib("libcutlass_pin.so")
    x = _sweep()
    if fmt == orc.UE8M0:
        x = np.abs(x)
    got = orc.encode(fmt, x)
    exp = np.empty(x.size, np.uint8)
    pin.pin_encode(ctypes.c_int(fmt), ctypes.c_int64(x.size), ctypes.c_void_p(x.ctypes.data),
                   ctypes.c_void_p(exp.ctypes.data))
    bad = np.nonzero(got != exp)[0]
    assert bad.size == 0, f"{bad.size} mismatches, first x={x[bad[:4]]} oracle={got[bad[:4]]} cutlass={exp[bad[:4]]}"
    codes = np.arange(256 if fmt in (0, 4) else (64 if fmt in (1, 3) else 16), dtype=np.uint8)
    dec = orc.decode(fmt, codes)
    ref = np.empty(codes.size, np.float32)
    pin.pin_decode(ctypes.c_int(fmt), ctypes.c_int64(codes.size), ctypes.c_void_p(codes.ctypes.data),
                   ctypes.c_void_p(ref.ctypes.data))
    same = (dec.view(np.uint32) == ref.view(np.uint32)) | (np.isnan(dec) & np.isnan(ref))
    assert same.all()


def test_scale_rule_known_values(orc):
    # UE8M0 rounds up to a power of two (CUTLASS float_ue8m0_t): 1.3 -> 2^1 byte 0x80,
    # 1.3/448 -> 2^-8 byte 0x77, 447.9 -> 2^9? no: 447.9 -> 512 = 0x88; 2^k stays.
    v = np.array([1.3, 1.3 / 448, 447.9, 1.0, 0.5, 2.0 ** 127, 3e38], np.float32)
    assert list(orc.encode(orc.UE8M0, v)) == [0x80, 0x77, 0x88, 0x7F, 0x7E, 0xFE, 0xFE]
    # -0.0 keeps its sign bit in every element format
    z = np.array([-0.0], np.float32)
    assert [orc.encode(f, z)[0] for f in (orc.E4M3, orc.E2M3, orc.E2M1)] == [0x80, 0x20, 0x8]


def test_reference_host_checks_binary(ref_built):
    exe = os.path.join(ref_built.REF_DIR, "host_checks")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and "Host checks passed" in r.stdout


def test_precision_rules_match_reference(ref_built):
    orc = ref_built
    ref = orc.ref_lib("libref_host.so")
    ref.ref_precision_candidate.argtypes = [ctypes.c_float] * 3 + [ctypes.c_int, ctypes.c_float]
    ref.ref_select_precision.argtypes = [ctypes.c_float] * 4 + [ctypes.c_int, ctypes.c_float]
    # tests/host_checks.cpp:20-26
    for gap, exp in [(1.25, 4), (0.75, 6), (0.74, 8)]:
        assert orc.precision_candidate(60, 28, 4, 4, gap) == exp == ref.ref_precision_candidate(60, 28, 4, 4, gap)
    for gap in (0.0, 0.75, 1.25, 1e6):
        for ec in (0.0, 1.0, 1e6):
            assert orc.select_precision(60, 28, 4, ec, 4, gap) == 8 == ref.ref_select_precision(60, 28, 4, ec, 4, gap)


def test_assignment_known_answers(orc):
    # tests/cuda_checks.cu:96-109 and tests/host_checks.cpp:27-39
    rows, k = 35, 8
    dist = np.array([100, 4, 9, 200, 1, 40, 30, 20], np.float32)
    dots = np.tile(-0.5 * dist, (rows, 1))
    lab, gap = orc.assign_clusters(np.zeros(rows), np.zeros(k), dots)
    assert np.all(lab == 4) and np.all(gap == 100)
    dots[:, 1] = -0.5
    lab, gap = orc.assign_clusters(np.zeros(rows), np.zeros(k), dots)
    assert np.all(lab == 1) and np.all(gap == 100)


def test_bound_quirks(orc):
    # tests/cuda_checks.cu:111-133
    rows, d = 35, 128
    x = np.zeros((rows, d), np.float32)
    x[:, 0], x[:, 1] = 1.3, 6.0
    pn = orc.l2_norm(x)
    u = orc.point_bounds(x, pn)
    assert all(u[(r // 32) * 96 + 64 + r % 32] == pn[r] for r in range(rows))
    x[:, 0], x[:, 1] = 6.0, 1.4
    pn = orc.l2_norm(x)
    u = orc.point_bounds(x, pn)
    e = float(orc.decode(orc.E3M2, orc.encode(orc.E3M2, np.array([1.4], np.float32)))[0]) - np.float32(1.4)
    assert all(abs(u[(r // 32) * 96 + 32 + r % 32] - (pn[r] + d * e * e)) < 1e-4 for r in range(rows))
    prec = orc.assign_precisions(rows, d, u, np.full(rows, 1e6, np.float32), 1.0, 0.0)
    assert np.all(prec == 8)


def test_clustering_known_answers(orc):
    # tests/cuda_checks.cu:142-168
    n, d, k = 35, 128, 4
    x = np.zeros((n, d), np.float32)
    x[:, 0] = (np.arange(n) % k) * 10
    c = np.zeros((k, d), np.float32)
    c[:, 0] = np.arange(k) * 10 + 1
    it, _, lab = orc.kmeans_mixed(x, c, max_iterations=3, tolerance=0.0)
    assert 2 <= it <= 3 and np.array_equal(lab, np.arange(n) % k)
    it, _, _ = orc.kmeans_mixed(x, c, max_iterations=1, tolerance=0.0)
    assert it == 1
    cent, counts = orc.update_centroids(x, np.zeros(n, np.int32), c)
    assert np.array_equal(cent[1:], c[1:]) and counts[0] == n


def test_golden_vectors(orc):
    g = np.load(GOLDEN)
    a, b = reference_fixture_a(), reference_fixture_b()
    pid = g["pid"]
    for bits in (4, 6, 8):
        v, s, e = orc.quantize_rows(bits, a, pid, errors=True)
        assert np.array_equal(v, g[f"q{bits}_values"])
        assert np.array_equal(s, g[f"q{bits}_scales"])
        assert np.array_equal(e.view(np.uint32), g[f"q{bits}_errors"].view(np.uint32))
    v, s, _ = orc.quantize_rows(8, b)
    assert np.array_equal(v, g["qb_values"]) and np.array_equal(s, g["qb_scales"])


def test_gemm_oracle_matches_float_reconstruction(orc):
    a = reference_fixture_a()
    b = reference_fixture_b()
    av, as_, _ = orc.quantize_rows(8, a)
    bv, bs, _ = orc.quantize_rows(8, b)
    out, mag = orc.gemm_mx(8, av, as_, bv, bs, 256)
    ad = orc.dequantize_rows(8, av, as_, 256).astype(np.float64)
    bd = orc.dequantize_rows(8, bv, bs, 256).astype(np.float64)
    assert np.allclose(out, ad @ bd.T, rtol=0, atol=1e-9 * (1 + mag.max()))


def test_lloyd_fp32_and_mixed_agree_on_separated_data(orc):
    g = np.random.default_rng(1)
    k, d = 8, 128
    centers = g.uniform(-50, 50, (k, d)).astype(np.float32)
    x = (centers[np.arange(4000) % k] + g.standard_normal((4000, d))).astype(np.float32)
    c0 = x[:k].copy()
    it1, c1, l1 = orc.kmeans_mixed(x, c0, max_iterations=20, tolerance=1e-4)
    it2, c2, l2 = orc.lloyd_fp32(x, c0, 20, 1e-4)
    assert np.array_equal(l1, l2)
    assert abs(orc.inertia(x, c1, l1) - orc.inertia(x, c2, l2)) <= 1e-4 * orc.inertia(x, c2, l2)


def test_oracle_candidate_policy_fills_every_group(orc):
    """Under policy 1 (precision_candidate's choice, include/precision.hpp:10-17)
    the oracle's loop puts points in the MXFP4, MXFP6 and MXFP8 groups once the
    first iteration has produced gaps; policy 0 (the reference) keeps one MXFP8
    group."""
    from test_precision_groups_gpu import _data
    x, c0 = _data(256)
    it, _, _, g = orc.kmeans_mixed(x, c0, max_iterations=4, tolerance=0.0, policy=1, group_sizes=True)
    assert it == 4 and np.array_equal(g[0], [0, 0, len(x)]) and np.all(g[1:] > 0)
    assert np.all(g.sum(axis=1) == len(x))
    it, _, _, g = orc.kmeans_mixed(x, c0, max_iterations=2, tolerance=0.0, policy=0, group_sizes=True)
    assert np.array_equal(g, [[0, 0, len(x)]] * 2)
