"""Host-side arithmetic of bench.py (no GPU): the update pass's HBM roofline
from CUDA-event kernel times, the GEMM traffic read from the committed ncu
summary, and the peak denominators."""
import os
import sys

import pytest

from conftest import ROOT

sys.path.insert(0, ROOT)
import bench  # noqa: E402


def test_update_roofline_arithmetic():
    rows = bench.N_POINTS
    stats = {"accumulate_runs": (100, 71.882), "mx_gemm_argmin": (100, 312.5)}
    r = bench.update_roofline(stats, rows, bench.D_PAD, 6535.4)
    per_launch = rows * (4.0 * bench.D_PAD + 8.0)
    assert r["algorithmic_bytes_per_launch"] == per_launch
    assert r["achieved"] == pytest.approx(per_launch * 100 / 0.071882 / 1e9)
    assert r["frac"] == pytest.approx(r["achieved"] / 6535.4)
    assert r["unit"] == "GB/s" and r["bound"] == "hbm" and r["launches"] == 100
    assert r["ms_per_launch"] == pytest.approx(0.71882)
    # the privatised variant counts as the same pass
    r2 = bench.update_roofline({"accumulate_private": (10, 7.1882)}, rows, bench.D_PAD, 6535.4)
    assert r2["achieved"] == pytest.approx(r["achieved"])


def test_update_roofline_absent():
    assert bench.update_roofline({}, 1000, 128, 6535.4) is None
    assert bench.update_roofline({"accumulate_runs": (0, 0.0)}, 1000, 128, 6535.4) is None
    assert bench.quantize_roofline({}, 1000, 128, 6535.4, 1) is None  # fused into the GEMM at D = 128


def test_measured_traffic_and_peaks():
    head = bench.CONFIGS[bench.HEADLINE]
    t = bench.measured_traffic(bench.N_POINTS, head)
    assert t is not None and t > 0
    assert bench.measured_traffic(bench.N_POINTS // 2, head) == pytest.approx(t / 2)
    assert bench.measured_traffic(bench.N_POINTS, bench.CONFIGS[2]) is None
    pk, kind = bench.peaks()
    assert kind in ("measured", "fallback")
    assert pk["hbm_gbs"] > 0 and pk.get("bf16_tflops_sustained", pk.get("bf16_tflops")) > 0
    assert os.path.exists(os.path.join(ROOT, "profiles", "mx_gemm_argmin_config4.md"))


def test_quantize_roofline_arithmetic():
    rows, d = 4194304, 256
    # 30 iterations ran, 10 more were enqueued after the stop (no-op launches)
    r = bench.quantize_roofline({"quantize_points": (40, 30 * 0.9 + 10 * 0.003)}, 30 * rows, d, 6535.4, 30)
    per_iteration = rows * (5.0 * d + d / 32.0 + 4.0)
    assert r["algorithmic_bytes_per_iteration"] == per_iteration
    assert r["achieved"] == pytest.approx(30 * per_iteration / (27.03e-3) / 1e9)
    assert r["frac"] == pytest.approx(r["achieved"] / 6535.4)


def test_config_table_matches_baseline():
    """bench.CONFIGS[1..4] carry BASELINE.json configs[1..4]'s N, D, K, seed and
    iteration counts; the headline is configs[3]."""
    import json
    cfgs = json.load(open(os.path.join(ROOT, "BASELINE.json")))["configs"]
    for i, c in bench.CONFIGS.items():
        text = cfgs[i].replace(",", "")
        assert f"N={c['n']} " in text and f"K={c['k']} " in text, (i, text)
        assert f"seed {c['seed']}" in text, (i, text)
        assert f"D={c['d_raw']}" in text, (i, text)
    assert bench.HEADLINE == 3 and bench.N_POINTS == 8388608 and bench.D_PAD == 128
