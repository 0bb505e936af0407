"""Parity of the remaining ops on the GPU against the oracle: norms, point
bounds, precision, dense assignment (incl. the reference's known answers),
centroid update, shift, the FP32 product, and the reference's own CUDA test
suite (tests/cuda_checks.cu) compiled against this library."""
import os
import subprocess

import numpy as np
import pytest

from conftest import ROOT, blobs

pytestmark = pytest.mark.gpu


def _to(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda:0")


def test_l2_norm_bit_exact(torch_cuda, mxk, orc):
    torch = torch_cuda
    g = np.random.default_rng(0)
    # (up to 65536 rows with d % 4 == 0 take the row-per-thread kernel, more rows
    # with d % 128 == 0 the 32-row staged kernel, the rest the shared-memory
    # transpose)
    for n, d in [(1, 1), (33, 100), (4097, 128), (1000, 768), (70001, 132), (300, 30), (70001, 128),
                 (65601, 256)]:
        x = (g.standard_normal((n, d)) * 10).astype(np.float32)
        out = torch.empty(n, dtype=torch.float32, device="cuda:0")
        mxk.compute_l2_norm(_to(torch, x), out)
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy().view(np.uint32), orc.l2_norm(x).view(np.uint32))


def test_point_bounds_and_precision(torch_cuda, mxk, orc):
    torch = torch_cuda
    g = np.random.default_rng(1)
    n, d = 1000, 256
    x = (g.standard_normal((n, d)) * np.exp2(g.integers(-8, 8, size=(n, d // 32))).repeat(32, axis=1)).astype(np.float32)
    nt = torch.empty(n, dtype=torch.float32, device="cuda:0")
    xt = _to(torch, x)
    mxk.compute_l2_norm(xt, nt)
    upper = torch.empty(((n + 31) // 32) * 96, dtype=torch.float32, device="cuda:0")
    mxk.precompute_point_bounds(xt, nt, upper)
    torch.cuda.synchronize()
    exp = orc.point_bounds(x, orc.l2_norm(x))
    got = upper.cpu().numpy()
    valid = np.zeros_like(exp, dtype=bool)
    for p in range(n):
        valid[(p // 32) * 96 + p % 32 + np.array([0, 32, 64])] = True
    assert np.array_equal(got[valid].view(np.uint32), exp[valid].view(np.uint32))
    prec = torch.empty(n, dtype=torch.int32, device="cuda:0")
    for gap in (0.0, 1e6):
        gaps = torch.full((n,), gap, dtype=torch.float32, device="cuda:0")
        mxk.assign_precisions(n, d, upper, gaps, 1.0, 0.0, prec)
        torch.cuda.synchronize()
        assert np.all(prec.cpu().numpy() == 8), "MXFP8 override (include/precision.hpp:20-26)"


def test_bound_quirks(torch_cuda, mxk, orc):
    """tests/cuda_checks.cu:111-133: the error scan skips feature 0 of each block;
    the FP6 estimate uses E3M2."""
    torch = torch_cuda
    rows, d = 35, 128
    x = np.zeros((rows, d), np.float32)
    x[:, 0], x[:, 1] = 1.3, 6.0
    nt = torch.empty(rows, dtype=torch.float32, device="cuda:0")
    up = torch.empty(((rows + 31) // 32) * 96, dtype=torch.float32, device="cuda:0")
    xt = _to(torch, x)
    mxk.compute_l2_norm(xt, nt)
    mxk.precompute_point_bounds(xt, nt, up)
    torch.cuda.synchronize()
    u, pn = up.cpu().numpy(), nt.cpu().numpy()
    for r in range(rows):
        assert u[(r // 32) * 96 + 64 + r % 32] == pn[r]
    x[:, 0], x[:, 1] = 6.0, 1.4
    xt = _to(torch, x)
    mxk.compute_l2_norm(xt, nt)
    mxk.precompute_point_bounds(xt, nt, up)
    torch.cuda.synchronize()
    u, pn = up.cpu().numpy(), nt.cpu().numpy()
    e3m2 = float(orc.decode(orc.E3M2, orc.encode(orc.E3M2, np.array([1.4], np.float32)))[0]) - np.float32(1.4)
    for r in range(rows):
        assert abs(u[(r // 32) * 96 + 32 + r % 32] - (pn[r] + d * e3m2 * e3m2)) < 1e-4


def test_assign_known_answers(torch_cuda, mxk):
    """tests/cuda_checks.cu:96-109 (distances {100,4,9,200,1,40,30,20})."""
    torch = torch_cuda
    rows, k = 35, 8
    dist = np.array([100, 4, 9, 200, 1, 40, 30, 20], np.float32)
    dots = np.tile(-0.5 * dist, (rows, 1)).astype(np.float32)
    z = torch.zeros(rows, device="cuda:0")
    zc = torch.zeros(k, device="cuda:0")
    lab = torch.empty(rows, dtype=torch.int32, device="cuda:0")
    gap = torch.empty(rows, dtype=torch.float32, device="cuda:0")
    mxk.assign_clusters(rows, k, z, zc, _to(torch, dots), lab, gap)
    torch.cuda.synchronize()
    assert np.all(lab.cpu().numpy() == 4) and np.all(gap.cpu().numpy() == 100)
    dots[:, 1] = -0.5
    mxk.assign_clusters(rows, k, z, zc, _to(torch, dots), lab, gap)
    torch.cuda.synchronize()
    assert np.all(lab.cpu().numpy() == 1) and np.all(gap.cpu().numpy() == 100)


def test_assign_random_bit_exact(torch_cuda, mxk, orc):
    torch = torch_cuda
    g = np.random.default_rng(3)
    rows, k = 3000, 300
    dots = (g.standard_normal((rows, k)) * 5).astype(np.float32)
    dots[:, 7] = dots[:, 3]  # exact ties
    pn = g.uniform(0, 50, rows).astype(np.float32)
    cn = g.uniform(0, 50, k).astype(np.float32)
    pid = g.permutation(rows).astype(np.int32)
    for p in (None, pid):
        lab = torch.empty(rows, dtype=torch.int32, device="cuda:0")
        gap = torch.empty(rows, dtype=torch.float32, device="cuda:0")
        mxk.assign_clusters(rows, k, _to(torch, pn), _to(torch, cn), _to(torch, dots), lab, gap,
                            pid=None if p is None else _to(torch, p))
        torch.cuda.synchronize()
        el, eg = orc.assign_clusters(pn, cn, dots, p)
        assert np.array_equal(lab.cpu().numpy(), el)
        assert np.array_equal(gap.cpu().numpy().view(np.uint32), eg.view(np.uint32))


@pytest.mark.parametrize("n,d,k", [(10000, 128, 64), (200000, 128, 256), (5000, 256, 2048), (3000, 96, 20)])
def test_update_centroids(torch_cuda, mxk, orc, n, d, k):
    torch = torch_cuda
    g = np.random.default_rng(n + k)
    x = (g.standard_normal((n, d)) * 3).astype(np.float32)
    lab = g.integers(0, k, n).astype(np.int32)
    lab[lab == 1] = 0  # cluster 1 empty: keeps its previous center
    old = g.standard_normal((k, d)).astype(np.float32)
    cent = torch.empty((k, d), dtype=torch.float32, device="cuda:0")
    counts = torch.empty(k, dtype=torch.int32, device="cuda:0")
    mxk.update_centroids(_to(torch, x), _to(torch, lab), _to(torch, old), cent, counts)
    torch.cuda.synchronize()
    ec, ecnt = orc.update_centroids(x, lab, old)
    assert np.array_equal(counts.cpu().numpy(), ecnt)
    got = cent.cpu().numpy()
    assert np.array_equal(got[1], old[1])
    # per-cluster sums in a different order: relative 1e-5 of the mean magnitude
    scale = np.abs(x).mean() * np.sqrt(np.maximum(ecnt, 1))[:, None] / np.maximum(ecnt, 1)[:, None]
    assert np.all(np.abs(got - ec) <= 1e-5 * (np.abs(ec) + scale) + 1e-7)


def test_centroid_shift(torch_cuda, mxk, orc):
    torch = torch_cuda
    g = np.random.default_rng(9)
    a = g.standard_normal(100003).astype(np.float32)
    b = a + g.standard_normal(100003).astype(np.float32) * 1e-3
    s = torch.empty(1, device="cuda:0")
    got = mxk.centroid_shift(_to(torch, a), _to(torch, b), s)
    exp = float(np.sum((a.astype(np.float64) - b) ** 2))
    assert abs(got - exp) <= 1e-5 * exp
    assert abs(s.item() - got) == 0


def test_gemm_fp32(torch_cuda, mxk, orc):
    torch = torch_cuda
    g = np.random.default_rng(4)
    for m, n, k in [(300, 260, 128), (129, 17, 100), (1, 1, 1)]:
        a = g.standard_normal((m, k)).astype(np.float32)
        b = g.standard_normal((n, k)).astype(np.float32)
        out = torch.empty((m, n), device="cuda:0")
        mxk.gemm_fp32(_to(torch, a), _to(torch, b), out)
        torch.cuda.synchronize()
        exp = orc.gemm_f32(a, b)
        mag = np.abs(a).astype(np.float64) @ np.abs(b).T.astype(np.float64)
        assert np.all(np.abs(out.cpu().numpy() - exp) <= 1e-6 * (1 + mag))


def test_reference_cuda_checks_binary():
    """ParCIS/MX-KMeans tests/cuda_checks.cu (its three GPU check suites),
    compiled in this container against include/kmeans.cuh + libmxkmeans.so by
    oracle/Makefile, run on the B200."""
    exe = os.path.join(ROOT, "oracle", "_ref", "cuda_checks")
    if not os.path.exists(exe):
        pytest.skip("oracle/_ref/cuda_checks was not built (needs the reference checkout)")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "CUDA checks passed" in r.stdout


def test_bounded_wait_gives_up_and_reports_timeout(torch_cuda, mxk):
    """Failure detection of the kernels' bounded waits, without a GPU fault: a
    CTA waits on an mbarrier that nothing arrives on with a limit of 10^5 cycles.
    The kernel returns (both waiting warps give up: one on its limit, one on the
    CTA's abort flag), the call reports MXK_ERR_TIMEOUT, and the error word is
    clear again for the next call."""
    torch = torch_cuda
    outcome = torch.full((2,), -1, dtype=torch.int32, device="cuda")
    assert mxk.check_wait_timeout(100000, outcome) == mxk.ERR_TIMEOUT
    assert b"timed out" in mxk.load().mxk_last_error()
    assert outcome.tolist() == [0, 0]
    # the next public call that reads the error word succeeds
    a = torch.zeros(128 * 128, dtype=torch.uint8, device="cuda")
    sa = torch.full((128 * 4,), 127, dtype=torch.uint8, device="cuda")
    out = torch.full((128, 128), -1.0, device="cuda")
    mxk.gemm_mx(8, 128, 128, 128, a, sa, a, sa, out)
    torch.cuda.synchronize()
    assert torch.count_nonzero(out).item() == 0
