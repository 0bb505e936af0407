"""Shared fixtures: the CUDA library binding (mx-kmeans_b200/mxk.py), the CPU
oracle (oracle/oracle.py) and helpers.  Tests that need a GPU are marked `gpu`."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# The reference checkout, when present, sits beside this repository (override
# with MXK_REFERENCE); only the tests that rebuild oracle/_ref need it.
REFERENCE_DIR = os.environ.get("MXK_REFERENCE", os.path.join(os.path.dirname(ROOT), "reference"))
for sub in ("mx-kmeans_b200", "oracle"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def orc():
    import oracle
    oracle.lib()
    return oracle


@pytest.fixture(scope="session")
def mxk():
    import mxk as m
    m.load()
    return m


@pytest.fixture(scope="session")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def rng(seed=0):
    return np.random.default_rng(seed)


def reference_fixture_a(m=131, d=256):
    """tests/cuda_checks.cu:37-41: sin(row*17+j) * 2^((row + j/32) % 9 - 4)"""
    row = np.arange(m, dtype=np.float32)[:, None]
    j = np.arange(d)[None, :]
    return (np.sin((row * 17 + j).astype(np.float32)) *
            np.ldexp(np.float32(1.0), ((np.arange(m)[:, None] + j // 32) % 9 - 4))).astype(np.float32)


def reference_fixture_b(n=132, d=256):
    """tests/cuda_checks.cu:42-44: cos(row*7+j) * 2^((row*2 + j/32) % 7 - 3)"""
    row = np.arange(n, dtype=np.float32)[:, None]
    j = np.arange(d)[None, :]
    return (np.cos((row * 7 + j).astype(np.float32)) *
            np.ldexp(np.float32(1.0), ((np.arange(n)[:, None] * 2 + j // 32) % 7 - 3))).astype(np.float32)


def blobs(n, d, k, seed, spread=10.0, sigma=1.0, pad_to=128):
    """Seeded Gaussian blobs, zero-padded to a multiple of pad_to features."""
    g = np.random.default_rng(seed)
    centers = g.uniform(-spread, spread, size=(k, d)).astype(np.float32)
    lab = g.integers(0, k, size=n)
    x = centers[lab] + g.normal(0, sigma, size=(n, d)).astype(np.float32)
    dp = (d + pad_to - 1) // pad_to * pad_to
    out = np.zeros((n, dp), np.float32)
    out[:, :d] = x
    return out


def assert_centroids_close(cg, co, rtol=1e-4):
    """Centroids within rtol relative: per centroid, |c_gpu - c_oracle| <= rtol |c_oracle|."""
    err = np.linalg.norm(np.asarray(cg, np.float64) - co, axis=1)
    lim = rtol * np.linalg.norm(np.asarray(co, np.float64), axis=1) + 1e-6
    assert np.all(err <= lim), f"{int((err > lim).sum())} centroids differ by more than {rtol} relative"


def gap_band_mismatches(orc, x, centroids, labels, fp32=False, tol=1e-5):
    """North-star label rule for one assignment step: the labels a step assigned
    against `centroids` may differ from the oracle's only where the oracle's
    nearest and second-nearest distances are within tol of the distance scale
    (|x|^2 + max |c|^2).  MX steps use the oracle's MX products
    (src/kernels/gemm.cu + assignment.cu), FP32 steps its FP32 products
    (gemm.cu:365-380).  Asserts the rule; returns the number of differing labels."""
    x = np.ascontiguousarray(x, np.float32)
    pn = orc.l2_norm(x)
    cn = orc.l2_norm(centroids)
    if fp32:
        dots = orc.gemm_f32(x, centroids).astype(np.float32)
        lo, _ = orc.assign_clusters(pn, cn, dots)
    else:
        _, _, lo, dots = orc.lloyd_step(x, pn, centroids, want_dots=True)
    _, first, second = orc.top2(pn, cn, dots)
    diff = np.asarray(labels) != lo
    scale = pn + cn.max()
    bad = diff & ((second - first) > tol * scale)
    assert not bad.any(), (f"{int(bad.sum())} labels differ from the oracle with a top-2 gap above "
                           f"{tol} of the distance scale (first rows {np.flatnonzero(bad)[:8].tolist()})")
    return int(diff.sum())


def traced_run(torch, mxk, x, c0, iterations, tolerance=0.0, fp32_iterations=0, cache_points=False):
    """One Lloyd call on cuda:0 with the per-iteration trace armed.
    -> (iterations run, final centroids, final labels, centroids [it][k][d] each
    iteration assigned against, labels [it][n] each iteration assigned, group
    sizes [it][3]) as numpy arrays."""
    dev = "cuda:0"
    xt = x if isinstance(x, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    ct = (c0.clone() if isinstance(c0, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(c0)).to(dev))
    n, k, d = xt.shape[0], ct.shape[0], ct.shape[1]
    tc = torch.zeros((iterations, k, d), dtype=torch.float32, device=dev)
    tl = torch.full((iterations, n), -1, dtype=torch.int32, device=dev)
    tg = torch.zeros((iterations, 3), dtype=torch.int32, device=dev)
    lab = torch.full((n,), -1, dtype=torch.int32, device=dev)
    mxk.trace_next_call(iterations, tc, tl, tg)
    it = mxk.kmeans_mixed(xt, ct, lab, mxk.Options(max_iterations=iterations, tolerance=tolerance,
                                                   fp32_iterations=fp32_iterations), cache_points=cache_points)
    torch.cuda.synchronize()
    return it, ct.cpu().numpy(), lab.cpu().numpy(), tc.cpu().numpy(), tl.cpu().numpy(), tg.cpu().numpy()
