"""K2 parity: tcgen05 block-scaled GEMM (dense and fused-argmin epilogues).

Reference: src/kernels/gemm.cu:348-363 checked by tests/cuda_checks.cu:75-86
(|expected - actual| <= 1e-4 (1 + sum |products|), expected = double products of
reconstructed values).  The bar here is the tighter 1e-5 relative to the
absolute-product sum; FP32 tensor-core accumulation of exact MX products stays
far inside it.
"""
import numpy as np
import pytest

from conftest import blobs, reference_fixture_a, reference_fixture_b

pytestmark = pytest.mark.gpu
GEMM_RTOL = 1e-5


def _to(torch, a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to("cuda:0")
    return t if dtype is None else t.to(dtype)


def _quantized(orc, bits, x, pid=None):
    v, s, _ = orc.quantize_rows(bits, x, pid)
    return v, s


@pytest.mark.parametrize("bits", [8, 6, 4])
def test_reference_fixture_gemm(torch_cuda, mxk, orc, bits):
    torch = torch_cuda
    a, b = reference_fixture_a(), reference_fixture_b()
    pid = np.arange(a.shape[0] - 1, -1, -1, dtype=np.int32)
    av, as_ = _quantized(orc, bits, a, pid)
    bv, bs = _quantized(orc, 8, b)
    m, n, k = a.shape[0], b.shape[0], a.shape[1]
    out = torch.zeros((m, n), dtype=torch.float32, device="cuda:0")
    mxk.gemm_mx(bits, m, n, k, _to(torch, av), _to(torch, as_), _to(torch, bv), _to(torch, bs), out)
    torch.cuda.synchronize()
    exp, mag = orc.gemm_mx(bits, av, as_, bv, bs, k)
    got = out.cpu().numpy().astype(np.float64)
    assert np.all(np.isfinite(got))
    err = np.abs(exp - got)
    assert np.all(err <= GEMM_RTOL * (1 + mag)), f"max rel err {np.max(err / (1 + mag))}"


@pytest.mark.parametrize("m,n,k", [(128, 128, 128), (1, 4, 128), (300, 260, 384), (1000, 2048, 128), (257, 136, 1024)])
def test_shapes_mxfp8(torch_cuda, mxk, orc, m, n, k):
    torch = torch_cuda
    g = np.random.default_rng(m * 7 + n)
    a = (g.standard_normal((m, k)) * 4).astype(np.float32)
    b = (g.standard_normal((n, k)) * 0.5).astype(np.float32)
    av, as_ = _quantized(orc, 8, a)
    bv, bs = _quantized(orc, 8, b)
    out = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda:0")
    mxk.gemm_mx(8, m, n, k, _to(torch, av), _to(torch, as_), _to(torch, bv), _to(torch, bs), out)
    torch.cuda.synchronize()
    exp, mag = orc.gemm_mx(8, av, as_, bv, bs, k)
    got = out.cpu().numpy().astype(np.float64)
    assert np.all(np.isfinite(got))
    assert np.all(np.abs(exp - got) <= GEMM_RTOL * (1 + mag))


def _norms(torch, mxk, x):
    xt = _to(torch, x)
    nt = torch.empty(x.shape[0], dtype=torch.float32, device="cuda:0")
    mxk.compute_l2_norm(xt, nt)
    return nt


@pytest.mark.parametrize("n,k,d", [(5000, 256, 128), (2000, 1000, 256), (777, 52, 768)])
def test_fused_argmin_matches_dense_path(torch_cuda, mxk, orc, n, k, d):
    """The fused kernel's labels/gaps equal gemm_mx (dense) + assign_clusters
    on the same inputs: same tensor-core products, same distance rule."""
    torch = torch_cuda
    x = blobs(n, d, 16, seed=n)
    c = x[np.random.default_rng(k).choice(n, k, replace=False)]
    xv, xs = _quantized(orc, 8, x)
    cv, cs = _quantized(orc, 8, c)
    pn, cn = _norms(torch, mxk, x), _norms(torch, mxk, c)
    X, XS, C, CS = _to(torch, xv), _to(torch, xs), _to(torch, cv), _to(torch, cs)
    dots = torch.empty((n, k), dtype=torch.float32, device="cuda:0")
    mxk.gemm_mx(8, n, k, d, X, XS, C, CS, dots)
    lab_dense = torch.empty(n, dtype=torch.int32, device="cuda:0")
    gap_dense = torch.empty(n, dtype=torch.float32, device="cuda:0")
    mxk.assign_clusters(n, k, pn, cn, dots, lab_dense, gap_dense)
    lab_f = torch.full((n,), -5, dtype=torch.int32, device="cuda:0")
    gap_f = torch.empty(n, dtype=torch.float32, device="cuda:0")
    mxk.assign_mx_fused(8, n, k, d, X, XS, C, CS, pn, cn, lab_f, gap_f)
    lab_ng = torch.full((n,), -5, dtype=torch.int32, device="cuda:0")
    mxk.assign_mx_fused(8, n, k, d, X, XS, C, CS, pn, cn, lab_ng, None)
    torch.cuda.synchronize()
    assert torch.equal(lab_f, lab_dense)
    assert torch.equal(lab_ng, lab_dense)
    # dense path uses pid=None (gap init -1), fused uses the -1e38 init of the MX
    # path; with k >= 2 both see the same two largest distances.
    assert torch.equal(gap_f, gap_dense)


def test_fused_argmin_vs_oracle(torch_cuda, mxk, orc):
    """Labels equal the oracle's except where its top-2 gap is below tolerance."""
    torch = torch_cuda
    n, k, d = 20000, 512, 128
    x = blobs(n, 96, 64, seed=11)
    c = x[np.random.default_rng(2).choice(n, k, replace=False)]
    xv, xs = _quantized(orc, 8, x)
    cv, cs = _quantized(orc, 8, c)
    pn_t, cn_t = _norms(torch, mxk, x), _norms(torch, mxk, c)
    lab = torch.empty(n, dtype=torch.int32, device="cuda:0")
    mxk.assign_mx_fused(8, n, k, d, _to(torch, xv), _to(torch, xs), _to(torch, cv), _to(torch, cs), pn_t, cn_t, lab)
    torch.cuda.synchronize()
    exp, _ = orc.gemm_mx(8, xv, xs, cv, cs, d)
    pn, cn = orc.l2_norm(x), orc.l2_norm(c)
    assert np.array_equal(pn, pn_t.cpu().numpy()) and np.array_equal(cn, cn_t.cpu().numpy())
    near, first, second = orc.top2(pn, cn, exp.astype(np.float32))
    got = lab.cpu().numpy()
    diff = got != near
    tol = 1e-5 * (pn[:, None] + cn[None, :]).max(axis=1)
    assert np.all((second - first)[diff] <= tol[diff]), f"{diff.sum()} labels differ outside the tie band"
    assert diff.mean() < 1e-3


def test_empty_and_tiny(torch_cuda, mxk, orc):
    torch = torch_cuda
    # m = 0 is a no-op; k = 4 centroids with one point
    mxk.gemm_mx(8, 0, 4, 128, torch.zeros(16, dtype=torch.uint8, device="cuda:0"),
                torch.zeros(16, dtype=torch.uint8, device="cuda:0"), torch.zeros(512, dtype=torch.uint8, device="cuda:0"),
                torch.zeros(16, dtype=torch.uint8, device="cuda:0"), torch.zeros(4, device="cuda:0"))
    with pytest.raises(ValueError):
        mxk.gemm_mx(8, 4, 4, 96, torch.zeros(512, dtype=torch.uint8, device="cuda:0"),
                    torch.zeros(16, dtype=torch.uint8, device="cuda:0"), torch.zeros(512, dtype=torch.uint8, device="cuda:0"),
                    torch.zeros(16, dtype=torch.uint8, device="cuda:0"), torch.zeros(16, device="cuda:0"))


@pytest.mark.parametrize("k", [136, 1000, 9000])
def test_fused_ties_and_tails(torch_cuda, mxk, orc, k):
    """Duplicated centroids (exact distance ties inside a 32-column chunk, across
    the four column quarters and across 128-column tiles) must resolve to the
    lowest index like assign_clusters; k not a multiple of 32/128 exercises the
    tail path; k > 8192 reads the centroid norms from global memory."""
    torch = torch_cuda
    n, d = 3000, 128
    g = np.random.default_rng(k)
    c = (g.standard_normal((k, d)) * 2).astype(np.float32)
    for dup in [(3, 7), (5, 40), (17, 100), (2, 131), (60, k - 1)]:
        if dup[1] < k:
            c[dup[1]] = c[dup[0]]
    x = c[g.integers(0, k, n)] + 0.01 * g.standard_normal((n, d)).astype(np.float32)
    x[:50] = c[7]  # exactly on a duplicated centroid
    xv, xs = _quantized(orc, 8, x.astype(np.float32))
    cv, cs = _quantized(orc, 8, c)
    pn, cn = _norms(torch, mxk, x.astype(np.float32)), _norms(torch, mxk, c)
    X, XS, C, CS = _to(torch, xv), _to(torch, xs), _to(torch, cv), _to(torch, cs)
    dots = torch.empty((n, k), dtype=torch.float32, device="cuda:0")
    mxk.gemm_mx(8, n, k, d, X, XS, C, CS, dots)
    lab_dense = torch.empty(n, dtype=torch.int32, device="cuda:0")
    gap_dense = torch.empty(n, dtype=torch.float32, device="cuda:0")
    mxk.assign_clusters(n, k, pn, cn, dots, lab_dense, gap_dense)
    lab_f = torch.empty(n, dtype=torch.int32, device="cuda:0")
    gap_f = torch.empty(n, dtype=torch.float32, device="cuda:0")
    mxk.assign_mx_fused(8, n, k, d, X, XS, C, CS, pn, cn, lab_f, gap_f)
    lab_ng = torch.empty(n, dtype=torch.int32, device="cuda:0")
    perm = torch.from_numpy(g.permutation(n).astype(np.int32)).to("cuda:0")
    # with a pid permutation the labels land at pid[row]; rows are then the
    # permuted points, so feed the permuted quantized rows
    Xp, XSp = X.view(n, d)[perm.long()].contiguous(), XS.view(n, d // 32)[perm.long()].contiguous()
    mxk.assign_mx_fused(8, n, k, d, Xp, XSp, C, CS, pn, cn, lab_ng, None, pid=perm)
    torch.cuda.synchronize()
    assert torch.equal(lab_f, lab_dense)
    assert torch.equal(gap_f, gap_dense)
    assert torch.equal(lab_ng, lab_dense)
    assert np.all(lab_dense.cpu().numpy()[:50] == 3)


def test_start_hint_does_not_change_results(torch_cuda, mxk, orc):
    """Labels and gaps are the same whatever tile the centroid sweep starts at:
    random hints, hints equal to the true labels, and no hint, on data with exact
    ties (duplicated centroids in different 128-centroid tiles)."""
    torch = torch_cuda
    n, d, k = 4000, 128, 640
    g = np.random.default_rng(5)
    c = (g.standard_normal((k, d)) * 2).astype(np.float32)
    c[600:] = c[:40]
    c[300:310] = c[10:20]
    x = c[g.integers(0, k, n)] + 0.05 * g.standard_normal((n, d)).astype(np.float32)
    x[:200] = c[15]
    xv, xs = _quantized(orc, 8, x.astype(np.float32))
    cv, cs = _quantized(orc, 8, c)
    pn, cn = _norms(torch, mxk, x.astype(np.float32)), _norms(torch, mxk, c)
    X, XS, C, CS = _to(torch, xv), _to(torch, xs), _to(torch, cv), _to(torch, cs)
    ref_l = torch.empty(n, dtype=torch.int32, device="cuda:0")
    ref_g = torch.empty(n, dtype=torch.float32, device="cuda:0")
    mxk.assign_mx_fused(8, n, k, d, X, XS, C, CS, pn, cn, ref_l, ref_g)
    torch.cuda.synchronize()
    hints = [torch.from_numpy(g.integers(0, k, n).astype(np.int32)).cuda(),
             ref_l.clone(),
             torch.full((n,), k - 1, dtype=torch.int32, device="cuda:0"),
             torch.full((n,), -7, dtype=torch.int32, device="cuda:0")]
    for hint in hints:
        lab = torch.empty(n, dtype=torch.int32, device="cuda:0")
        gap = torch.empty(n, dtype=torch.float32, device="cuda:0")
        mxk.assign_mx_fused(8, n, k, d, X, XS, C, CS, pn, cn, lab, gap, start_hint=hint)
        lab2 = torch.empty(n, dtype=torch.int32, device="cuda:0")
        mxk.assign_mx_fused(8, n, k, d, X, XS, C, CS, pn, cn, lab2, None, start_hint=hint)
        torch.cuda.synchronize()
        assert torch.equal(lab, ref_l) and torch.equal(lab2, ref_l)
        assert torch.equal(gap, ref_g)
    assert np.all(ref_l.cpu().numpy()[:200] == 15)
