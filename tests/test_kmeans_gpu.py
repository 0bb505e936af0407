"""Lloyd driver parity (kmeans_mixed, src/kmeans.cu:12-68) on the GPU against
the oracle and the reference's clustering checks (tests/cuda_checks.cu:142-168).

Tolerances (north star): labels identical except where a point's top-2 distance
gap is below 1e-5 of the distance scale; centroids and inertia within 1e-4
relative."""
import numpy as np
import pytest

from conftest import assert_centroids_close, blobs, gap_band_mismatches, traced_run

pytestmark = pytest.mark.gpu


def check_steps(orc, x, it, c_final, tc, tl, fp32_iterations=0):
    """Step-wise parity of a traced run: every iteration's labels against the
    oracle's assignment from the same centroids (gap-band rule), and the centroids
    the next iteration starts from against the oracle's update of those labels
    (src/kernels/update.cu:7-31: per-cluster means, empty clusters keep theirs).
    -> total number of labels inside the band that differ."""
    differing = 0
    for t in range(it):
        differing += gap_band_mismatches(orc, x, tc[t], tl[t], fp32=t < fp32_iterations)
        c_next = tc[t + 1] if t + 1 < it else c_final
        co, _ = orc.update_centroids(x, tl[t], tc[t])
        assert_centroids_close(c_next, co)
    return differing


def _to(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda:0")


def _run(torch, mxk, x, c0, **opts):
    xt, ct = _to(torch, x), _to(torch, c0)
    lab = torch.full((x.shape[0],), -1, dtype=torch.int32, device="cuda:0")
    it = mxk.kmeans_mixed(xt, ct, lab, mxk.Options(**opts))
    return it, ct.cpu().numpy(), lab.cpu().numpy()


def test_reference_clustering_checks(torch_cuda, mxk):
    torch = torch_cuda
    n, d, k = 35, 128, 4
    x = np.zeros((n, d), np.float32)
    x[:, 0] = (np.arange(n) % k) * 10
    c = np.zeros((k, d), np.float32)
    c[:, 0] = np.arange(k) * 10 + 1.0
    it, _, lab = _run(torch, mxk, x, c, max_iterations=3, tolerance=0.0)
    assert 2 <= it <= 3
    assert np.array_equal(lab, np.arange(n) % k)
    it, _, _ = _run(torch, mxk, x, c, max_iterations=1, tolerance=0.0)
    assert it == 1


def test_one_iteration_vs_oracle(torch_cuda, mxk, orc):
    torch = torch_cuda
    n, d, k = 30000, 128, 64
    x = blobs(n, 96, 40, seed=3, spread=5.0, sigma=0.75)
    c0 = x[np.random.default_rng(1).choice(n, k, replace=False)].copy()
    it, cg, lg = _run(torch, mxk, x, c0, max_iterations=1, tolerance=0.0)
    assert it == 1
    shift, co, lo, dots = orc.lloyd_step(x, orc.l2_norm(x), c0, want_dots=True)
    near, first, second = orc.top2(orc.l2_norm(x), orc.l2_norm(c0), dots)
    diff = lg != lo
    scale = orc.l2_norm(x) + orc.l2_norm(c0).max()
    assert np.all((second - first)[diff] <= 1e-5 * scale[diff])
    if not diff.any():
        assert np.allclose(cg, co, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("n,d,k,iters", [(20000, 128, 32, 8), (8000, 256, 128, 5)])
def test_full_run_vs_oracle(torch_cuda, mxk, orc, n, d, k, iters):
    torch = torch_cuda
    x = blobs(n, d, k, seed=n + d, spread=10.0, sigma=1.0)
    c0 = x[np.random.default_rng(7).choice(n, k, replace=False)].copy()
    it_g, cg, lg, tc, tl, _ = traced_run(torch, mxk, x, c0, iters, tolerance=1e-4)
    it_o, co, lo = orc.kmeans_mixed(x, c0, max_iterations=iters, tolerance=1e-4)
    ig, io = orc.inertia(x, cg, lg), orc.inertia(x, co, lo)
    assert abs(ig - io) <= 1e-4 * io
    assert np.array_equal(tl[it_g - 1], lg)
    # every iteration: labels by the gap-band rule, next centroids within 1e-4
    differing = check_steps(orc, x, it_g, cg, tc, tl)
    if differing == 0 and np.array_equal(lg, lo):
        assert it_g == it_o
        assert_centroids_close(cg, co)


def test_fp32_iterations(torch_cuda, mxk, orc):
    torch = torch_cuda
    n, d, k = 6000, 128, 16
    x = blobs(n, 64, k, seed=5)
    c0 = x[:k].copy()
    it_g, cg, lg, tc, tl, tg = traced_run(torch, mxk, x, c0, 4, fp32_iterations=2)
    it_o, co, lo = orc.kmeans_mixed(x, c0, max_iterations=4, fp32_iterations=2, tolerance=0.0)
    assert it_g == it_o
    # two FP32 iterations (FP32 products, no MX groups), then two MX iterations
    assert np.array_equal(tg[:2], np.zeros((2, 3), np.int32))
    assert np.array_equal(tg[2:], np.array([[0, 0, n]] * 2, np.int32))
    check_steps(orc, x, it_g, cg, tc, tl, fp32_iterations=2)
    assert abs(orc.inertia(x, cg, lg) - orc.inertia(x, co, lo)) <= 1e-4 * orc.inertia(x, co, lo)


def test_nonfinite_shift_raises(torch_cuda, mxk):
    torch = torch_cuda
    n, d, k = 256, 128, 4
    x = np.full((n, d), 3e38, np.float32)
    c0 = np.zeros((k, d), np.float32)
    # every distance is +inf (the point norms overflow): the argmin finds no finite
    # minimum; the reference would index its sums with INT_MAX here, this library
    # reports the non-finite state instead (src/kmeans.cu:64 wording).
    with pytest.raises(mxk.MxkError, match="Non-finite"):
        _run(torch, mxk, x, c0, max_iterations=2, tolerance=0.0)


def test_rejects_unpadded_d(torch_cuda, mxk):
    torch = torch_cuda
    with pytest.raises(ValueError):
        _run(torch, mxk, np.zeros((8, 96), np.float32), np.zeros((4, 96), np.float32), max_iterations=1)


def test_duplicate_centroids_keep_lowest_index(torch_cuda, mxk, orc):
    """Exact distance ties between duplicated centroids resolve to the lowest
    index in every iteration, including the ones whose sweep over centroid tiles
    starts at the previous label's tile.  Integer-valued clusters whose points sit
    exactly on their centers keep every mean exact, so duplicates stay duplicates."""
    torch = torch_cuda
    n_per, d, k = 40, 128, 256
    g = np.random.default_rng(21)
    base = g.integers(-8, 9, size=(200, d)).astype(np.float32)
    x = np.repeat(base, n_per, axis=0)
    x = x[g.permutation(len(x))]
    c0 = np.zeros((k, d), np.float32)
    c0[:200] = base
    c0[200:] = base[:56]          # duplicates with higher indices (other centroid tile)
    c0[137] = base[5]             # and one inside the second tile
    it, cg, lg = _run(torch, mxk, x, c0, max_iterations=3, tolerance=0.0)
    assert not np.any(lg >= 200), "a tie went to the higher duplicate index"
    assert not np.any(lg == 137)
    it_o, co, lo = orc.kmeans_mixed(x, c0, max_iterations=3, tolerance=0.0)
    assert np.array_equal(lg, lo)


def test_stop_rule_on_device_matches_exact_iteration_count(torch_cuda, mxk):
    """The stopping rule runs on the device and the driver enqueues iterations
    ahead of reading it: iterations enqueued after the stop must change nothing.
    Integer-valued points make every sum exact, so runs are deterministic: the
    per-iteration shifts are recovered from runs capped at 1, 2, ... iterations,
    a tolerance is placed between them, and the early-stopping run must equal
    the run capped at the expected iteration bit for bit."""
    torch = torch_cuda
    n, d, k = 12000, 128, 24
    x = np.rint(blobs(n, 64, k, seed=21, spread=12.0, sigma=2.0)).astype(np.float32)
    c0 = x[np.random.default_rng(5).choice(n, k, replace=False)].copy()
    cents = [c0.astype(np.float64)]
    for cap in range(1, 9):
        it, c, _ = _run(torch, mxk, x, c0, max_iterations=cap, tolerance=0.0)
        assert it == cap
        cents.append(c.astype(np.float64))
    shifts = [float(((cents[i] - cents[i - 1]) ** 2).sum()) for i in range(1, 9)]
    # first iteration j >= 2 whose shift is clearly below every earlier one
    j = next(i + 1 for i in range(1, 8) if shifts[i] < 0.9 * min(shifts[:i]))
    tol = 0.5 * (shifts[j - 1] + min(shifts[:j - 1]))
    it_ref, c_ref, l_ref = _run(torch, mxk, x, c0, max_iterations=j, tolerance=0.0)
    for cap in (j, j + 1, j + 30):
        it2, c2, l2 = _run(torch, mxk, x, c0, max_iterations=cap, tolerance=tol)
        assert it2 == j
        assert np.array_equal(l2, l_ref) and np.array_equal(c2, c_ref)
    # a tolerance no shift meets: the count is the cap
    cap = min(j + 2, 8)
    if min(shifts[:cap]) > 0.0:
        it3, _, _ = _run(torch, mxk, x, c0, max_iterations=cap, tolerance=0.0)
        assert it3 == cap
    # a loose tolerance stops on the first iteration
    it4, _, _ = _run(torch, mxk, x, c0, max_iterations=60, tolerance=1e30)
    assert it4 == 1


def test_large_k_two_iterations_match_oracle(torch_cuda, mxk, orc):
    """The benchmark's K = 2048 at D = 128 (fused quantize, 11 centroid tiles,
    label-sorted second iteration).  n gives each CTA about three row tiles and a
    partial last tile.  Integer-valued points make every sum exact, so every
    cluster whose members agree with the oracle's must have the identical
    centroid."""
    torch = torch_cuda
    n, d, k = 56909, 128, 2048
    x = np.rint(blobs(n, 96, 256, seed=17, spread=20.0, sigma=3.0)).astype(np.float32)
    c0 = x[np.random.default_rng(3).choice(n, k, replace=False)].copy()
    it_g, cg, lg, tc, tl, _ = traced_run(torch, mxk, x, c0, 2)
    assert it_g == 2
    check_steps(orc, x, it_g, cg, tc, tl)
    for t in range(2):
        # exact sums: every cluster whose members agree with the oracle's
        # assignment from the same centroids has the oracle's centroid bit for bit
        _, _, lo, _ = orc.lloyd_step(x, orc.l2_norm(x), tc[t])
        co, _ = orc.update_centroids(x, tl[t], tc[t])
        same = tl[t] == lo
        keep = np.bincount(tl[t], minlength=k) > 0
        keep[np.unique(np.concatenate([tl[t][~same], lo[~same]]))] = False
        assert keep.sum() > 0.9 * k
        c_next = tc[t + 1] if t + 1 < it_g else cg
        assert np.array_equal(c_next[keep], co[keep])


@pytest.mark.parametrize("n,d,k,init", [(30000, 256, 1024, "farthest"), (20000, 768, 2048, "kmeans++")])
def test_config_shapes_one_iteration_vs_oracle(torch_cuda, mxk, orc, n, d, k, init):
    """configs[2] / configs[4] shapes at a small N (D = 256 and 768: several K
    chunks; K = 2048 at D = 768: centroid scales streamed with the ring), from
    the library's own initialisation, one Lloyd iteration against the oracle."""
    torch = torch_cuda
    x = blobs(n, d, 64, seed=d + k, spread=10.0, sigma=1.0)
    xt = torch.from_numpy(x).cuda()
    ct = torch.empty((k, d), device="cuda")
    if init == "farthest":
        mxk.init_farthest(xt, ct)
    else:
        mxk.init_kmeanspp(xt, ct, 19)
    c0 = ct.cpu().numpy()
    lab = torch.full((n,), -1, dtype=torch.int32, device="cuda")
    it = mxk.kmeans_mixed(xt, ct, lab, mxk.Options(max_iterations=1, tolerance=0.0))
    assert it == 1
    lg, cg = lab.cpu().numpy(), ct.cpu().numpy()
    shift, co, lo, dots = orc.lloyd_step(x, orc.l2_norm(x), c0, want_dots=True)
    near, first, second = orc.top2(orc.l2_norm(x), orc.l2_norm(c0), dots)
    diff = lg != lo
    scale = orc.l2_norm(x) + orc.l2_norm(c0).max()
    assert np.all((second - first)[diff] <= 1e-5 * scale[diff])
    moved = np.unique(np.concatenate([lg[diff], lo[diff]]))
    keep = np.ones(k, bool)
    keep[moved] = False
    assert np.allclose(cg[keep], co[keep], rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("n,blobs_k,spread,sigma,iters", [(56909, 300, 12.0, 2.0, (2, 3, 5)),
                                                         (300000, 2048, 8.0, 0.6, (4, 8))])
def test_pruned_assignment_equals_unpruned(torch_cuda, mxk, n, blobs_k, spread, sigma, iters):
    """From the second iteration on, the driver skips centroid tiles that the
    previous iteration's labels and distances prove cannot hold a point's nearest
    centroid.  Replay: the labels of iteration t (from a run capped at t) must
    equal an unpruned assignment (mxk_assign_f32_fused, no tile mask) against the
    centroids a run capped at t - 1 ends with.  Integer-valued points make every
    update exact, so both runs see the same centroids."""
    # (the second case: many row tiles per CTA, most of them needing a single
    # centroid tile, mixed with multi-tile ones)
    torch = torch_cuda
    d, k = 128, 2048
    x = np.rint(blobs(n, 96, blobs_k, seed=31, spread=spread, sigma=sigma) * 4).astype(np.float32)
    xt = torch.from_numpy(x).cuda()
    c0 = torch.empty((k, d), device="cuda")
    mxk.init_kmeanspp(xt, c0, 5)
    pn = torch.empty(n, device="cuda")
    mxk.compute_l2_norm(xt, pn)

    def run(iters):
        ct = c0.clone()
        lab = torch.full((n,), -1, dtype=torch.int32, device="cuda")
        assert mxk.kmeans_mixed(xt, ct, lab, mxk.Options(max_iterations=iters, tolerance=0.0)) == iters
        return ct, lab

    for t in iters:
        c_prev, _ = run(t - 1)
        _, lab_t = run(t)
        qc = torch.empty(k * d, dtype=torch.uint8, device="cuda")
        sc = torch.empty(k * d // 32, dtype=torch.uint8, device="cuda")
        mxk.quantize_rows(8, c_prev, qc, sc)
        cn = torch.empty(k, device="cuda")
        mxk.compute_l2_norm(c_prev, cn)
        lab_u = torch.full((n,), -1, dtype=torch.int32, device="cuda")
        mxk.assign_f32_fused(n, k, d, xt, qc, sc, pn, cn, lab_u)
        torch.cuda.synchronize()
        assert torch.equal(lab_t, lab_u), f"iteration {t}: {(lab_t != lab_u).sum().item()} labels differ"


@pytest.mark.parametrize("n,d,k", [(56909, 128, 2048), (20000, 256, 300)])
def test_cached_points_equal_default(torch_cuda, mxk, n, d, k):
    """mxk_kmeans_mixed_cached (points quantized once, regathered when the
    visiting order changes) gives the default path's labels, centroids and
    iteration count; integer data keeps both runs deterministic."""
    torch = torch_cuda
    x = np.rint(blobs(n, d - 32, 200, seed=41, spread=10.0, sigma=1.5, pad_to=d) * 2).astype(np.float32)
    xt = torch.from_numpy(x).cuda()
    c0 = torch.empty((k, d), device="cuda")
    mxk.init_kmeanspp(xt, c0, 11)
    out = []
    for cached in (False, True):
        ct = c0.clone()
        lab = torch.full((n,), -1, dtype=torch.int32, device="cuda")
        it = mxk.kmeans_mixed(xt, ct, lab, mxk.Options(max_iterations=7, tolerance=0.0), cache_points=cached)
        torch.cuda.synchronize()
        out.append((it, ct.cpu().numpy(), lab.cpu().numpy()))
    assert out[0][0] == out[1][0]
    assert np.array_equal(out[0][2], out[1][2])
    assert np.array_equal(out[0][1], out[1][1])


@pytest.mark.parametrize("n,d,k,blobs_k,seed", [(60000, 128, 2048, 1500, 3), (40000, 256, 1024, 700, 11),
                                                (30000, 768, 2048, 1200, 19), (30000, 768, 8192, 3000, 23)])
def test_pruned_assignment_equals_unpruned_nonint(torch_cuda, mxk, n, d, k, blobs_k, seed):
    """Exact pruning on non-integer data at the configs[2..4] feature widths
    (D = 128, 256, 768; up to 43 centroid tiles): every traced iteration's labels
    equal an unpruned assignment (tcgen05 GEMM + argmin with no tile mask) of the
    same points against the centroids that iteration used, bit for bit, over
    six iterations; and the mask did skip tiles."""
    torch = torch_cuda
    iters = 6
    x = blobs(n, d - 32 if d > 128 else 96, blobs_k, seed=seed, spread=5.0, sigma=0.75, pad_to=d)
    xt = torch.from_numpy(x).cuda()
    c0 = torch.empty((k, d), device="cuda")
    mxk.init_kmeanspp(xt, c0, seed)
    mxk.gemm_tiles_multiplied(reset=True)
    it, _, _, tc, tl, _ = traced_run(torch, mxk, xt, c0, iters)
    multiplied = mxk.gemm_tiles_multiplied(reset=True)
    # (few points per cluster at K = 8192 settle after two iterations: an exactly
    # zero shift meets tol 0; iterations enqueued past the stop multiply nothing;
    # iteration 1 is pruned in every case)
    assert 2 <= it <= iters
    unpruned = it * ((n + 127) // 128) * ((k + 191) // 192)
    assert multiplied < 0.9 * unpruned, f"pruning inactive: {multiplied} of {unpruned} tiles multiplied"
    pn = torch.empty(n, device="cuda")
    mxk.compute_l2_norm(xt, pn)
    qx = torch.empty(n * d, dtype=torch.uint8, device="cuda")
    sx = torch.empty(n * d // 32, dtype=torch.uint8, device="cuda")
    mxk.quantize_rows(8, xt, qx, sx)
    for t in range(1, it):
        ct = torch.from_numpy(tc[t]).cuda()
        qc = torch.empty(k * d, dtype=torch.uint8, device="cuda")
        sc = torch.empty(k * d // 32, dtype=torch.uint8, device="cuda")
        mxk.quantize_rows(8, ct, qc, sc)
        cn = torch.empty(k, device="cuda")
        mxk.compute_l2_norm(ct, cn)
        lab_u = torch.full((n,), -1, dtype=torch.int32, device="cuda")
        mxk.assign_mx_fused(8, n, k, d, qx, sx, qc, sc, pn, cn, lab_u)
        lu = lab_u.cpu().numpy()
        assert np.array_equal(tl[t], lu), f"iteration {t}: {(tl[t] != lu).sum()} labels differ from unpruned"


def test_running_sums_over_a_long_run(torch_cuda, mxk, orc):
    """Pruned iterations keep FP64 running cluster sums and move only the rows
    whose label changed; rows whose bounds prove their label leave the GEMM.
    Over a 40-iteration run on non-integer data, every iteration's next
    centroids must stay within 1e-4 of the oracle's fresh update from that
    iteration's labels (no drift), and sampled iterations' labels follow the
    gap-band rule."""
    torch = torch_cuda
    n, d, k, iters = 60000, 128, 512, 40
    x = blobs(n, 96, 400, seed=77, spread=5.0, sigma=0.9)
    xt = torch.from_numpy(x).cuda()
    c0 = torch.empty((k, d), device="cuda")
    mxk.init_kmeanspp(xt, c0, 77)
    mxk.gemm_rows_processed(reset=True)
    it, cg, lg, tc, tl, _ = traced_run(torch, mxk, xt, c0, iters)
    rows = mxk.gemm_rows_processed(reset=True)
    assert it >= 10  # (a run whose labels stop changing meets tol 0 with a zero shift)
    assert rows < 0.9 * n * it, "rows with proven labels should leave the GEMM"
    for t in range(it):
        c_next = tc[t + 1] if t + 1 < it else cg
        co, _ = orc.update_centroids(x, tl[t], tc[t])
        assert_centroids_close(c_next, co)
    for t in sorted({1, 5, it // 2, it - 1}):
        gap_band_mismatches(orc, x, tc[t], tl[t])


def test_many_label_changes_switch_to_a_fresh_accumulation(torch_cuda, mxk, orc):
    """Pruned iterations move only the rows whose label changed, unless more than
    n / 8 labels changed: then the device switches that iteration to a fresh
    accumulation of every point (the running sums are replaced).  Points without
    cluster structure (uniform in a cube) and random initial rows keep many
    labels changing for several iterations, so both branches run within one
    call; every iteration's next centroids must match the oracle's fresh update
    from that iteration's labels (src/kernels/update.cu:7-31) within 1e-4, and
    sampled iterations' labels follow the gap-band rule."""
    torch = torch_cuda
    n, d, k, iters = 40000, 128, 256, 12
    g = np.random.default_rng(8)
    x = np.zeros((n, d), np.float32)
    x[:, :96] = g.uniform(-1.0, 1.0, size=(n, 96)).astype(np.float32)
    c0 = x[g.choice(n, k, replace=False)].copy()
    it, cg, lg, tc, tl, _ = traced_run(torch, mxk, x, c0, iters)
    assert it == iters
    changed = [int((tl[t] != tl[t - 1]).sum()) for t in range(1, it)]
    assert max(changed) > n // 8, f"no iteration changed more than n / 8 labels: {changed}"
    assert min(changed) < n // 8, f"every iteration changed more than n / 8 labels: {changed}"
    for t in range(it):
        c_next = tc[t + 1] if t + 1 < it else cg
        co, _ = orc.update_centroids(x, tl[t], tc[t])
        assert_centroids_close(c_next, co)
    for t in (1, 2, it // 2, it - 1):
        gap_band_mismatches(orc, x, tc[t], tl[t])
