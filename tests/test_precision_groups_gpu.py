"""The per-precision groups of the Lloyd loop (src/kmeans.cu:42-57) through
the library's precision-policy hook.  The reference's select_precision always
returns MXFP8 (include/precision.hpp:20-26), so its 4/6/8 machinery --
point error bounds, the two-largest distance gaps, the policy kernel, the
stable compaction and one quantize + block-scaled GEMM + assignment per group
(MXFP4 and MXFP6 A operands included) -- only runs when the candidate it
discards is allowed to stand: mxk_set_precision_policy(1), against the oracle's
loop under the same rule (orc_kmeans_mixed_ex, policy 1).

Data: blobs near the origin plus two far, empty clusters; a point's
two-largest gap 2|x . (f2 - f1)| then spreads over a wide range, so after the
first iteration (gaps start at 0: all MXFP8) the candidate puts points in all
three groups.  Integer-valued coordinates keep every sum exact, so the GPU and
the oracle follow the same trajectory: the group sizes of every iteration, the
labels and the centroids must agree exactly."""
import numpy as np
import pytest

from conftest import assert_centroids_close, blobs, traced_run

pytestmark = pytest.mark.gpu


def _data(d):
    n, k = 20000, 18
    x = np.rint(blobs(n, d - 32, 16, seed=13, spread=6.0, sigma=1.0, pad_to=d)).astype(np.float32)
    g = np.random.default_rng(2)
    c0 = np.zeros((k, d), np.float32)
    c0[:16] = x[g.choice(n, 16, replace=False)]
    c0[16, 0] = 40.0   # far clusters that never receive a point (empty clusters keep
    c0[17, 1] = 40.0   # their centroid, src/kernels/update.cu:26-29)
    return x, c0


@pytest.mark.parametrize("d", [128, 256])
def test_candidate_policy_groups_match_oracle(torch_cuda, mxk, orc, d):
    torch = torch_cuda
    x, c0 = _data(d)
    iters = 6
    mxk.set_precision_policy(1)
    try:
        it, cg, lg, tc, tl, tg = traced_run(torch, mxk, x, c0, iters)
    finally:
        mxk.set_precision_policy(0)
    it_o, co, lo, go = orc.kmeans_mixed(x, c0, max_iterations=iters, tolerance=0.0, policy=1, group_sizes=True)
    assert it == it_o and it >= 4  # (exact sums: the run may converge, shift 0, before the cap)
    # (entries past the stop are empty on both sides)
    assert np.array_equal(tg, go), f"group sizes differ:\n{tg}\n{go}"
    assert np.array_equal(tg[0], [0, 0, x.shape[0]])  # gaps start at zero: every point MXFP8
    assert np.all(tg[1:it] > 0), f"every group must be used after the first iteration:\n{tg}"
    assert np.array_equal(lg, lo)
    assert_centroids_close(cg, co)


def test_reference_policy_is_default_and_unchanged(torch_cuda, mxk, orc):
    """With the hook back at 0 the same data runs the forced-MXFP8 path: one
    MXFP8 group per iteration, the oracle's reference-policy result."""
    torch = torch_cuda
    x, c0 = _data(128)
    it, cg, lg, _, _, tg = traced_run(torch, mxk, x, c0, 4)
    it_o, co, lo, go = orc.kmeans_mixed(x, c0, max_iterations=4, tolerance=0.0, policy=0, group_sizes=True)
    assert np.array_equal(tg, np.array([[0, 0, x.shape[0]]] * 4, np.int32))
    assert np.array_equal(go, tg)
    assert np.array_equal(lg, lo)
    assert_centroids_close(cg, co)

