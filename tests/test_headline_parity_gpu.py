"""Parity of the benchmarked path itself: the benchmark's configs[3] at its full size
(N = 8,388,608, D = 96 padded to 128, K = 2048, the bench's seeded blobs and
K-Means++ centroids), 20 Lloyd iterations of kmeans_mixed with exact tile
pruning and the fused quantizer, traced per iteration and checked step by step
against the oracle (src/kmeans.cu:28-67):

* labels: for 65,536 sampled rows per checked iteration, the oracle's MX
  assignment from the centroids that iteration used; a label may differ only
  where the oracle's top-2 distance gap is below 1e-5 of the distance scale;
* centroids: the centroids the next iteration starts from against the oracle's
  update (src/kernels/update.cu:7-31) over all N points with the iteration's
  labels, within 1e-4 relative."""
import importlib.util
import os

import numpy as np
import pytest

from conftest import ROOT, assert_centroids_close, gap_band_mismatches

pytestmark = pytest.mark.gpu


def _bench():
    spec = importlib.util.spec_from_file_location("mxk_bench", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_headline_config_sampled_rows_vs_oracle(torch_cuda, mxk, orc):
    torch = torch_cuda
    bench = _bench()
    dev = torch.device("cuda:0")
    n, k, d, iters = bench.N_POINTS, bench.K_CLUSTERS, bench.D_PAD, bench.ITERS
    x = bench.make_dataset(torch, n, dev)
    c0 = torch.empty((k, d), device=dev)
    mxk.init_kmeanspp(x, c0, bench.SEED)
    tc = torch.zeros((iters, k, d), device=dev)
    tl = torch.full((iters, n), -1, dtype=torch.int32, device=dev)
    cent = c0.clone()
    lab = torch.full((n,), -1, dtype=torch.int32, device=dev)
    mxk.gemm_tiles_multiplied(reset=True)
    mxk.trace_next_call(iters, tc, tl)
    it = mxk.kmeans_mixed(x, cent, lab, mxk.Options(max_iterations=iters, tolerance=0.0))
    torch.cuda.synchronize()
    assert it == iters
    multiplied = mxk.gemm_tiles_multiplied(reset=True)
    unpruned = iters * ((n + 127) // 128) * ((k + 191) // 192)
    assert multiplied < 0.6 * unpruned, "the benchmarked path prunes centroid tiles"
    assert torch.equal(tl[iters - 1], lab)

    x_host = x.cpu().numpy()
    g = np.random.default_rng(2024)
    for t in (1, 2, 5, 10, iters - 1):
        rows = np.sort(g.choice(n, 65536, replace=False))
        labels_t = tl[t].cpu().numpy()
        ct = tc[t].cpu().numpy()
        gap_band_mismatches(orc, x_host[rows], ct, labels_t[rows])
        c_next = (tc[t + 1] if t + 1 < it else cent).cpu().numpy()
        co, _ = orc.update_centroids(x_host, labels_t, ct)
        assert_centroids_close(c_next, co)
