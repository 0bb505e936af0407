"""Row-sharded kmeans_mixed over NCCL on two GPUs (skipped with fewer), and the
host-buffer multi-GPU entry kmeans_mixed_multi on one and two GPUs.

Each rank runs mxk.kmeans_mixed_sharded on its contiguous shard; rank 0 also runs
the single-GPU kmeans_mixed on all points from the same initial centroids.  The
points are integer-valued, so every partial and all-reduced sum is exact in FP32
and the two runs must agree bit for bit (labels, centroids, iteration count)."""
import datetime
import os

import numpy as np
import pytest

from test_sharded_cpu import _spawn, _blob_data

pytestmark = pytest.mark.gpu


def _run(rank, world, port, n, d, k, seed, iters):
    import torch
    import torch.distributed as dist
    import mxk
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    comm = mxk.bootstrap_comm()
    x, c0 = _blob_data(n, d, k, seed)
    first, rows = mxk.shard_rows(n, world, rank)
    xs = torch.from_numpy(x[first:first + rows]).cuda()
    cent = torch.from_numpy(c0).cuda()
    labels = torch.empty(rows, dtype=torch.int32, device="cuda")
    opts = mxk.Options(max_iterations=iters, tolerance=0.0)
    it = mxk.kmeans_mixed_sharded(comm, xs, cent, labels, opts)
    torch.cuda.synchronize()
    out = {"first": first, "labels": labels.cpu().numpy(), "cent": cent.cpu().numpy(), "iters": it}
    if rank == 0:
        xf = torch.from_numpy(x).cuda()
        cf = torch.from_numpy(c0).cuda()
        lf = torch.empty(n, dtype=torch.int32, device="cuda")
        out["single"] = (lf, cf, mxk.kmeans_mixed(xf, cf, lf, opts))
        torch.cuda.synchronize()
        out["single"] = (lf.cpu().numpy(), cf.cpu().numpy(), out["single"][2])
    dist.barrier()
    comm.close()
    dist.destroy_process_group()
    return out


# the second case has four centroid tiles, so from the second iteration on each
# rank prunes tiles from its own rows' bounds
@pytest.mark.parametrize("n,d,k,seed,iters", [(20011, 128, 40, 9, 8), (60013, 128, 700, 3, 10)])
def test_two_gpu_sharded_matches_single_gpu(n, d, k, seed, iters):
    import torch
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    out = _spawn(_run, 2, n, d, k, seed, iters)
    labels = np.concatenate([out[r]["labels"] for r in sorted(out, key=lambda r: out[r]["first"])])
    single_labels, single_cent, single_iters = out[0]["single"]
    # integer data converge exactly (shift 0 <= tol 0): all runs stop together
    assert out[0]["iters"] == out[1]["iters"] == single_iters <= iters
    assert np.array_equal(out[0]["cent"], out[1]["cent"])
    assert np.array_equal(out[0]["cent"], single_cent)
    assert np.array_equal(labels, single_labels)


@pytest.mark.parametrize("gpus", [1, 2])
def test_multi_entry_matches_single_gpu(torch_cuda, mxk, gpus):
    """mxk_kmeans_mixed_multi (host buffers, one thread per GPU, NCCL inside the
    library) against kmeans_mixed on one GPU: bit-identical on integer data."""
    torch = torch_cuda
    if torch.cuda.device_count() < gpus:
        pytest.skip(f"needs {gpus} GPUs")
    n, d, k, seed, iters = 20011, 128, 40, 9, 8
    x, c0 = _blob_data(n, d, k, seed)
    opts = mxk.Options(max_iterations=iters, tolerance=0.0)
    xf = torch.from_numpy(x).cuda()
    cf = torch.from_numpy(c0).cuda()
    lf = torch.empty(n, dtype=torch.int32, device="cuda")
    single_iters = mxk.kmeans_mixed(xf, cf, lf, opts)
    torch.cuda.synchronize()
    cent = np.ascontiguousarray(c0.copy())
    labels = np.full(n, -1, np.int32)
    it = mxk.kmeans_mixed_multi(np.ascontiguousarray(x), cent, labels, opts, gpus)
    assert it == single_iters
    assert np.array_equal(labels, lf.cpu().numpy())
    assert np.array_equal(cent, cf.cpu().numpy())
    assert torch.cuda.current_device() == 0
