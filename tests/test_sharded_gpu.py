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


@pytest.mark.parametrize("gpus,n", [(1, 20011), (2, 20011), (1, 1100011), (2, 1100011)])
def test_multi_entry_matches_single_gpu(torch_cuda, mxk, gpus, n):
    """mxk_kmeans_mixed_multi (host buffers, one thread per GPU, NCCL inside the
    library) against kmeans_mixed on one GPU: bit-identical on integer data.
    The larger n spans several of the 256 MB upload chunks on which the first
    iteration starts while the rest of the copy is in flight (a partial last
    chunk included)."""
    torch = torch_cuda
    if torch.cuda.device_count() < gpus:
        pytest.skip(f"needs {gpus} GPUs")
    d, k, seed, iters = 128, 40, 9, 8
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


MULTI_FAILURE_CHILD = r'''
import sys
import numpy as np
sys.path[:0] = [sys.argv[1], sys.argv[2]]
import mxk
from test_sharded_cpu import _blob_data
n, d, k = 20011, 128, 40
x, c0 = _blob_data(n, d, k, 9)
opts = mxk.Options(max_iterations=8, tolerance=0.0)
mxk.inject_rank_failure(1, 3)
try:
    mxk.kmeans_mixed_multi(np.ascontiguousarray(x), c0.copy(), np.zeros(n, np.int32), opts, 2)
    print("NO-ERROR")
except mxk.MxkError as e:
    print("ERROR", e.status, e.message)
mxk.inject_rank_failure(-1, -1)
cent, labels = c0.copy(), np.zeros(n, np.int32)
it = mxk.kmeans_mixed_multi(np.ascontiguousarray(x), cent, labels, opts, 2)
print("RECOVERED", it)
'''


def _two_gpu_failure_env():
    env = dict(os.environ)
    env["NCCL_NVLS_ENABLE"] = "0"  # no NVLink multicast objects in a test where a rank leaves
    return env


def test_multi_entry_reports_an_injected_rank_failure(tmp_path):
    """mxk_kmeans_mixed_multi with two in-process ranks, rank 1 leaving between
    steps (on the host, after its enqueued work has finished) at iteration 3:
    rank 0's collective for that iteration has no partner.  Rank 0's host wait
    polls the ranks' shared failure flag, aborts its communicator and returns,
    so the call reports the failure instead of hanging; the next call works.
    Child process, NVLS off; nothing on the GPU faults or waits without limit."""
    import subprocess
    import sys
    import torch
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    script = tmp_path / "child.py"
    script.write_text(MULTI_FAILURE_CHILD)
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    r = subprocess.run([sys.executable, str(script), os.path.join(root, "mx-kmeans_b200"), here],
                       capture_output=True, text=True, timeout=180, env=_two_gpu_failure_env())
    assert r.returncode == 0, r.stdout + r.stderr
    lines = r.stdout.splitlines()
    err = [l for l in lines if l.startswith("ERROR")]
    assert err, r.stdout + r.stderr
    assert "injected rank failure" in err[0]
    assert any(l.startswith("RECOVERED") for l in lines), r.stdout


def _leave(rank, world, port, n, d, k):
    """Both ranks run one sharded call; then rank 1 leaves (no further call, its
    process and memory stay until rank 0 is done) and rank 0 runs another, which
    has to end through the watchdog (MXK_COMM_TIMEOUT_S) with an error."""
    import time
    import torch
    import torch.distributed as dist
    import mxk
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    comm = mxk.bootstrap_comm()
    x, c0 = _blob_data(n, d, k, 9)
    first, rows = mxk.shard_rows(n, world, rank)
    xs = torch.from_numpy(x[first:first + rows]).cuda()
    cent = torch.from_numpy(c0).cuda()
    labels = torch.empty(rows, dtype=torch.int32, device="cuda")
    opts = mxk.Options(max_iterations=3, tolerance=0.0)
    assert mxk.kmeans_mixed_sharded(comm, xs, cent, labels, opts) >= 1
    torch.cuda.synchronize()
    dist.barrier()  # between steps: neither rank has work or collectives in flight
    out = {}
    if rank == 0:
        cent.copy_(torch.from_numpy(c0))
        t0 = time.monotonic()
        try:
            mxk.kmeans_mixed_sharded(comm, xs, cent, labels, opts)
            out["status"] = 0
        except mxk.MxkError as e:
            out["status"], out["message"] = e.status, e.message
        out["seconds"] = time.monotonic() - t0
        # the aborted communicator refuses further work without touching NCCL
        try:
            mxk.kmeans_mixed_sharded(comm, xs, cent, labels, opts)
            out["reuse"] = 0
        except mxk.MxkError as e:
            out["reuse"] = e.status
    dist.barrier()  # rank 1 stays until rank 0 has its answer
    if rank == 0:
        comm.close()  # (the aborted handle: frees the wrapper only)
    # rank 1's communicator lost its peer: its process exits without a
    # collective teardown, which would wait for rank 0
    dist.destroy_process_group()
    return out


def test_sharded_watchdog_ends_a_wait_for_a_rank_that_left(monkeypatch):
    """Two GPUs, NCCL with NVLS off: after a completed sharded call, rank 1 makes
    no further call; rank 0's next call enqueues a collective rank 1 never
    joins.  With MXK_COMM_TIMEOUT_S=5 rank 0's host wait polls instead of
    blocking, aborts the communicator once the limit passes without progress,
    and the call returns MXK_ERR_TIMEOUT (or MXK_ERR_COMM when NCCL reports the
    peer first) within seconds; a later call on the aborted handle is refused."""
    import torch
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    monkeypatch.setenv("NCCL_NVLS_ENABLE", "0")
    monkeypatch.setenv("MXK_COMM_TIMEOUT_S", "5")
    out = _spawn(_leave, 2, 20011, 128, 40)
    r0 = out[0]
    assert r0["status"] in (5, 6), r0  # MXK_ERR_TIMEOUT or MXK_ERR_COMM
    assert r0["seconds"] < 60, r0
    assert r0["reuse"] == 6, r0
