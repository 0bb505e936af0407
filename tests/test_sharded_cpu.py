"""Row-sharded (multi-GPU) path, host side, on CPU with world_size-2 gloo groups.

The library's sharded Lloyd iteration (mxk_kmeans_mixed_sharded) is: every rank
assigns its contiguous shard of rows against the replicated centroids, sums its
points per cluster, all-reduces the K x D sums and K counts, and then computes
identical means (an empty cluster keeps its center), shift and stop decision.
These tests run that decomposition with the oracle on each rank and a gloo
all-reduce, and check it against the unsharded oracle step; they also check the
partition rule and that a rank that never joins ends the others' bootstrap with
an error instead of a hang (the NCCL calls are replaced by host fakes)."""
import datetime
import os
import socket
import sys
import time
import traceback

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _spawn(target, world, *args):
    """Run target(rank, world, port, result_queue, *args) in `world` spawned
    processes; -> {rank: result} (an exception on a rank is re-raised here)."""
    import torch.multiprocessing as tmp
    ctx = tmp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_entry, args=(target, r, world, port, q) + args) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    deadline = time.time() + 120
    while len(results) < world and time.time() < deadline:
        try:
            rank, ok, payload = q.get(timeout=1)
        except Exception:
            if all(not p.is_alive() for p in procs) and q.empty():
                break
            continue
        results[rank] = (ok, payload)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    for rank, (ok, payload) in results.items():
        if not ok:
            raise AssertionError(f"rank {rank} failed:\n{payload}")
    return {r: payload for r, (ok, payload) in results.items()}


def _entry(target, rank, world, port, q, *args):
    sys.path[:0] = [os.path.join(ROOT, "mx-kmeans_b200"), os.path.join(ROOT, "oracle")]
    try:
        q.put((rank, True, target(rank, world, port, *args)))
    except BaseException:
        q.put((rank, False, traceback.format_exc()))


def _init(rank, world, port, timeout_s=60):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _blob_data(n, d, k, seed):
    """Integer-valued points: every partial and total sum is exact in FP32, so the
    sharded and unsharded updates must agree bit for bit."""
    g = np.random.default_rng(seed)
    centers = g.integers(-40, 40, (k, d)).astype(np.float32)
    lab = g.integers(0, k, n)
    x = centers[lab] + g.integers(-3, 4, (n, d)).astype(np.float32)
    c0 = x[g.choice(n, k, replace=False)].copy()
    return x, c0


def _sharded_step(rank, world, port, n, d, k, seed):
    import mxk
    import oracle
    import torch
    dist = _init(rank, world, port)
    x, c0 = _blob_data(n, d, k, seed)
    first, rows = mxk.shard_rows(n, world, rank)
    xs = x[first:first + rows]
    # local assignment against the replicated centroids (row-independent)
    _, _, labels, _ = oracle.lloyd_step(xs, oracle.l2_norm(xs), c0, threads=1)
    sums = np.zeros((k, d), np.float32)
    np.add.at(sums, labels, xs)
    counts = np.bincount(labels, minlength=k).astype(np.int32)
    ts, tc = torch.from_numpy(sums), torch.from_numpy(counts)
    dist.all_reduce(ts)
    dist.all_reduce(tc)
    sums, counts = ts.numpy(), tc.numpy()
    cent = np.where(counts[:, None] > 0, sums / np.maximum(counts, 1)[:, None].astype(np.float32), c0)
    shift = oracle.centroid_shift(c0, cent)
    dist.destroy_process_group()
    return first, labels, cent.astype(np.float32), shift


def test_shard_rows_partition():
    import mxk
    for n in (0, 1, 7, 4096, 8388607):
        for world in (1, 2, 3, 4, 8):
            parts = [mxk.shard_rows(n, world, r) for r in range(world)]
            assert parts[0][0] == 0
            for (f0, c0), (f1, _) in zip(parts, parts[1:]):
                assert f1 == f0 + c0
            assert parts[-1][0] + parts[-1][1] == n
            sizes = [c for _, c in parts]
            assert max(sizes) - min(sizes) <= 1
            assert sizes == sorted(sizes, reverse=True)  # remainder to the low ranks
    with pytest.raises(ValueError):
        mxk.shard_rows(10, 2, 2)


@pytest.mark.parametrize("world", [2])
def test_sharded_step_equals_unsharded(orc, world):
    n, d, k, seed = 3001, 64, 12, 5
    out = _spawn(_sharded_step, world, n, d, k, seed)
    x, c0 = _blob_data(n, d, k, seed)
    shift, cent, labels, _ = orc.lloyd_step(x, orc.l2_norm(x), c0, threads=1)
    got_labels = np.concatenate([out[r][1] for r in sorted(out, key=lambda r: out[r][0])])
    assert np.array_equal(got_labels, labels)
    for r in out:  # every rank ends with the same centroids and shift
        assert np.array_equal(out[r][2], cent)
        assert out[r][3] == shift


def _bootstrap(rank, world, port, leave):
    import mxk
    dist = _init(rank, world, port, timeout_s=4)
    made = {}

    class FakeComm:  # stands in for the NCCL communicator
        def __init__(self, nranks, r, uid):
            made.update(nranks=nranks, rank=r, uid=uid)

    mxk.comm_unique_id = lambda: b"id-from-rank-0".ljust(128, b"\0")
    mxk.Comm = FakeComm
    if leave and rank == 1:
        os._exit(0)  # this rank is gone before the exchange
    t0 = time.time()
    try:
        mxk.bootstrap_comm()
        outcome = ("ok", made)
    except Exception as e:  # the peer never joined
        outcome = ("error", type(e).__name__, time.time() - t0)
    return outcome


def test_bootstrap_comm_exchanges_id():
    out = _spawn(_bootstrap, 2, False)
    for r in (0, 1):
        kind, made = out[r]
        assert kind == "ok"
        assert made["rank"] == r and made["nranks"] == 2
        assert made["uid"].startswith(b"id-from-rank-0")


def test_bootstrap_comm_fails_when_a_rank_leaves():
    out = _spawn(_bootstrap, 2, True)
    assert 0 in out and out[0][0] == "error", out
    assert out[0][2] < 60  # ended by the group's timeout, not a hang


WATCHDOG_TEST = r'''
#include <cstdio>
#include "watchdog.hpp"
using namespace mxk;
struct Fake { int polls = 0, ready_at, peer_at; double t = 0.0; };
static WaitResult run(Fake& f, double limit) {
    return guarded_wait(
        [&] { ++f.polls; return f.polls >= f.ready_at ? Probe::kReady : Probe::kPending; },
        [&] { return f.peer_at > 0 && f.polls >= f.peer_at; },
        limit, [&] { return f.t; }, [&] { f.t += 0.5; });
}
int main() {
    int bad = 0;
    { Fake f{0, 1, 0}; bad += run(f, 10.0) != WaitResult::kReady || f.polls != 1; }       // done at once
    { Fake f{0, 7, 0}; bad += run(f, 10.0) != WaitResult::kReady || f.polls != 7; }       // done after polling
    { Fake f{0, 1000, 4}; bad += run(f, 10.0) != WaitResult::kPeerFailed || f.polls != 4; } // peer fails first
    { Fake f{0, 1000, 0}; bad += run(f, 2.0) != WaitResult::kTimedOut || f.t > 2.5; }     // no progress
    { Fake f{0, 4, 4}; bad += run(f, 10.0) != WaitResult::kReady; }                       // completion wins a tie
    { Fake f{0, 1000, 50}; bad += run(f, 0.0) != WaitResult::kPeerFailed || f.polls != 50; } // no time limit:
                                                                                          // only a peer ends it
    {   // a failed query is reported as such, not as a timeout
        int n = 0; double t = 0.0;
        WaitResult r = guarded_wait([&] { return ++n < 3 ? Probe::kPending : Probe::kFailed; }, [] { return false; },
                                    10.0, [&] { return t; }, [&] { t += 1.0; });
        bad += r != WaitResult::kFailed || n != 3;
    }
    std::printf("%d\n", bad);
    return bad != 0;
}
'''


def test_comm_watchdog_logic(tmp_path):
    """The sharded loop's opt-in host watchdog (MXK_COMM_TIMEOUT_S): a wait ends
    ready when the work completes, with a peer failure as soon as the
    communicator (or another in-process rank) reports one, with a timeout when
    nothing progresses within the limit (none without a limit), and with the
    query's own failure otherwise.  Fake probes and clock,
    so no GPU, NCCL or real failure is involved."""
    import subprocess
    src = tmp_path / "w.cpp"
    src.write_text(WATCHDOG_TEST)
    exe = tmp_path / "w"
    subprocess.run(["g++", "-std=c++17", "-O1", "-I", os.path.join(ROOT, "mx-kmeans_b200", "csrc"), str(src),
                    "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and r.stdout.strip() == "0", r.stdout + r.stderr
