"""Benchmark of the MX-KMeans Lloyd iteration on B200 (BASELINE.json metric:
Lloyd point-iterations/sec; MX-GEMM fraction of tensor peak).

Workload: BASELINE configs[3] -- N = 8,388,608 points, D = 96 zero-padded to
128, K = 2048 clusters, seeded Gaussian blobs (centers U[-5,5]^96, sigma 0.75,
seed 3), K-Means++ initial centroids, 20 Lloyd iterations with tol 0 (a run can
stop earlier on an exactly unchanged shift; the reported rate uses the
iterations actually run).  One step = one kmeans_mixed call over the whole
dataset, from the same initial centroids (the reference CLI's timed unit,
src/main.cu:115-123).  With --gpus N (torchrun, one rank per GPU) the points are
row-sharded and every iteration NCCL-allreduces the K x D sums and K counts:
strong scaling of the fixed N.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "mx-kmeans_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

N_POINTS, D_RAW, D_PAD, K_CLUSTERS, ITERS, SEED = 8388608, 96, 128, 2048, 20, 3
METRIC = "Lloyd point-iters/sec"
UNIT = "point-iters/s"
WORKLOAD = ("configs[3]: N=8388608, D=96 zero-padded to 128, K=2048, blobs centers U[-5,5]^96 sigma 0.75, "
            "seed 3, K-Means++ init, 20 iterations (tol 0), MXFP8 points/centroids, FP32 update")


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="mxk", choices=["mxk", "reference"])
    # profiling aids (the ncu commands under profiles/ use them; bench lines never do)
    p.add_argument("--n", type=int, default=N_POINTS, help="points (default: configs[3]'s N)")
    p.add_argument("--init", default="kmeans++", choices=["kmeans++", "random"],
                   help="random = K distinct random rows (fast set-up for profiling runs)")
    p.add_argument("--quick", action="store_true", help="skip the e2e and CPU-baseline legs")
    return p.parse_args()


def measured_traffic(rows):
    """dram__bytes_read.sum + dram__bytes_write.sum of one full-size fused-GEMM
    launch, from the ncu capture summarised in profiles/ (scaled to `rows`: every
    byte it counts is per point row); None if the summary is missing."""
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "profiles", "mx_gemm_argmin_config4.md")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_full_launch:"):
                return float(line.split(":")[1]) * rows / N_POINTS
    except OSError:
        pass
    return None


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def update_roofline(stats, rows, peak_gbs):
    """Achieved HBM bandwidth of the centroid update (the label-run or
    privatised accumulation pass, one launch per iteration) from its CUDA-event
    times in `stats` ({kernel: (launches, total_ms)}): algorithmic bytes per
    launch = each point's FP32 row, its id and its label, rows * (4 D_pad + 8).
    None when the pass did not run."""
    launches = sum(stats.get(k, (0, 0.0))[0] for k in ("accumulate_runs", "accumulate_private"))
    total_ms = sum(stats.get(k, (0, 0.0))[1] for k in ("accumulate_runs", "accumulate_private"))
    if not launches or total_ms <= 0.0:
        return None
    alg_bytes = rows * (4.0 * D_PAD + 8.0)
    gbs = alg_bytes * launches / (total_ms / 1e3) / 1e9
    return {"bound": "hbm", "achieved": gbs, "peak": peak_gbs, "unit": "GB/s", "frac": gbs / peak_gbs,
            "algorithmic_bytes_per_launch": alg_bytes, "ms_per_launch": total_ms / launches,
            "launches": launches, "kernel": "accumulate_runs"}


# ----------------------------------------------------------------------------- data

def make_dataset(torch, n, device):
    """Seeded blobs of configs[3] on the device (identical on every rank)."""
    g = torch.Generator(device=device).manual_seed(SEED)
    centers = torch.rand((K_CLUSTERS, D_RAW), generator=g, device=device) * 10.0 - 5.0
    labels = torch.randint(0, K_CLUSTERS, (n,), generator=g, device=device)
    x = torch.zeros((n, D_PAD), device=device)
    chunk = 1 << 22
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        x[s:e, :D_RAW] = centers[labels[s:e]] + 0.75 * torch.randn((e - s, D_RAW), generator=g, device=device)
    return x


# ----------------------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clock / throttle-reason samples of this rank's GPU during the
    timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.monotonic(), line.strip()))

    def stop(self, window=None):
        """Summary of the samples that arrived within `window` = (t0, t1) of
        time.monotonic() (all samples when None)."""
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for t, line in self.lines:
            if window and not window[0] <= t <= window[1] + 0.05:
                continue
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


def physical_index(local_rank):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        parts = [p for p in vis.split(",") if p.strip()]
        if local_rank < len(parts) and parts[local_rank].strip().isdigit():
            return int(parts[local_rank])
    return local_rank


# ----------------------------------------------------------------------------- CPU legs

def cpu_sampler(fn_name, n_total, target_s=12.0):
    """A bounded sample of the workload for an oracle Lloyd iteration on the host
    cores, sized to about target_s seconds of CPU work.  -> (run, rows, sample
    text, cores): run() times one iteration over a fresh sample of `rows` points."""
    import numpy as np
    import oracle
    threads = oracle.hardware_threads()
    g = np.random.default_rng(SEED)
    centers = g.uniform(-5, 5, (K_CLUSTERS, D_RAW)).astype(np.float32)

    def sample(n):
        x = np.zeros((n, D_PAD), np.float32)
        x[:, :D_RAW] = centers[g.integers(0, K_CLUSTERS, n)] + 0.75 * g.standard_normal((n, D_RAW)).astype(np.float32)
        return x

    c0 = sample(K_CLUSTERS)

    def run_on(x):
        t = time.perf_counter()
        if fn_name == "lloyd_fp32":
            oracle.lloyd_fp32(x, c0, 1, 0.0, threads)
        else:
            oracle.lloyd_step(x, oracle.l2_norm(x), c0, threads)
        return time.perf_counter() - t

    n = 4096
    t = run_on(sample(n))
    rows = int(min(n_total, max(n, n * target_s / max(t, 1e-3))))
    rows = max(4096, rows // 4096 * 4096)
    kind = "FP32 Lloyd (oracle port of the reference's host-visible algorithm)" if fn_name == "lloyd_fp32" else \
        "MX Lloyd step (oracle port of kmeans_mixed: MXFP8 quantize, product, assign, update)"
    text = f"1 iteration of {kind} over {rows} of the {n_total} points, K={K_CLUSTERS}, D={D_PAD}"
    return (lambda: run_on(sample(rows))), rows, text, threads


def cpu_sample_rate(fn_name, n_total):
    """Point-iterations per second of one bounded sample; -> (rate, sample text, cores)."""
    run, rows, text, cores = cpu_sampler(fn_name, n_total)
    return rows / run(), text, cores


def reference_arm(args, rank):
    """The reference's Lloyd step on the host cores (its GPU path is sm_120a-only):
    W untimed and K timed steps, each one iteration over a bounded sample."""
    if rank != 0:
        return
    steps = max(args.steps, 1)
    run, rows, sample, cores = cpu_sampler("lloyd_step", args.n, target_s=min(12.0, 60.0 / steps))
    for _ in range(max(args.warmup, 0)):
        run()
    seconds = sum(run() for _ in range(steps))
    value = rows * steps / seconds
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": steps, "warmup": args.warmup, "ms_per_step": seconds * 1e3 / steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "mxfp8+f32", "data": "synthetic",
            "config": {"workload": WORKLOAD},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": ("the reference's Lloyd path is sm_120a-only CUDA (no CPU implementation); this arm times the "
                     "oracle's C restatement of kmeans_mixed on the host cores, each step one iteration over a "
                     "bounded sample of the workload")}
    print(json.dumps(line), flush=True)


def run_e2e(torch, dist, mxk, x, c_init, cent, labels, comm, opts, stream, barrier, world, n, rows, args):
    """Same metric through the C ABI from pinned HOST buffers: each step copies the
    rank's points and the initial centroids in, runs kmeans_mixed, and copies the
    labels and final centroids out, all inside the timed region."""
    x_host = x.cpu().pin_memory()
    c_host = c_init.cpu().pin_memory()
    lab_host = torch.empty(rows, dtype=torch.int32).pin_memory()
    cent_host = torch.empty_like(c_host).pin_memory()
    x_dev = torch.empty_like(x)
    e2e_steps = max(1, min(args.steps, 3))

    def e2e_step():
        x_dev.copy_(x_host, non_blocking=True)
        cent.copy_(c_host, non_blocking=True)
        if comm is not None:
            it = mxk.kmeans_mixed_sharded(comm, x_dev, cent, labels, opts)
        else:
            it = mxk.kmeans_mixed(x_dev, cent, labels, opts)
        lab_host.copy_(labels, non_blocking=True)
        cent_host.copy_(cent, non_blocking=True)
        return it

    e2e_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    e2e_iters = 0
    for _ in range(e2e_steps):
        e2e_iters += e2e_step()
    e1.record(stream)
    barrier()
    te = torch.tensor([e0.elapsed_time(e1)], device=x.device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = n * e2e_iters / (float(te.item()) / 1e3)

    return {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": int(x.numel() * 4 + c_init.numel() * 4),
            "d2h_bytes_per_step": int(rows * 4 + c_init.numel() * 4), "steps": e2e_steps}


# ----------------------------------------------------------------------------- GPU arm

def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        reference_arm(args, rank)
        return

    import numpy as np
    import torch
    import torch.distributed as dist
    import mxk

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=600),
                                device_id=dev)
    mxk.load()
    n = args.n
    x_full = make_dataset(torch, n, dev)
    if args.init == "kmeans++":
        # the library's GPU K-Means++: the rows the reference's init_centroids
        # (include/host_utils.hpp:80-119) picks for this seed; untimed set-up
        c_init = torch.empty((K_CLUSTERS, x_full.shape[1]), device=dev)
        mxk.init_kmeanspp(x_full, c_init, SEED)
    else:
        g = torch.Generator(device=dev).manual_seed(SEED)
        c_init = x_full[torch.randperm(n, generator=g, device=dev)[:K_CLUSTERS]].clone()
    row0, rows = mxk.shard_rows(n, world, rank)
    x = x_full[row0:row0 + rows].contiguous()
    del x_full
    torch.cuda.empty_cache()
    cent = torch.empty_like(c_init)
    labels = torch.empty(rows, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream()
    opts = mxk.Options(max_iterations=ITERS, tolerance=0.0)

    comm = mxk.bootstrap_comm() if world > 1 else None

    def step(cache_points=False):
        cent.copy_(c_init)
        if comm is not None:
            return mxk.kmeans_mixed_sharded(comm, x, cent, labels, opts)
        return mxk.kmeans_mixed(x, cent, labels, opts, cache_points=cache_points)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # The clock sampler starts before the warm-up (nvidia-smi takes a while to
    # come up); only the samples that arrive during the timed region are kept.
    sampler = ClockSampler(physical_index(local_rank))
    sampler.start()
    for _ in range(max(args.warmup, 0)):
        step()

    # ---- timed region (device time, CUDA events on the launching stream)
    mxk.profile_enable(True)
    launches0 = mxk.launch_count()
    mxk.gemm_tiles_multiplied(reset=True)
    barrier()
    t_wall0 = time.monotonic()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    iters = 0
    for _ in range(args.steps):
        iters += step()
    ev1.record(stream)
    barrier()
    t_wall1 = time.monotonic()
    launches = mxk.launch_count() - launches0
    tiles_done = mxk.gemm_tiles_multiplied(reset=True)
    stats = mxk.profile_read()
    mxk.profile_enable(False)
    clocks = sampler.stop(window=(t_wall0, t_wall1))
    ms = ev0.elapsed_time(ev1)
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    value = n * iters / (ms_max / 1e3)

    # ---- the opt-in point cache (mxk_kmeans_mixed_cached), reported separately:
    # the points' MXFP8 bytes computed once per call instead of every iteration
    cached = None
    if world == 1 and not args.quick:
        for _ in range(2):
            step(cache_points=True)
        barrier()
        c0e, c1e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0e.record(stream)
        c_iters = sum(step(cache_points=True) for _ in range(args.steps))
        c1e.record(stream)
        barrier()
        c_ms = c0e.elapsed_time(c1e)
        cached = {"value": n * c_iters / (c_ms / 1e3), "unit": UNIT, "ms_per_step": c_ms / args.steps,
                  "steps": args.steps, "api": "mxk_kmeans_mixed_cached",
                  "note": "opt-in: point MXFP8 bytes cached per call (the reference re-quantizes every iteration; "
                          "same results); not the headline"}

    # ---- end to end through the C ABI with host buffers
    e2e = None
    if not args.quick:
        e2e = run_e2e(torch, dist, mxk, x, c_init, cent, labels, comm, opts, stream, barrier, world, n, rows, args)

    # ---- roofline of the dominant kernel (fused MX GEMM + argmin)
    pk, pk_kind = peaks()
    gemm = stats.get("mx_gemm_argmin")
    roofline = None
    if gemm and gemm[0]:
        # Tensor work actually executed: the 128 x 192 tiles the GEMM multiplied
        # (exact pruning skips tiles that cannot hold a nearest centroid), each
        # 2 * 128 * 192 * D_pad FLOPs.  The nominal Lloyd work 2 N K D_pad per
        # iteration is reported beside it.
        flops_per_iter = 2.0 * rows * K_CLUSTERS * D_PAD
        tile_flops = 2.0 * 128 * 192 * D_PAD
        executed = tiles_done * tile_flops
        unpruned = iters * ((rows + 127) // 128) * ((K_CLUSTERS + 191) // 192) * tile_flops
        seconds = gemm[1] / 1e3
        tflops = executed / seconds / 1e12
        peak_tf = 2.0 * pk.get("bf16_tflops_sustained", pk.get("bf16_tflops"))
        # algorithmic DRAM bytes per launch: each point's FP32 row (quantized in
        # the kernel), its id, norm, previous label, new label and distance,
        # and in the pruned iterations (all but the first) its 8-byte bound record
        alg_bytes = rows * (4.0 * D_PAD + 20.0 + 8.0 * (ITERS - 1) / ITERS)
        gbs = alg_bytes * iters / seconds / 1e9
        peak_gbs = pk.get("hbm_gbs", 6650.0)
        # the binding roofline is the one whose ideal time is longer
        hbm_bound = alg_bytes / (peak_gbs * 1e9) > (executed / max(iters, 1)) / (peak_tf * 1e12)
        traffic = measured_traffic(rows)
        roofline = {"bound": "hbm" if hbm_bound else "tensor",
                    "achieved": gbs if hbm_bound else tflops, "peak": peak_gbs if hbm_bound else peak_tf,
                    "unit": "GB/s" if hbm_bound else "TFLOP/s",
                    "frac": gbs / peak_gbs if hbm_bound else tflops / peak_tf, "traffic": traffic,
                    "algorithmic_bytes_per_launch": alg_bytes,
                    "tensor_tflops_executed": tflops, "tensor_frac_executed": tflops / peak_tf,
                    "traffic_unit": "DRAM bytes per launch of a pruned iteration (ncu capture of iteration 10 "
                                    "scaled to these rows; profiles/mx_gemm_argmin_config4.md)",
                    "kernel": "mx_gemm_argmin", "ms_per_iteration": gemm[1] / max(iters, 1),
                    "executed_flops_per_iteration": executed / max(iters, 1),
                    "nominal_flops_per_iteration": flops_per_iter,
                    "tiles_multiplied_fraction": executed / unpruned if unpruned else None,
                    "nominal_tflops": flops_per_iter * iters / (gemm[1] / 1e3) / 1e12,
                    "peak_source": f"hbm_gbs, 2 x bf16_tflops_sustained of {pk_kind} MEASURED_PEAKS.json "
                                   "(dense MXFP8 tensor rate is twice BF16)"}
    kernel_ms = {k: {"launches": v[0], "total_ms": round(v[1], 3)} for k, v in sorted(stats.items(), key=lambda kv: -kv[1][1])}
    update = update_roofline(stats, rows, pk.get("hbm_gbs", 6650.0))

    cpu = None
    if rank == 0 and world == 1 and not args.quick:
        v, sample, cores = cpu_sample_rate("lloyd_fp32", n)
        cpu = {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "mxfp8+f32", "data": "synthetic",
                "config": {"workload": WORKLOAD, "points": n, "dims": D_PAD, "clusters": K_CLUSTERS,
                           "iterations_per_step": iters / args.steps, "parallelism": f"row-shard x{world}",
                           "l2": "inputs (4.3 GB of points per step) larger than the 126 MB L2"},
                "e2e": e2e,
                "gpu_launches": int(launches), "roofline": roofline, "update_roofline": update,
                "cpu_baseline": cpu, "clocks": clocks,
                "cached_points": cached,
                "kernel_ms": kernel_ms}
        print(json.dumps(line), flush=True)
    if comm is not None:
        comm.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
