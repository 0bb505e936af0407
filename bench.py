"""Benchmark of the MX-KMeans Lloyd iteration on B200 (metric: Lloyd
point-iterations/sec; MX-GEMM fraction of tensor peak).

Default workload (the headline): configs[3] -- N = 8,388,608 points,
D = 96 zero-padded to 128, K = 2048 clusters, seeded Gaussian blobs (centers
U[-5,5], sigma 0.75, seed 3), K-Means++ initial centroids, 20 Lloyd iterations
with tol 0 (a run can stop earlier on an exactly unchanged shift; the reported
rate uses the iterations actually run).  One step = one kmeans_mixed call over
the whole dataset, from the same initial centroids (the reference CLI's timed
unit, src/main.cu:115-123).  --config 1, 2 or 4 selects the other benchmark
configurations (their own N, D, K, data, initialisation and iterations) for
the per-kernel rooflines they add (the point quantize at D = 256 and 768); the
driver's headline line is configs[3].  With --gpus N (torchrun, one rank per
GPU) the points are row-sharded and every iteration NCCL-allreduces the K x D
sums and K counts: strong scaling of the fixed N.

    python bench.py [--config C] [--gpus N] [--steps K] [--warmup W] [--impl reference]
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

METRIC = "Lloyd point-iters/sec"
UNIT = "point-iters/s"

# The benchmark's configs[1..4] (configs[0] is the reference's CPU quick-start
# case, covered by the parity tests).  Data are seeded synthetic stand-ins with
# each configuration's shapes and distributions (no dataset is named).
CONFIGS = {
    1: dict(n=1048576, d_raw=128, d_pad=128, k=256, seed=7, init="kmeans++", iters=50, tol=1e-4, gen="blobs_varstd",
            text="configs[1]: N=1048576, D=128, K=256, blobs centers U[-10,10]^128 per-cluster sigma U[0.5,2.0], "
                 "seed 7, K-Means++ init, maxiter 50 (tol 1e-4), MXFP8 points/centroids, FP32 update"),
    2: dict(n=4194304, d_raw=256, d_pad=256, k=1024, seed=11, init="farthest", iters=30, tol=1e-4, gen="blobs_scaled",
            text="configs[2]: N=4194304, D=256, K=1024, blobs centers U[-10,10]^256 sigma 1.0 then per-feature "
                 "scale 2^U[-8,8], seed 11, farthest-first init, maxiter 30 (tol 1e-4), MXFP8 points/centroids"),
    3: dict(n=8388608, d_raw=96, d_pad=128, k=2048, seed=3, init="kmeans++", iters=20, tol=0.0, gen="blobs",
            text="configs[3]: N=8388608, D=96 zero-padded to 128, K=2048, blobs centers U[-5,5]^96 sigma 0.75, "
                 "seed 3, K-Means++ init, 20 iterations (tol 0), MXFP8 points/centroids, FP32 update"),
    4: dict(n=16777216, d_raw=768, d_pad=768, k=8192, seed=19, init="kmeans++sub", iters=10, tol=0.0, gen="sphere_zipf",
            text="configs[4]: N=16777216, D=768, K=8192, unit-sphere centers + N(0,0.05^2) renormalised, Zipf(1.1) "
                 "cluster sizes, seed 19, K-Means++ on a 1M-point subsample, 10 iterations (tol 0), MXFP8"),
}
HEADLINE = 3
_H = CONFIGS[HEADLINE]
N_POINTS, D_RAW, D_PAD, K_CLUSTERS, ITERS, SEED = _H["n"], _H["d_raw"], _H["d_pad"], _H["k"], _H["iters"], _H["seed"]
WORKLOAD = _H["text"]


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--config", type=int, default=HEADLINE, choices=sorted(CONFIGS),
                   help="the benchmark's configs[C] (default: configs[3], the headline)")
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="mxk", choices=["mxk", "reference"])
    # profiling aids (the committed ncu commands use them; bench lines never do)
    p.add_argument("--n", type=int, default=0, help="points (default: the configuration's N)")
    p.add_argument("--init", default="kmeans++", choices=["kmeans++", "random"],
                   help="random = K distinct random rows (fast set-up for profiling runs)")
    p.add_argument("--quick", action="store_true", help="skip the e2e and CPU-baseline legs")
    return p.parse_args()


def measured_traffic(rows_per_launch, cfg):
    """dram__bytes_read.sum + dram__bytes_write.sum per fused-GEMM launch at
    the DRAM bytes per processed point row of every GEMM launch of
    one 20-iteration call, from the committed summary of that ncu capture,
    times the rows a launch processed here on average; None for the other
    configurations or if the summary is missing."""
    if cfg is not CONFIGS[HEADLINE]:
        return None
    path = os.path.join(ROOT, "profiles", "mx_gemm_argmin_config4.md")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_row:"):
                return float(line.split(":")[1]) * rows_per_launch
    except OSError:
        pass
    return None


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def update_roofline(stats, rows, d_pad, peak_gbs):
    """Achieved HBM bandwidth of the centroid update (the label-run or
    privatised accumulation pass, one launch per iteration) from its CUDA-event
    times in `stats` ({kernel: (launches, total_ms)}): algorithmic bytes per
    launch = each point's FP32 row, its id and its label, rows * (4 D_pad + 8).
    None when the pass did not run."""
    launches = sum(stats.get(k, (0, 0.0))[0] for k in ("accumulate_runs", "accumulate_private"))
    total_ms = sum(stats.get(k, (0, 0.0))[1] for k in ("accumulate_runs", "accumulate_private"))
    if not launches or total_ms <= 0.0:
        return None
    alg_bytes = rows * (4.0 * d_pad + 8.0)
    gbs = alg_bytes * launches / (total_ms / 1e3) / 1e9
    return {"bound": "hbm", "achieved": gbs, "peak": peak_gbs, "unit": "GB/s", "frac": gbs / peak_gbs,
            "algorithmic_bytes_per_launch": alg_bytes, "ms_per_launch": total_ms / launches,
            "launches": launches, "kernel": "accumulate_runs"}


def quantize_roofline(stats, rows_total, d_pad, peak_gbs, iterations):
    """Achieved HBM bandwidth of the per-iteration point quantize
    (quantize_rows on the rows the GEMM processes, in visiting order, MXFP8,
    the scale atoms of the GEMM's point tiles) from its CUDA-event times:
    algorithmic bytes = rows_total (all rows quantized in the timed region) *
    (4 D_pad read + D_pad values + D_pad / 32 scales written + 4 for the row's
    point id), over the launches' total time (launches enqueued after the loop
    stopped do nothing and count only their few microseconds).  None when the
    quantize is fused into the GEMM (D = 128) and has no launch of its own."""
    launches, total_ms = stats.get("quantize_points", (0, 0.0))
    if not launches or total_ms <= 0.0 or iterations <= 0:
        return None
    alg_bytes = rows_total * (5.0 * d_pad + d_pad / 32.0 + 4.0)
    gbs = alg_bytes / (total_ms / 1e3) / 1e9
    return {"bound": "hbm", "achieved": gbs, "peak": peak_gbs, "unit": "GB/s", "frac": gbs / peak_gbs,
            "algorithmic_bytes_per_iteration": alg_bytes / iterations, "ms_per_iteration": total_ms / iterations,
            "launches": launches, "kernel": "quantize_points"}


# ----------------------------------------------------------------------------- data

def make_dataset(torch, n, device, cfg=None):
    """Seeded synthetic points of a benchmark configuration on the device
    (identical on every rank), zero-padded to D_pad."""
    cfg = cfg or CONFIGS[HEADLINE]
    k, d_raw, d_pad, seed = cfg["k"], cfg["d_raw"], cfg["d_pad"], cfg["seed"]
    g = torch.Generator(device=device).manual_seed(seed)
    gen = cfg["gen"]
    x = torch.zeros((n, d_pad), device=device)
    chunk = 1 << 22  # (the headline's random stream: same chunking as its first measurements)
    if gen == "sphere_zipf":
        centers = torch.randn((k, d_raw), generator=g, device=device)
        centers /= centers.norm(dim=1, keepdim=True)
        w = torch.arange(1, k + 1, device=device, dtype=torch.float64).pow(-1.1)
        cdf = (w.cumsum(0) / w.sum()).float()
        for s in range(0, n, chunk):
            e = min(n, s + chunk)
            u = torch.rand((e - s,), generator=g, device=device)
            lab = torch.searchsorted(cdf, u).clamp_(max=k - 1)
            v = centers[lab] + 0.05 * torch.randn((e - s, d_raw), generator=g, device=device)
            x[s:e, :d_raw] = v / v.norm(dim=1, keepdim=True)
        return x
    spread = 5.0 if gen == "blobs" else 10.0
    centers = torch.rand((k, d_raw), generator=g, device=device) * (2 * spread) - spread
    sigma = (torch.rand((k, 1), generator=g, device=device) * 1.5 + 0.5 if gen == "blobs_varstd"
             else torch.full((k, 1), 0.75 if gen == "blobs" else 1.0, device=device))
    scale = (torch.pow(2.0, torch.rand((d_raw,), generator=g, device=device) * 16.0 - 8.0)
             if gen == "blobs_scaled" else None)
    labels = torch.randint(0, k, (n,), generator=g, device=device)
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        lab = labels[s:e]
        v = centers[lab] + sigma[lab] * torch.randn((e - s, d_raw), generator=g, device=device)
        x[s:e, :d_raw] = v * scale if scale is not None else v
    return x


def initial_centroids(torch, mxk, x, cfg, init):
    """The configuration's initialisation with the library's GPU versions of the
    reference's functions (the rows include/host_utils.hpp:80-141 picks for the
    seed); untimed set-up."""
    k, seed = cfg["k"], cfg["seed"]
    c = torch.empty((k, x.shape[1]), device=x.device)
    if init == "random":
        g = torch.Generator(device=x.device).manual_seed(seed)
        return x[torch.randperm(x.shape[0], generator=g, device=x.device)[:k]].clone()
    if cfg["init"] == "farthest":
        mxk.init_farthest(x, c)
    elif cfg["init"] == "kmeans++sub":
        mxk.init_kmeanspp(x[:min(x.shape[0], 1 << 20)], c, seed)  # the i.i.d. rows' first 1M
    else:
        mxk.init_kmeanspp(x, c, seed)
    return c


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

def cpu_sampler(fn_name, cfg, n_total, target_s=12.0):
    """A bounded sample of the workload for an oracle Lloyd iteration on the host
    cores, sized to about target_s seconds of CPU work.  -> (run, rows, sample
    text, cores): run() times one iteration over a fresh sample of `rows` points
    drawn from the configuration's distribution."""
    import numpy as np
    import oracle
    threads = oracle.hardware_threads()
    k, d_raw, d_pad, gen = cfg["k"], cfg["d_raw"], cfg["d_pad"], cfg["gen"]
    g = np.random.default_rng(cfg["seed"])
    if gen == "sphere_zipf":
        centers = g.standard_normal((k, d_raw)).astype(np.float32)
        centers /= np.linalg.norm(centers, axis=1, keepdims=True)
        w = np.arange(1, k + 1, dtype=np.float64) ** -1.1
        p = w / w.sum()
    else:
        spread = 5.0 if gen == "blobs" else 10.0
        centers = g.uniform(-spread, spread, (k, d_raw)).astype(np.float32)
        p = None
    sig = (g.uniform(0.5, 2.0, (k, 1)) if gen == "blobs_varstd" else
           np.full((k, 1), 0.75 if gen == "blobs" else (0.05 if gen == "sphere_zipf" else 1.0))).astype(np.float32)
    scale = (2.0 ** g.uniform(-8, 8, d_raw)).astype(np.float32) if gen == "blobs_scaled" else None

    def sample(n):
        lab = g.choice(k, n, p=p) if p is not None else g.integers(0, k, n)
        v = centers[lab] + sig[lab] * g.standard_normal((n, d_raw)).astype(np.float32)
        if gen == "sphere_zipf":
            v /= np.linalg.norm(v, axis=1, keepdims=True)
        if scale is not None:
            v *= scale
        x = np.zeros((n, d_pad), np.float32)
        x[:, :d_raw] = v
        return x

    c0 = sample(k)

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
    text = f"1 iteration of {kind} over {rows} of the {n_total} points, K={k}, D={d_pad}"
    return (lambda: run_on(sample(rows))), rows, text, threads


def cpu_sample_rate(fn_name, cfg, n_total):
    """Point-iterations per second of one bounded sample; -> (rate, sample text, cores)."""
    run, rows, text, cores = cpu_sampler(fn_name, cfg, n_total)
    return rows / run(), text, cores


def reference_arm(args, cfg, rank):
    """The reference's Lloyd step on the host cores (its GPU path is sm_120a-only):
    W untimed and K timed steps, each one iteration over a bounded sample."""
    if rank != 0:
        return
    steps = max(args.steps, 1)
    n = args.n or cfg["n"]
    run, rows, sample, cores = cpu_sampler("lloyd_step", cfg, n, target_s=min(12.0, 60.0 / steps))
    for _ in range(max(args.warmup, 0)):
        run()
    seconds = sum(run() for _ in range(steps))
    value = rows * steps / seconds
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": steps, "warmup": args.warmup, "ms_per_step": seconds * 1e3 / steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "mxfp8+f32", "data": "synthetic",
            "config": {"workload": cfg["text"]},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": ("the reference's Lloyd path is sm_120a-only CUDA (no CPU implementation); this arm times the "
                     "oracle's C restatement of kmeans_mixed on the host cores, each step one iteration over a "
                     "bounded sample of the workload")}
    print(json.dumps(line), flush=True)


def run_e2e(torch, dist, mxk, x, c_init, cent, labels, comm, opts, stream, barrier, world, n, rows, args):
    """Same metric end to end from pinned HOST buffers, copies inside the timed
    region.  One GPU: the library's host-buffer entry mxk_kmeans_mixed_multi
    (num_gpus = 1: it allocates, uploads the points and initial centroids, runs
    kmeans_mixed and downloads labels and centroids), timed by the host clock
    around the blocking call.  Several ranks (one process per GPU): each rank
    copies its shard and the centroids in, runs kmeans_mixed_sharded and copies
    labels and centroids out, timed with CUDA events (max over ranks)."""
    e2e_steps = max(1, min(args.steps, 3))
    x_host = x.cpu().pin_memory()
    c_host = c_init.cpu().pin_memory()
    lab_host = torch.empty(rows, dtype=torch.int32).pin_memory()
    cent_host = torch.empty_like(c_host).pin_memory()
    h2d = int(x.numel() * 4 + c_init.numel() * 4)
    d2h = int(rows * 4 + c_init.numel() * 4)
    if world == 1:
        xn, ln, cn = x_host.numpy(), lab_host.numpy(), cent_host.numpy()

        def call():
            cn[...] = c_host.numpy()
            return mxk.kmeans_mixed_multi(xn, cn, ln, opts, 1)

        call()
        barrier()
        t0 = time.perf_counter()
        e2e_iters = sum(call() for _ in range(e2e_steps))
        seconds = time.perf_counter() - t0
        return {"value": n * e2e_iters / seconds, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "steps": e2e_steps, "api": "mxk_kmeans_mixed_multi (host buffers)"}

    x_dev = torch.empty_like(x)

    def e2e_step():
        x_dev.copy_(x_host, non_blocking=True)
        cent.copy_(c_host, non_blocking=True)
        it = mxk.kmeans_mixed_sharded(comm, x_dev, cent, labels, opts)
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
    dist.all_reduce(te, op=dist.ReduceOp.MAX)
    return {"value": n * e2e_iters / (float(te.item()) / 1e3), "unit": UNIT, "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "steps": e2e_steps, "api": "mxk_kmeans_mixed_sharded from pinned host copies"}


def dense_roofline(torch, mxk, x, cent, labels, cfg, stream, peak_tf, launches=10):
    """The same fused GEMM + argmin with no tile mask (every 128 x 192 tile
    multiplied), on the loop's final centroids with its label-sorted visiting
    order and previous labels as sweep hints (the steady-state unpruned
    iteration), timed with CUDA events: executed TFLOP/s against the dense
    MXFP8 rate, 2 x bf16_tflops_sustained."""
    n, d, k = x.shape[0], x.shape[1], cent.shape[0]
    dev = x.device
    qc = torch.empty(k * d, dtype=torch.uint8, device=dev)
    sc = torch.empty(k * d // 32, dtype=torch.uint8, device=dev)
    mxk.quantize_rows(8, cent, qc, sc)
    pn = torch.empty(n, device=dev)
    mxk.compute_l2_norm(x, pn)
    cn = torch.empty(k, device=dev)
    mxk.compute_l2_norm(cent, cn)
    order = torch.argsort(labels, stable=True).to(torch.int32)
    out = torch.empty(n, dtype=torch.int32, device=dev)
    if d == 128:  # the loop's fused-quantize kernel
        def launch():
            mxk.assign_f32_fused(n, k, d, x, qc, sc, pn, cn, out, pid=order, start_hint=labels)
        kind = "fused quantize + MXFP8 GEMM + argmin (mxk_assign_f32_fused), no tile mask"
    else:
        qx = torch.empty(n * d, dtype=torch.uint8, device=dev)
        sx = torch.empty(n * d // 32, dtype=torch.uint8, device=dev)
        mxk.quantize_rows(8, x, qx, sx)

        def launch():
            mxk.assign_mx_fused(8, n, k, d, qx, sx, qc, sc, pn, cn, out, pid=order, start_hint=labels)
        kind = "MXFP8 GEMM + argmin (mxk_assign_mx_fused), no tile mask"
    for _ in range(2):
        launch()
    torch.cuda.synchronize()
    mxk.gemm_tiles_multiplied(reset=True)
    # the kernel's own time from the library's per-launch CUDA events (host
    # work between the API calls -- tensor maps, the centroid scale layout --
    # is not the kernel's); the calls' bracketing time is reported beside it
    mxk.profile_enable(True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(launches):
        launch()
    e1.record(stream)
    torch.cuda.synchronize()
    stats = mxk.profile_read()
    mxk.profile_enable(False)
    tiles = mxk.gemm_tiles_multiplied(reset=True)
    call_ms = e0.elapsed_time(e1) / launches
    gemm = stats.get("mx_gemm_argmin", (0, 0.0))
    ms = gemm[1] / gemm[0] if gemm[0] else call_ms
    executed = tiles / launches * 2.0 * 128 * 192 * d
    nominal = 2.0 * n * k * d
    tf = executed / (ms / 1e3) / 1e12
    return {"bound": "tensor", "achieved": tf, "peak": peak_tf, "unit": "TFLOP/s", "frac": tf / peak_tf,
            "ms_per_launch": ms, "ms_per_api_call": call_ms,
            "executed_flops_per_launch": executed, "nominal_flops_per_launch": nominal,
            "nominal_tflops": nominal / (ms / 1e3) / 1e12, "launches": launches, "kernel": kind}


# ----------------------------------------------------------------------------- GPU arm

def main():
    args = parse()
    cfg = CONFIGS[args.config]
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        reference_arm(args, cfg, rank)
        return

    import torch
    import torch.distributed as dist
    import mxk

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=600),
                                device_id=dev)
    mxk.load()
    n = args.n or cfg["n"]
    k, d_pad, iters_cfg = cfg["k"], cfg["d_pad"], cfg["iters"]
    x_full = make_dataset(torch, n, dev, cfg)
    c_init = initial_centroids(torch, mxk, x_full, cfg, args.init)
    row0, rows = mxk.shard_rows(n, world, rank)
    x = x_full[row0:row0 + rows].contiguous()
    del x_full
    torch.cuda.empty_cache()
    cent = torch.empty_like(c_init)
    labels = torch.empty(rows, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream()
    opts = mxk.Options(max_iterations=iters_cfg, tolerance=cfg["tol"])

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
    mxk.gemm_rows_processed(reset=True)
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
    rows_done = mxk.gemm_rows_processed(reset=True)
    stats = mxk.profile_read()
    mxk.profile_enable(False)
    clocks = sampler.stop(window=(t_wall0, t_wall1))
    ms = ev0.elapsed_time(ev1)
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    value = n * iters / (ms_max / 1e3)

    pk, pk_kind = peaks()
    peak_gbs = pk.get("hbm_gbs", 6650.0)
    peak_tf = 2.0 * pk.get("bf16_tflops_sustained", pk.get("bf16_tflops"))

    # ---- the dense (unpruned) MX GEMM on the final state, and the opt-in point
    # cache (mxk_kmeans_mixed_cached), reported beside the headline
    dense = None
    cached = None
    if world == 1 and not args.quick:
        dense = dense_roofline(torch, mxk, x, cent, labels, cfg, stream, peak_tf)
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

    # ---- end to end with host buffers
    e2e = None
    if not args.quick:
        e2e = run_e2e(torch, dist, mxk, x, c_init, cent, labels, comm, opts, stream, barrier, world, n, rows, args)

    # ---- roofline of the dominant kernel (fused MX GEMM + argmin)
    gemm = stats.get("mx_gemm_argmin")
    roofline = None
    if gemm and gemm[0]:
        # Tensor work actually executed: the 128 x 192 tiles the GEMM multiplied
        # (exact pruning skips tiles that cannot hold a nearest centroid), each
        # 2 * 128 * 192 * D_pad FLOPs.  The nominal Lloyd work 2 N K D_pad per
        # iteration is reported beside it.
        flops_per_iter = 2.0 * rows * k * d_pad
        tile_flops = 2.0 * 128 * 192 * d_pad
        executed = tiles_done * tile_flops
        unpruned = iters * ((rows + 127) // 128) * ((k + 191) // 192) * tile_flops
        seconds = gemm[1] / 1e3
        tflops = executed / seconds / 1e12
        # algorithmic DRAM bytes: for each point row the GEMM processed (rows
        # whose labels the bounds proved beforehand leave it), the row (FP32,
        # quantized in the kernel, at D = 128; else its MXFP8 bytes and scales),
        # its id, norm, previous label, new label and distance, and in the
        # pruned iterations (all but each call's first) its 8-byte bound record
        per_row = 4.0 * d_pad if d_pad == 128 else d_pad + d_pad / 32.0
        first_rows = rows * args.steps  # the first iteration of each call is unpruned
        bytes_total = rows_done * (per_row + 20.0) + max(rows_done - first_rows, 0) * 8.0
        alg_bytes = bytes_total / max(iters, 1)
        gbs = bytes_total / seconds / 1e9
        # the binding roofline is the one whose ideal time is longer
        hbm_bound = alg_bytes / (peak_gbs * 1e9) > (executed / max(iters, 1)) / (peak_tf * 1e12)
        traffic = measured_traffic(rows_done / max(iters, 1), cfg)
        roofline = {"bound": "hbm" if hbm_bound else "tensor",
                    "achieved": gbs if hbm_bound else tflops, "peak": peak_gbs if hbm_bound else peak_tf,
                    "unit": "GB/s" if hbm_bound else "TFLOP/s",
                    "frac": gbs / peak_gbs if hbm_bound else tflops / peak_tf, "traffic": traffic,
                    "traffic_source": ("ncu capture (dram__bytes_read.sum + dram__bytes_write.sum) of every GEMM "
                                       "launch of one 20-iteration call at N = 2,097,152, per processed row, times "
                                       "this run's rows per launch; profiles/mx_gemm_argmin_config4.md; not "
                                       "measured in this run") if traffic else None,
                    "algorithmic_bytes_per_launch": alg_bytes,
                    "tensor_tflops_executed": tflops, "tensor_frac_executed": tflops / peak_tf,
                    "kernel": "mx_gemm_argmin", "ms_per_iteration": gemm[1] / max(iters, 1),
                    "executed_flops_per_iteration": executed / max(iters, 1),
                    "nominal_flops_per_iteration": flops_per_iter,
                    "tiles_multiplied_fraction": executed / unpruned if unpruned else None,
                    "rows_processed_fraction": rows_done / (rows * iters) if iters else None,
                    "nominal_tflops": flops_per_iter * iters / (gemm[1] / 1e3) / 1e12,
                    "peak_source": f"hbm_gbs, 2 x bf16_tflops_sustained of {pk_kind} MEASURED_PEAKS.json "
                                   "(dense MXFP8 tensor rate is twice BF16)"}
    kernel_ms = {kk: {"launches": v[0], "total_ms": round(v[1], 3)}
                 for kk, v in sorted(stats.items(), key=lambda kv: -kv[1][1])}
    update = update_roofline(stats, rows, d_pad, peak_gbs)
    # (the point quantize encodes the rows the GEMM processes)
    quant = quantize_roofline(stats, rows_done, d_pad, peak_gbs, iters)

    cpu = None
    if rank == 0 and world == 1 and not args.quick:
        v, sample, cores = cpu_sample_rate("lloyd_fp32", cfg, n)
        cpu = {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "mxfp8+f32", "data": "synthetic",
                "config": {"workload": cfg["text"], "points": n, "dims": d_pad, "clusters": k,
                           "iterations_per_step": iters / args.steps, "parallelism": f"row-shard x{world}",
                           "l2": f"inputs ({n * d_pad * 4 / 1e9:.1f} GB of points per step) larger than the "
                                 "126 MB L2"},
                "e2e": e2e,
                "gpu_launches": int(launches), "roofline": roofline, "roofline_dense": dense,
                "update_roofline": update, "quantize_roofline": quant,
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
