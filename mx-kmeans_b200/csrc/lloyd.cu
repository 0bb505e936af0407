// Lloyd driver of MX-KMeans on one GPU or on row shards over several GPUs.
//
// Reference: ParCIS/MX-KMeans src/kmeans.cu:12-68 (kmeans_mixed).  Per iteration,
// in the reference's order:
//   previous = centroids; centroid norms;
//   FP32 iteration (it < fp32_iterations): FP32 product + assignment; or
//   MX iteration: centroids -> MXFP8 (+ max squared error); ec, lc; precision of
//   every point (select_precision: always MXFP8); stable per-precision compaction;
//   for bits in {4,6,8}: quantize the group's points, product, assignment;
//   update (sums, counts, empty-cluster keep); shift; stop when shift <= tol.
//
// Differences of form, not of result: ec/lc and the group sizes stay on the
// device (no host round trips), the per-group quantize/GEMM read their row
// counts from device memory, the product and assignment are one tcgen05 kernel
// (no N x K buffer), workspaces come from the stream-ordered allocator, and the
// shift is reduced in a fixed order so every rank of a sharded run sees the same
// value.  The stopping rule runs on the device: the shift kernel sets a stop
// word that turns every later launch of the call into a no-op, so the host
// enqueues up to kLookahead iterations beyond the last one whose state it has
// read and never waits on the GPU between iterations (the reference reads the
// shift back and synchronizes every iteration).  Labels, centroids and the
// returned iteration count are those of the iteration that met the rule.  The
// update kernel also keeps the previous centroids (the reference's copy at the
// top of the iteration), zeroes the sums for the next iteration and writes the
// loop state into pinned host memory, so an iteration issues no copies or
// memsets.
//
// The reference's precision policy ignores the two-largest distance gap
// (include/precision.hpp:20-26), so under it the driver's fused assignment does
// not track the gap and puts every point in the MXFP8 group without running the
// policy, the point bounds or the compaction (the same groups).  The test hook
// mxk_set_precision_policy(1) lets precision_candidate's choice stand instead;
// the driver then runs the reference's full sequence: point bounds, gaps, the
// policy kernel, the stable compaction and one quantize + GEMM per group.
#include <dlfcn.h>

#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include <nccl.h>

#include "common.cuh"
#include "kernels.cuh"
#include "precision.hpp"
#include "watchdog.hpp"

namespace mxk {

// ---------------------------------------------------------------------------
// NCCL, loaded on first use (the single-GPU library has no NCCL dependency).

struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
    bool ok = false;
};

static NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
#define MXK_SYM(field, name) api.field = reinterpret_cast<decltype(api.field)>(dlsym(h, name))
        MXK_SYM(GetUniqueId, "ncclGetUniqueId");
        MXK_SYM(CommInitRank, "ncclCommInitRank");
        MXK_SYM(CommDestroy, "ncclCommDestroy");
        MXK_SYM(CommAbort, "ncclCommAbort");
        MXK_SYM(CommGetAsyncError, "ncclCommGetAsyncError");
        MXK_SYM(AllReduce, "ncclAllReduce");
        MXK_SYM(GroupStart, "ncclGroupStart");
        MXK_SYM(GroupEnd, "ncclGroupEnd");
        MXK_SYM(GetErrorString, "ncclGetErrorString");
#undef MXK_SYM
        api.ok = api.GetUniqueId && api.CommInitRank && api.CommDestroy && api.AllReduce && api.GroupStart &&
                 api.GroupEnd && api.GetErrorString;
    });
    return api;
}

static int fail_nccl(const char* what, ncclResult_t r) {
    return fail(MXK_ERR_COMM, std::string(what) + ": " + (nccl().GetErrorString ? nccl().GetErrorString(r) : "?"));
}

struct Comm {
    ncclComm_t comm = nullptr;  // null once aborted by the watchdog
    int nranks = 1, rank = 0;
    // Set by mxk_kmeans_mixed_multi, whose ranks are threads of one process: a
    // flag any rank raises when it fails, so that the others stop waiting for
    // its collectives (their host waits poll it and abort their communicator).
    std::atomic<int>* group_failed = nullptr;
};

// Test hook (mxk_inject_rank_failure): the sharded loop of this rank returns an
// error on the host when it reaches this iteration, after the work it has
// enqueued has finished (a rank that leaves between steps).
static std::atomic<int> g_inject_rank{-1};
static std::atomic<int> g_inject_iteration{-1};

// Seconds without progress after which a sharded run aborts its communicator
// (environment variable MXK_COMM_TIMEOUT_S; unset or <= 0: wait without limit,
// as a blocking synchronize does).
static double comm_timeout_s() {
    static const double v = [] {
        const char* e = std::getenv("MXK_COMM_TIMEOUT_S");
        return e ? std::atof(e) : 0.0;
    }();
    return v;
}

// Waits for ev.  In a sharded run with MXK_COMM_TIMEOUT_S set, polls the event
// and the communicator's asynchronous error instead (guarded_wait): a failed
// peer, or no progress within the limit, aborts the communicator -- its
// collectives in flight then return -- and the call reports an error instead
// of blocking for good.  An aborted communicator must be destroyed and made
// again.
// The same polling (without a time limit unless MXK_COMM_TIMEOUT_S is set)
// runs whenever the communicator belongs to a group of threads of this process
// (mxk_kmeans_mixed_multi), which a failed rank signals through its flag.
static bool polled_waits(const Comm* comm) {
    return comm && comm->nranks > 1 && comm->comm && (comm_timeout_s() > 0.0 || comm->group_failed) &&
           nccl().CommGetAsyncError && nccl().CommAbort;
}

static int wait_event(Comm* comm, cudaEvent_t ev) {
    const double limit = comm_timeout_s();
    if (!polled_waits(comm)) {
        MXK_CUDA(cudaEventSynchronize(ev));
        return MXK_OK;
    }
    NcclApi& api = nccl();
    cudaError_t query_error = cudaSuccess;
    ncclResult_t peer_error = ncclSuccess;
    const WaitResult r = guarded_wait(
        [&] {
            const cudaError_t e = cudaEventQuery(ev);
            if (e == cudaSuccess) return Probe::kReady;
            if (e == cudaErrorNotReady) return Probe::kPending;
            query_error = e;
            return Probe::kFailed;
        },
        [&] {
            if (comm->group_failed && comm->group_failed->load()) {
                peer_error = ncclRemoteError;
                return true;
            }
            ncclResult_t async = ncclSuccess;
            const ncclResult_t q = api.CommGetAsyncError(comm->comm, &async);
            peer_error = q != ncclSuccess ? q : async;
            return peer_error != ncclSuccess && peer_error != ncclInProgress;
        },
        limit, monotonic_seconds, short_pause);
    if (r == WaitResult::kReady) return MXK_OK;
    if (r == WaitResult::kFailed) return fail_cuda("cudaEventQuery", query_error);
    api.CommAbort(comm->comm);
    comm->comm = nullptr;
    if (r == WaitResult::kPeerFailed)
        return fail_nccl("sharded Lloyd: a peer rank failed, communicator aborted", peer_error);
    return fail(MXK_ERR_TIMEOUT, "sharded Lloyd: no progress within MXK_COMM_TIMEOUT_S seconds, communicator aborted");
}

// ---------------------------------------------------------------------------
// Precision policy of the Lloyd loop (mxk_set_precision_policy): 0 = the
// reference's select_precision (always MXFP8), 1 = the candidate it computes
// and discards, which puts points in the MXFP4/MXFP6 groups.

static std::atomic<int> g_precision_policy{0};

// One-shot per-device trace of the next Lloyd call (mxk_trace_next_call).
struct TraceRequest {
    float* centroids = nullptr;
    int* labels = nullptr;
    int* group_sizes = nullptr;
    int max_iterations = 0;
};
static std::mutex g_trace_mutex;
static TraceRequest g_trace[64];

static TraceRequest take_trace(int device) {
    std::lock_guard<std::mutex> lock(g_trace_mutex);
    if (device < 0 || device >= 64) return TraceRequest{};
    const TraceRequest t = g_trace[device];
    g_trace[device] = TraceRequest{};
    return t;
}

// ---------------------------------------------------------------------------
// Workspace: stream-ordered allocations from the library's per-device pool,
// returned to it at the end of the call.  The pool keeps the memory mapped, so a
// repeated call does not map its ~1.4 GB of workspace again;
// mxk_release_workspace gives it back to the driver.

namespace {

struct Arena {
    cudaStream_t stream;
    std::vector<void*> ptrs;
    explicit Arena(cudaStream_t s) : stream(s) {}
    ~Arena() {
        for (void* p : ptrs) cudaFreeAsync(p, stream);
    }
    template <typename T>
    int alloc(T** out, int64_t count) {
        void* p = nullptr;
        const size_t bytes = sizeof(T) * (size_t)(count > 0 ? count : 1);
        cudaMemPool_t pool = workspace_pool();
        if (!pool) return fail(MXK_ERR_CUDA, "kmeans workspace: cannot create the memory pool");
        cudaError_t e = cudaMallocFromPoolAsync(&p, bytes, pool, stream);
        if (e != cudaSuccess) return fail_cuda("cudaMallocAsync (kmeans workspace)", e);
        ptrs.push_back(p);
        *out = static_cast<T*>(p);
        return MXK_OK;
    }
};

constexpr int64_t kFp32ChunkBytes = 512ll << 20;  // dense product chunk of the FP32 iterations
// Iterations enqueued ahead of the last one whose loop state the host has read.
// About 40 ms of GPU work at the benchmark shape, so a host thread descheduled or
// held in the driver for that long does not leave the GPU idle.
constexpr int kLookahead = 8;
// Row chunks of a host-buffer call's upload (bytes of points per chunk).
constexpr int64_t kUploadChunkBytes = 256ll << 20;
// Outside the pruned iterations of the fused path, the label-sorted visiting
// order is rebuilt every kResortEvery iterations.  It only shapes performance
// (assignments are per point; the update's FP64 sums are order-dependent in
// their last bits, as the reference's FP32 atomics are), and after the first
// iterations few labels change, so an order one iteration old is nearly as
// good: measured at configs[3], every second iteration saved the 0.21 ms sort
// on half of them and cost the GEMM < 0.02 ms.
constexpr int kResortEvery = 2;
// Pruned fused iterations rebuild the order once n / kResortChangeDiv labels
// have changed since the last rebuild.
constexpr int64_t kResortChangeDiv = 32;
// Pruned iterations from the (kSecondBoundFrom + 1)-th on have their GEMM record
// the second-nearest bounds: in the first ones the centroids still move too far
// for those bounds to prove a row (measured at configs[3]: no effect on the
// third and fourth iterations), and the record costs the GEMM ~10%.
constexpr int kSecondBoundFrom = 2;
// A pruned iteration with more than n / kFreshUpdateDiv label changes
// accumulates every point afresh (one streaming pass) instead of moving the
// changed rows (two FP64 reductions per feature and change): measured at
// configs[4], 20 ms of incremental update against 8 ms for the fresh pass.
constexpr int64_t kFreshUpdateDiv = 8;
// Full centroid-pair bound computations: the first kPairsFullFirst pruned
// iterations, then every kPairsFullEvery-th (drift updates in between).
constexpr int kPairsFullFirst = 3;
constexpr int kPairsFullEvery = 4;
// Drift updates only below this many rows per centroid: measured at configs[3]
// (K = 2048), the looser bounds cost the GEMM ~1.6% of its time against a
// ~22 us saving per iteration, a gain below ~4M rows on one GPU.
constexpr int64_t kPairsDriftRowsPerCentroid = 2048;

// Pinned host copies of the loop state words (one slot per iteration in flight)
// and the events that say when each copy has landed.  Leased per call from a
// per-device pool (MirrorLease) and kept until exit.
struct LoopMirror {
    int* host = nullptr;
    int* dev = nullptr;  // the same slots as the device sees them (host-mapped)
    cudaEvent_t ev[kLookahead + 1] = {};
    ~LoopMirror() {
        // an error return can leave copies into `host` in flight
        for (cudaEvent_t e : ev)
            if (e) cudaEventSynchronize(e);
        for (cudaEvent_t e : ev)
            if (e) cudaEventDestroy(e);
        if (host) cudaFreeHost(host);
    }
    int init() {
        MXK_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&host), sizeof(int) * 4 * (kLookahead + 1),
                               cudaHostAllocMapped));
        MXK_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&dev), host, 0));
        for (cudaEvent_t& e : ev) MXK_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        return MXK_OK;
    }
};

// Pinned memory and events are allocated once per device and reused by later
// calls: allocating them takes driver locks that another process (an NVML
// client such as nvidia-smi) can hold for tens of milliseconds, longer than the
// iterations enqueued ahead cover, so a per-call allocation could leave the GPU
// idle.
std::mutex g_mirror_mutex;
std::vector<LoopMirror*> g_mirror_pool[64];

struct MirrorLease {
    LoopMirror* m = nullptr;
    int device = -1;
    cudaStream_t stream = nullptr;
    int acquire(cudaStream_t s) {
        stream = s;
        MXK_CUDA(cudaGetDevice(&device));
        if (device < 0 || device >= 64) return fail(MXK_ERR_CUDA, "kmeans_mixed: device ordinal out of range");
        {
            std::lock_guard<std::mutex> lock(g_mirror_mutex);
            if (!g_mirror_pool[device].empty()) {
                m = g_mirror_pool[device].back();
                g_mirror_pool[device].pop_back();
                return MXK_OK;
            }
        }
        auto* fresh = new LoopMirror;
        const int st = fresh->init();
        if (st != MXK_OK) {
            delete fresh;
            return st;
        }
        m = fresh;
        return MXK_OK;
    }
    ~MirrorLease() {
        if (!m) return;
        // After an error return, copies from and into the slots can still be in
        // flight on the stream; the next call must not reuse the slots before.
        if (cudaStreamSynchronize(stream) != cudaSuccess) {
            cudaGetLastError();
            for (cudaEvent_t e : m->ev)
                if (e) cudaEventSynchronize(e);
        }
        std::lock_guard<std::mutex> lock(g_mirror_mutex);
        g_mirror_pool[device].push_back(m);
    }
    LoopMirror* operator->() const { return m; }
};

// Host-to-device copy of the points in row chunks on a side stream, an event
// after each, so that work on the first chunks can start while the rest is
// in flight.  The side stream first waits for the compute stream's prior work
// (the destination may have just been allocated on it).  Destruction waits for
// the copies.
struct ChunkedUpload {
    cudaStream_t side = nullptr;
    cudaEvent_t ready = nullptr;  // the compute stream's prior work
    std::vector<cudaEvent_t> ev;  // chunk c has landed
    std::vector<int64_t> start;   // chunk c is rows [start[c], start[c + 1])
    ~ChunkedUpload() {
        for (cudaEvent_t e : ev) {
            cudaEventSynchronize(e);
            cudaEventDestroy(e);
        }
        if (ready) cudaEventDestroy(ready);
        if (side) {
            cudaStreamSynchronize(side);
            cudaStreamDestroy(side);
        }
    }
    int begin(float* dst, const float* src, int64_t n, int d, cudaStream_t compute) {
        const int64_t chunk = std::max<int64_t>(kPointTileRows, (kUploadChunkBytes / (4 * (int64_t)d)) /
                                                                    kPointTileRows * kPointTileRows);
        for (int64_t r = 0; r < n; r += chunk) start.push_back(r);
        start.push_back(n);
        MXK_CUDA(cudaStreamCreateWithFlags(&side, cudaStreamNonBlocking));
        MXK_CUDA(cudaEventCreateWithFlags(&ready, cudaEventDisableTiming));
        MXK_CUDA(cudaEventRecord(ready, compute));
        MXK_CUDA(cudaStreamWaitEvent(side, ready, 0));
        for (size_t c = 0; c + 1 < start.size(); ++c) {
            cudaEvent_t e = nullptr;
            MXK_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
            ev.push_back(e);
            const int64_t r0 = start[c], rows = start[c + 1] - r0;
            MXK_CUDA(cudaMemcpyAsync(dst + r0 * d, src + r0 * d, sizeof(float) * (size_t)(rows * d),
                                     cudaMemcpyHostToDevice, side));
            MXK_CUDA(cudaEventRecord(e, side));
        }
        return MXK_OK;
    }
    size_t chunks() const { return ev.size(); }
};

int run_lloyd(Comm* comm, int64_t n, int d, int k, const float* points, float* centroids, int* labels,
              const mxk_options* options, int* iterations, cudaStream_t stream, bool cache_points = false,
              const float* host_points = nullptr) {
    MXK_REQUIRE(options && iterations, "kmeans_mixed: null options or iterations");
    PhaseRange call_range("kmeans_mixed");
    MXK_REQUIRE(k > 0 && d > 0 && n >= 0, "kmeans_mixed: require n >= 0, d > 0, k > 0");
    MXK_REQUIRE(d % 128 == 0, "kmeans_mixed: d must be padded to a multiple of 128");
    MXK_REQUIRE(points || n == 0, "kmeans_mixed: null points");
    MXK_REQUIRE(centroids && (labels || n == 0), "kmeans_mixed: null centroids or labels");
    MXK_REQUIRE(options->max_iterations > 0 && options->fp32_iterations >= 0 && options->tolerance >= 0.0f,
                "Require maxiter > 0, fp32-iters >= 0, and tol >= 0");
    clear_error();
    *iterations = 0;
    const int64_t kd = (int64_t)k * d;
    Arena ws(stream);
    float *pnorm = nullptr, *upper = nullptr, *gaps = nullptr, *cnorm = nullptr, *cerr = nullptr, *stats = nullptr,
          *prev = nullptr, *shift = nullptr;
    int *precision = nullptr, *ids = nullptr, *gcount = nullptr, *cscratch = nullptr, *counts = nullptr;
    uint8_t *qpoints = nullptr, *pscales = nullptr, *qcent = nullptr, *cscales = nullptr;
    // With the forced-MXFP8 policy the precision inputs and groups are not
    // needed (see kSelectPrecisionIsForcedMxfp8); the general path keeps them
    // and runs when mxk_set_precision_policy selects the candidate rule.
    const int policy = g_precision_policy.load();
    const bool forced8 = kSelectPrecisionIsForcedMxfp8 && policy == 0;
    int device = 0;
    MXK_CUDA(cudaGetDevice(&device));
    const TraceRequest trace = take_trace(device);
    MXK_REQUIRE(n < (1ll << 31), "kmeans_mixed: n must be below 2^31");
    MXK_CHECK(ws.alloc(&pnorm, n));
    MXK_CHECK(ws.alloc(&gaps, n));
    if (!forced8) {
        MXK_CHECK(ws.alloc(&upper, ((n + 31) / 32) * 96));
        MXK_CHECK(ws.alloc(&precision, n));
        MXK_CHECK(ws.alloc(&ids, 3 * n));
        MXK_CHECK(ws.alloc(&gcount, 4));
        MXK_CHECK(ws.alloc(&cscratch, compaction_scratch_ints(n)));
    }
    int *order = nullptr, *sort_scratch = nullptr, *sort_ctl = nullptr;
    MXK_CHECK(ws.alloc(&order, n));
    MXK_CHECK(ws.alloc(&sort_scratch, label_sort_scratch_ints(k)));
    MXK_CHECK(ws.alloc(&sort_ctl, 2));
    MXK_CUDA(cudaMemsetAsync(sort_ctl, 0, sizeof(int) * 2, stream));
    // Opt-in point cache: under the forced-MXFP8 policy the points' MXFP8 bytes
    // never change, so they are quantized once per call and only regathered
    // when the visiting order changes (the reference re-quantizes every
    // iteration; the results are the same).
    const bool cache = cache_points && forced8;
    uint8_t *qnat = nullptr, *snat = nullptr;
    if (cache) {
        MXK_CHECK(ws.alloc(&qnat, n * d));
        MXK_CHECK(ws.alloc(&snat, n * d / 32));
    }
    // (the fused quantize at d = 128 never materializes the MXFP8 point rows)
    const bool need_qpoints = !forced8 || d != 128 || cache;
    if (need_qpoints) {
        MXK_CHECK(ws.alloc(&qpoints, n * d));
        MXK_CHECK(ws.alloc(&pscales, scale_atom_bytes(n, d)));
    }
    MXK_CHECK(ws.alloc(&cnorm, k));
    if (!forced8) {
        MXK_CHECK(ws.alloc(&cerr, k));
        MXK_CHECK(ws.alloc(&stats, 2));
    }
    MXK_CHECK(ws.alloc(&qcent, kd));
    MXK_CHECK(ws.alloc(&cscales, scale_atom_bytes(k, d, kCentroidTileRows)));
    // scale atoms of padding rows are never written; keep them finite
    if (need_qpoints) MXK_CUDA(cudaMemsetAsync(pscales, 0, (size_t)scale_atom_bytes(n, d), stream));
    MXK_CUDA(cudaMemsetAsync(cscales, 0, (size_t)scale_atom_bytes(k, d, kCentroidTileRows), stream));
    MXK_CHECK(ws.alloc(&prev, kd));
    // This iteration's cluster sums in FP64 (every point, or the moved rows'
    // deltas), and the running sums and counts kept across iterations: a pruned
    // iteration's GEMM records the points whose label changed and the update
    // moves only those rows (the reference re-adds every point each iteration
    // in FP32; FP64 keeps the running sums of clusters that lose most of their
    // points clear of cancellation, so both round to the same FP32 sums up to
    // the reference's own summation error).
    double* sums = nullptr;
    MXK_CHECK(ws.alloc(&sums, kd));
    MXK_CHECK(ws.alloc(&counts, k));
    MXK_CUDA(cudaMemsetAsync(sums, 0, sizeof(double) * kd, stream));
    MXK_CUDA(cudaMemsetAsync(counts, 0, sizeof(int) * k, stream));
    double* acc_sums = nullptr;
    int *acc_counts = nullptr, *chg_count = nullptr, *upd_gate = nullptr;
    int4* chg = nullptr;
    MXK_CHECK(ws.alloc(&acc_sums, kd));
    MXK_CHECK(ws.alloc(&acc_counts, k));
    MXK_CHECK(ws.alloc(&shift, shift_scratch_floats()));
    MXK_CUDA(cudaMemsetAsync(shift, 0, sizeof(float) * shift_scratch_floats(), stream));  // (the finalize ticket)
    // Exact pruning of centroid tiles (prune.cu) from the previous iteration's
    // labels and distances: forced-MXFP8 path, at most 64 centroid tiles.
    const bool prune = forced8 && n > 0 && prune_supported(k, d);
    const int ctiles = (k + kCentroidTileRows - 1) / kCentroidTileRows;
    float *dmin = nullptr, *cdelta = nullptr, *chat = nullptr, *bmax32 = nullptr;
    // per row of the visiting order (RowState: moved along when the order is
    // rebuilt): (distance from the last GEMM, its bound on every other
    // centroid's distance, alpha, |x^|), written from the first pruned
    // iteration on, and the row's label
    float4* pinfo = nullptr;
    RowState rows_state;
    // per-centroid stats [2][k] and per-tile stats [2][2][ctiles], by iteration parity
    float4 *cstats = nullptr, *tstats = nullptr;
    uint64_t* tmask = nullptr;
    float4* rbound = nullptr;  // per row in visiting order: (distance bound, previous label, excluded tiles' bound)
    if (prune) {
        MXK_CHECK(ws.alloc(&pinfo, n));
        MXK_CHECK(ws.alloc(&rows_state.label, n));
        MXK_CHECK(ws.alloc(&rows_state.tmp_state, n));
        MXK_CHECK(ws.alloc(&rows_state.tmp_label, n));
        MXK_CHECK(ws.alloc(&rows_state.tmp_order, n));
        rows_state.state = pinfo;
        MXK_CHECK(ws.alloc(&chat, kd));
        MXK_CHECK(ws.alloc(&dmin, (int64_t)k * ctiles));
        MXK_CHECK(ws.alloc(&cdelta, k));
        MXK_CHECK(ws.alloc(&cstats, 2 * (int64_t)k));
        MXK_CHECK(ws.alloc(&tstats, 4 * (int64_t)ctiles));
        MXK_CHECK(ws.alloc(&bmax32, (k + 31) / 32));
        MXK_CHECK(ws.alloc(&tmask, (n + kPointTileRows - 1) / kPointTileRows));
        MXK_CHECK(ws.alloc(&rbound, n));
        MXK_CHECK(ws.alloc(&chg, n));
        MXK_CHECK(ws.alloc(&chg_count, 1));
        MXK_CHECK(ws.alloc(&upd_gate, 3));
        MXK_CUDA(cudaMemsetAsync(chg_count, 0, sizeof(int), stream));
    }
    // Row compaction in pruned iterations (not with the point cache, whose GEMM
    // reads contiguous pre-gathered point tiles): rows whose label the bounds
    // prove leave the GEMM.
    const bool compact = prune && !cache;
    WorkRows work;
    if (compact) {
        const int64_t row_tiles = (n + kPointTileRows - 1) / kPointTileRows;
        MXK_CHECK(ws.alloc(&work.pid, n));
        MXK_CHECK(ws.alloc(&work.rb, n));
        MXK_CHECK(ws.alloc(&work.cmask, row_tiles));
        MXK_CHECK(ws.alloc(&work.need_bits, row_tiles));
        MXK_CHECK(ws.alloc(&work.counts, row_tiles));
        MXK_CHECK(ws.alloc(&work.offsets, row_tiles));
        MXK_CHECK(ws.alloc(&work.seg_total, row_tiles / 1024 + 1));
        MXK_CHECK(ws.alloc(&work.rows, 1));
    }
    int* loop = nullptr;  // [0] stopped, [1] completed iterations, [2] non-finite shift, [3] rows (0 once stopped)
    MXK_CHECK(ws.alloc(&loop, 4));
    MirrorLease mirror;
    MXK_CHECK(mirror.acquire(stream));
    mirror->host[0] = mirror->host[1] = mirror->host[2] = 0;
    mirror->host[3] = (int)n;
    // (slot 0 is next written by iteration 0's state copy, after this one in stream order)
    MXK_CUDA(cudaMemcpyAsync(loop, mirror->host, sizeof(int) * 4, cudaMemcpyHostToDevice, stream));
    float* dots = nullptr;
    int64_t chunk_rows = 0;
    if (options->fp32_iterations > 0 && n > 0) {
        chunk_rows = std::max<int64_t>(128, kFp32ChunkBytes / (4 * (int64_t)k));
        if (chunk_rows > n) chunk_rows = n;
        MXK_CHECK(ws.alloc(&dots, chunk_rows * k));
    }

    // Host points (`points` is then the device buffer they go to): on the fused
    // MX path the first iteration works chunk by chunk as the rows land (their
    // norms, assignment and accumulation), overlapping the rest of the copy;
    // otherwise one copy first.
    const bool upload = host_points != nullptr && n > 0;
    const bool overlap = upload && prune && !cache && d == 128 && options->fp32_iterations == 0;
    ChunkedUpload up;
    if (overlap)
        MXK_CHECK(up.begin(const_cast<float*>(points), host_points, n, d, stream));
    else if (upload)
        MXK_CUDA(cudaMemcpyAsync(const_cast<float*>(points), host_points, sizeof(float) * (size_t)(n * d),
                                 cudaMemcpyHostToDevice, stream));

    // Once per run (kmeans.cu:24-27); with the chunked upload, per chunk below.
    if (!overlap) MXK_CHECK(launch_l2_norm(n, d, points, pnorm, stream));
    // (with pruning the sort reorders the visiting order, first the points' own;
    // the first pruned iteration writes the rows' pruning records)
    if (prune) MXK_CHECK(launch_identity_order(n, order, stream));
    if (cache) MXK_CHECK(launch_quantize(8, n, d, points, nullptr, qnat, snat, nullptr, nullptr, stream, 0));
    if (!forced8) MXK_CHECK(launch_point_bounds(n, d, points, pnorm, upper, stream));
    if (n) MXK_CUDA(cudaMemsetAsync(gaps, 0, sizeof(float) * n, stream));

    const bool sharded = comm && comm->nranks > 1;
    if (sharded && !nccl().ok) return fail(MXK_ERR_COMM, "NCCL (libnccl.so.2) could not be loaded");
    if (sharded && !comm->comm)
        return fail(MXK_ERR_COMM, "kmeans_mixed_sharded: the communicator was aborted; destroy and re-create it");
    const int inject_at = sharded && comm->rank == g_inject_rank.load() ? g_inject_iteration.load() : -1;
    bool cached_stale = true;  // the gathered copy of the cached rows does not follow the current order
    int pruned_its = 0;        // pruned iterations enqueued so far
    for (int it = 0; it < options->max_iterations; ++it) {
        if (it == inject_at) {
            // the injected failure: drain what this rank has enqueued (its peers
            // take part in those collectives), then leave between steps
            MXK_CUDA(cudaEventRecord(mirror->ev[kLookahead], stream));
            MXK_CHECK(wait_event(comm, mirror->ev[kLookahead]));
            return fail(MXK_ERR_CUDA, "injected rank failure (mxk_inject_rank_failure) at iteration " +
                                          std::to_string(it));
        }
        PhaseRange iteration_range("lloyd_iteration");
        // From the second iteration on, visit points grouped by their label of
        // the previous (or, every other iteration, the one before) iteration
        // (order.cu, rebuilt below after the assignment); the first iteration
        // keeps ascending point order.
        const int* ord = it > 0 && n > 0 ? order : nullptr;
        // Pruning needs the previous iteration's labels and distances from the
        // MX GEMM (not an FP32 iteration) and, in prev, the centroids it used.
        const bool prune_it = prune && it >= 1 && it - 1 >= options->fp32_iterations;
        float4* cst = cstats + (int64_t)(it & 1) * k;
        const float4* cst_old = cstats + (int64_t)((it + 1) & 1) * k;
        float4* tst = tstats + (int64_t)(it & 1) * 2 * ctiles;
        const float4* tst_old = tstats + (int64_t)((it + 1) & 1) * 2 * ctiles;
        // MX iterations with pruning: the centroid norms, the centroids' MXFP8
        // codes and scales and their pruning stats (this iteration's, the next
        // one's old ones) in one pass; otherwise the norms alone here.
        const bool prep = prune && it >= options->fp32_iterations;
        if (prep)
            MXK_CHECK(launch_centroid_prep(k, d, centroids, prune_it ? prev : nullptr, cnorm, chat, cst, cdelta, qcent,
                                           cscales, loop, stream));
        else
            MXK_CHECK(launch_l2_norm(k, d, centroids, cnorm, stream));
        if (prune_it) {
            // The centroid-pair bounds are computed in full (an FP32 Gram pass,
            // K^2 D).  With few rows per centroid (a shard of a multi-GPU run)
            // that pass weighs more than the slightly looser bounds cost the
            // GEMM, so there it runs only in the first pruned iterations, while
            // the centroids move most, and every kPairsFullEvery-th after; in
            // between the bounds are lowered by the centroids' movement bounds
            // (K x tiles work).  Either way the labels are exact.
            const bool drift_ok = n < (int64_t)k * kPairsDriftRowsPerCentroid;
            if (!drift_ok || pruned_its < kPairsFullFirst || pruned_its % kPairsFullEvery == 0)
                MXK_CHECK(launch_centroid_pairs(k, d, chat, cst, cdelta, dmin, tst, bmax32, loop, stream));
            else
                MXK_CHECK(launch_centroid_pairs_drift(k, d, cdelta, cst, dmin, tst, bmax32, loop, stream));
            // The second-nearest bounds in pinfo are used when the previous
            // iteration's GEMM recorded them (its tile stats, tst_old, describe
            // the centroids it used).
            const bool second_in = pruned_its > kSecondBoundFrom;
            // In the first pruned iteration the centroids have just moved far
            // from their initial rows (up to 30 at configs[3]), so the moved
            // bound sqrt(d_prev) + delta proves little; one pass over the points
            // gives every row its distance bound to its current centroid.
            const bool fresh = pruned_its == 0;
            if (fresh)
                MXK_CHECK(launch_row_distance_bound(n, k, d, ord, rows_state.label, pinfo, chat, cst, points, loop,
                                                    stream));
            MXK_CHECK(launch_tile_mask(n, k, d, ord, rows_state.label, pinfo, cst, cst_old, tst,
                                       second_in ? tst_old : nullptr, cdelta, dmin, tmask, rbound, loop, stream,
                                       compact ? &work : nullptr, fresh));
            ++pruned_its;
        }
        const bool traced = it < trace.max_iterations;
        if (traced && trace.centroids)
            MXK_CUDA(cudaMemcpyAsync(trace.centroids + (int64_t)it * kd, centroids, sizeof(float) * kd,
                                     cudaMemcpyDeviceToDevice, stream));
        if (traced && trace.group_sizes)  // FP32 iterations record no MX groups
            MXK_CUDA(cudaMemsetAsync(trace.group_sizes + 3 * it, 0, sizeof(int) * 3, stream));
        if (it < options->fp32_iterations) {
            // kmeans.cu:31-34: FP32 product, assignment without pid (gap init -1).
            for (int64_t r0 = 0; r0 < n; r0 += chunk_rows) {
                const int64_t rows = std::min<int64_t>(chunk_rows, n - r0);
                MXK_CHECK(launch_gemm_fp32(rows, k, d, points + r0 * d, centroids, dots, stream));
                MXK_CHECK(launch_assign_clusters(rows, k, pnorm + r0, cnorm, dots, nullptr, labels + r0, gaps + r0,
                                                 stream));
            }
            if (options->verbose && (!comm || comm->rank == 0))
                std::fprintf(stderr, "iteration=%d precision=FP32\n", it + 1);
        } else if (forced8) {
            // Every point is in the MXFP8 group, in the visiting sequence `ord`;
            // the group's row count is loop[3] (n, or 0 once the loop stopped).
            // In compacted iterations the quantize and GEMM take only the rows
            // whose labels the bounds left open (work.pid, count work.rows).
            const bool compacted = compact && prune_it;
            const int* gemm_pid = compacted ? work.pid : ord;
            const int* gemm_rows = compacted ? work.rows : loop + 3;
            if (!prep)  // (else the centroid pass above wrote the MXFP8 centroids)
                MXK_CHECK(launch_quantize(8, k, d, centroids, nullptr, qcent, cscales, nullptr, nullptr, stream,
                                          kCentroidTileRows, "quantize_centroids"));
            // MXFP8 at d = 128: the GEMM quantizes the point tiles itself from the
            // FP32 rows (same bytes as quantize_rows), so this pass disappears.
            const bool fused_q = d == 128 && !cache;
            if (cache) {
                // regather the cached rows when the visiting order has changed
                if (cached_stale)
                    MXK_CHECK(launch_gather_mxfp8_rows(n, d, qnat, snat, ord, qpoints, pscales, loop, stream));
                cached_stale = false;
            } else if (!fused_q) {
                MXK_CHECK(launch_quantize(8, n, d, points, gemm_pid, qpoints, pscales, nullptr, gemm_rows, stream,
                                          kPointTileRows, "quantize_points"));
            }
            MxArgmin am;
            am.point_norms = pnorm;
            am.centroid_norms = cnorm;
            am.pid = gemm_pid;
            am.labels = labels;
            am.gaps = nullptr;
            am.start_hint = it > 0 ? labels : nullptr;  // previous iteration's labels
            am.tile_mask = prune_it ? (compacted ? reinterpret_cast<const uint64_t*>(work.cmask) : tmask) : nullptr;
            am.row_bound = prune_it ? (compacted ? work.rb : rbound) : nullptr;
            am.changes = prune_it ? chg : nullptr;
            am.change_count = prune_it ? chg_count : nullptr;
            am.best_dist = prune_it ? reinterpret_cast<float*>(pinfo) : nullptr;
            am.best_dist_stride = 4;
            am.by_row = prune;  // (the rows' state follows the visiting order)
            am.row_labels = prune ? rows_state.label : nullptr;
            // (pinfo's second slot; pruned_its counts this iteration already)
            am.second_bound = prune_it && pruned_its > kSecondBoundFrom;
            am.beta_max32 = bmax32;
            if (overlap && it == 0) {
                // each chunk as it lands: norms, assignment (points in their own
                // order, no previous labels), fresh accumulation
                for (size_t c = 0; c < up.chunks(); ++c) {
                    const int64_t r0 = up.start[c], rows = up.start[c + 1] - r0;
                    MXK_CUDA(cudaStreamWaitEvent(stream, up.ev[c], 0));
                    MXK_CHECK(launch_l2_norm(rows, d, points + r0 * d, pnorm + r0, stream));
                    MxArgmin ac = am;
                    ac.point_norms = pnorm + r0;
                    ac.labels = labels + r0;
                    ac.row_labels = am.row_labels ? am.row_labels + r0 : nullptr;
                    MXK_CHECK(launch_gemm_mx(8, rows, k, d, nullptr, nullptr, qcent, cscales, nullptr, &ac, nullptr,
                                             stream, true, points + r0 * d, rows));
                    MXK_CHECK(launch_accumulate(rows, d, k, points + r0 * d, labels + r0, nullptr, sums, counts,
                                                stream, loop));
                }
            } else {
                MXK_CHECK(launch_gemm_mx(8, n, k, d, qpoints, pscales, qcent, cscales, nullptr, &am, gemm_rows,
                                         stream, true, fused_q ? points : nullptr, n));
            }
            if (traced && trace.group_sizes)  // (0, 0, rows of the MXFP8 group)
                MXK_CUDA(cudaMemcpyAsync(trace.group_sizes + 3 * it + 2, loop + 3, sizeof(int),
                                         cudaMemcpyDeviceToDevice, stream));
            if (options->verbose && (!comm || comm->rank == 0))
                std::fprintf(stderr, "iteration=%d fp4=0 fp6=0 fp8=%lld\n", it + 1, (long long)n);
        } else {
            MXK_CUDA(cudaMemsetAsync(cerr, 0, sizeof(float) * k, stream));
            MXK_CHECK(launch_quantize(8, k, d, centroids, nullptr, qcent, cscales, cerr, nullptr, stream,
                                      kCentroidTileRows, "quantize_centroids"));
            MXK_CHECK(launch_centroid_stats(k, cerr, cnorm, stats, stream));
            MXK_CHECK(launch_assign_precisions(n, d, upper, gaps, 0.0f, 0.0f, stats, precision, nullptr, stream,
                                               policy));
            MXK_CHECK(launch_group_compaction(n, precision, ord, ids, gcount, cscratch, stream, loop));
            static const int group_bits[3] = {4, 6, 8};
            for (int g = 0; g < 3; ++g) {
                // MXFP8 at d = 128: the GEMM quantizes the point tiles itself from the
                // FP32 rows (same bytes as quantize_rows), so this pass disappears.
                const bool fused_q = group_bits[g] == 8 && d == 128;
                if (!fused_q)
                    MXK_CHECK(launch_quantize(group_bits[g], n, d, points, ids + g * n, qpoints, pscales, nullptr,
                                              gcount + g, stream, kPointTileRows, "quantize_points"));
                MxArgmin am;
                am.point_norms = pnorm;
                am.centroid_norms = cnorm;
                am.pid = ids + g * n;
                am.labels = labels;
                // the candidate rule reads each point's two-largest gap of the last
                // MX iteration (assignment.cu:53-55); the reference's rule ignores it
                am.gaps = policy ? gaps : nullptr;
                am.start_hint = it > 0 ? labels : nullptr;  // previous iteration's labels
                MXK_CHECK(launch_gemm_mx(group_bits[g], n, k, d, qpoints, pscales, qcent, cscales, nullptr, &am,
                                         gcount + g, stream, true, fused_q ? points : nullptr, n));
            }
            if (traced && trace.group_sizes)
                MXK_CUDA(cudaMemcpyAsync(trace.group_sizes + 3 * it, gcount, sizeof(int) * 3, cudaMemcpyDeviceToDevice,
                                         stream));
            if (options->verbose && (!comm || comm->rank == 0)) {
                // pinned slot of this iteration, read after the event (the
                // watchdog's guarded wait in a sharded run)
                const int vslot = it % (kLookahead + 1);
                int* h = mirror->host + 4 * vslot;
                MXK_CUDA(cudaMemcpyAsync(h, gcount, sizeof(int) * 3, cudaMemcpyDeviceToHost, stream));
                MXK_CUDA(cudaEventRecord(mirror->ev[vslot], stream));
                MXK_CHECK(wait_event(comm, mirror->ev[vslot]));
                std::fprintf(stderr, "iteration=%d fp4=%d fp6=%d fp8=%d\n", it + 1, h[0], h[1], h[2]);
            }
        }
        if (traced && trace.labels)
            MXK_CUDA(cudaMemcpyAsync(trace.labels + (int64_t)it * n, labels, sizeof(int) * n, cudaMemcpyDeviceToDevice,
                                     stream));
        // A pruned MX iteration (forced MXFP8: its GEMM recorded the label
        // changes) adds only the moved rows to the running sums; any other
        // iteration accumulates every point afresh.
        const bool incremental = prune_it && forced8;
        // The points are sorted by the labels just assigned: the next iteration
        // visits them in that order, and a fresh accumulation below sees one
        // run per cluster.  Every kResortEvery-th iteration, or, in pruned
        // iterations of the fused path (which record their label changes), once
        // at least n / kResortChangeDiv labels have changed since the last sort
        // (decided on the device; the order stays a valid permutation either
        // way).  The last iteration of an incremental run needs no new order.
        // (With pruning the rows' state follows the order, and the FP32
        // iterations, which write no row labels, keep the point order.)
        const bool gated = incremental && !cache;
        const bool may_sort = !(prune && it < options->fp32_iterations);
        if (n > 0 && may_sort &&
            (gated ? it + 1 < options->max_iterations
                   : it % kResortEvery == 0 && (!incremental || it + 1 < options->max_iterations))) {
            if (gated)
                MXK_CHECK(launch_sort_gate(loop, chg_count, sort_ctl,
                                           (int)std::max<int64_t>(1, n / kResortChangeDiv), stream));
            // (the records exist from the first pruned iteration on)
            RowState rs = rows_state;
            if (pruned_its == 0) rs.state = nullptr;
            MXK_CHECK(launch_label_sort(n, k, labels, order, sort_scratch, stream, gated ? sort_ctl + 1 : loop,
                                        prune ? &rs : nullptr));
            cached_stale = true;
            ord = order;
        }
        // kmeans.cu:62-65 (sums and counts are zero: set before the loop, and
        // left zero by every finalize).  An incremental iteration of a
        // single-GPU run whose labels changed for more than n / kFreshUpdateDiv
        // rows accumulates every point afresh instead, decided on the device
        // (a sharded run keeps the incremental update: its ranks must agree).
        const bool switchable = incremental && !sharded;
        if (switchable)
            MXK_CHECK(launch_update_gate(loop, chg_count, (int)std::max<int64_t>(1, n / kFreshUpdateDiv), upd_gate,
                                         stream));
        if (incremental)
            MXK_CHECK(launch_accumulate_changes(d, k, points, chg, chg_count, sums, counts, stream,
                                                switchable ? upd_gate : loop));
        if ((!incremental || switchable) && !(overlap && it == 0))  // (accumulated per chunk above)
            MXK_CHECK(launch_accumulate(n, d, k, points, labels, ord, sums, counts, stream,
                                        switchable ? upd_gate + 1 : loop, switchable));
        if (sharded) {
            NcclApi& api = nccl();
            ncclResult_t r = api.GroupStart();
            if (r == ncclSuccess) r = api.AllReduce(sums, sums, (size_t)kd, ncclFloat64, ncclSum, comm->comm, stream);
            if (r == ncclSuccess) r = api.AllReduce(counts, counts, (size_t)k, ncclInt32, ncclSum, comm->comm, stream);
            ncclResult_t r2 = api.GroupEnd();
            if (r != ncclSuccess) return fail_nccl("ncclAllReduce", r);
            if (r2 != ncclSuccess) return fail_nccl("ncclGroupEnd", r2);
        }
        // The centroids are updated in place; the finalize kernel also keeps the
        // old ones in prev (the next iteration's pruning bounds and, there, the
        // previous centroids of update.cu:26-29), zeroes sums and counts, and
        // writes the loop state into this iteration's pinned host slot.
        const int slot = it % (kLookahead + 1);
        MXK_CHECK(launch_finalize(d, k, sums, counts, centroids, centroids, shift, stream, loop, options->tolerance,
                                  prev, true, mirror->dev + 4 * slot, acc_sums, acc_counts, !incremental,
                                  incremental ? chg_count : nullptr, switchable ? upd_gate + 2 : nullptr));
        MXK_CUDA(cudaEventRecord(mirror->ev[slot], stream));
        // Read the state of iteration it - lookahead.  FP32 iterations (whose
        // kernels do not consult the stop word) and verbose runs are read at once,
        // so no FP32 iteration is ever enqueued after the loop has stopped.
        const int lookahead = (options->verbose || it + 1 < options->fp32_iterations) ? 0 : kLookahead;
        const int seen = it - lookahead;
        if (seen >= 0) {
            const int sslot = seen % (kLookahead + 1);
            MXK_CHECK(wait_event(comm, mirror->ev[sslot]));
            if (mirror->host[4 * sslot]) break;  // stopped at or before iteration `seen`
        }
    }
    MXK_CUDA(cudaMemcpyAsync(mirror->host, loop, sizeof(int) * 4, cudaMemcpyDeviceToHost, stream));
    if (polled_waits(comm)) {  // the last iterations' collectives, under the watchdog
        MXK_CUDA(cudaEventRecord(mirror->ev[0], stream));
        MXK_CHECK(wait_event(comm, mirror->ev[0]));
    }
    MXK_CUDA(cudaStreamSynchronize(stream));
    MXK_CHECK(check_device_error(stream));
    if (mirror->host[2]) return fail(MXK_ERR_NONFINITE, "Non-finite centroid shift; check the input scale");
    *iterations = mirror->host[1];
    return MXK_OK;
}

}  // namespace

// For mxk_kmeans_mixed_multi (multi.cpp): kmeans_mixed (comm null) or
// kmeans_mixed_sharded over points copied from the host into dev_points within
// the call, the copy overlapping the first iteration where the path allows.
int kmeans_mixed_from_host(void* comm, int64_t n, int d, int k, const float* host_points, float* dev_points,
                           float* centroids, int* labels, const mxk_options* options, int* iterations,
                           cudaStream_t stream) {
    Comm* c = static_cast<Comm*>(comm);
    MXK_REQUIRE(host_points || n == 0, "kmeans_mixed_multi: null points");
    return run_lloyd(c, n, d, k, dev_points, centroids, labels, options, iterations, stream, false, host_points);
}

// For mxk_kmeans_mixed_multi (multi.cpp): the shared failure flag of its
// in-process ranks, and the abort of a failed rank's communicator (frees it).
void comm_attach_group_flag(void* comm, std::atomic<int>* flag) {
    if (comm) static_cast<Comm*>(comm)->group_failed = flag;
}

void comm_abort(void* comm) {
    auto* c = static_cast<Comm*>(comm);
    if (!c) return;
    if (c->comm && nccl().CommAbort) nccl().CommAbort(c->comm);
    c->comm = nullptr;
}

}  // namespace mxk

extern "C" {

int mxk_kmeans_mixed(int64_t n, int d, int k, const float* points, float* centroids, int* labels,
                     const mxk_options* options, int* iterations, void* stream) {
    return mxk::run_lloyd(nullptr, n, d, k, points, centroids, labels, options, iterations, mxk::as_stream(stream));
}

int mxk_kmeans_mixed_cached(int64_t n, int d, int k, const float* points, float* centroids, int* labels,
                            const mxk_options* options, int* iterations, void* stream) {
    return mxk::run_lloyd(nullptr, n, d, k, points, centroids, labels, options, iterations, mxk::as_stream(stream),
                          true);
}

int mxk_set_precision_policy(int policy) {
    MXK_REQUIRE(policy == 0 || policy == 1, "set_precision_policy: policy must be 0 (reference) or 1 (candidate)");
    mxk::g_precision_policy.store(policy);
    return MXK_OK;
}

int mxk_trace_next_call(const mxk_trace* trace) {
    MXK_REQUIRE(trace != nullptr && trace->max_iterations >= 0, "trace_next_call: bad arguments");
    int device = 0;
    MXK_CUDA(cudaGetDevice(&device));
    MXK_REQUIRE(device >= 0 && device < 64, "trace_next_call: device ordinal out of range");
    mxk::TraceRequest t;
    t.centroids = trace->centroids;
    t.labels = trace->labels;
    t.group_sizes = trace->group_sizes;
    t.max_iterations = trace->max_iterations;
    std::lock_guard<std::mutex> lock(mxk::g_trace_mutex);
    mxk::g_trace[device] = t;
    return MXK_OK;
}

int mxk_comm_unique_id(unsigned char id[128]) {
    mxk::NcclApi& api = mxk::nccl();
    if (!api.ok) return mxk::fail(MXK_ERR_COMM, "NCCL (libnccl.so.2) could not be loaded");
    ncclUniqueId uid;
    ncclResult_t r = api.GetUniqueId(&uid);
    if (r != ncclSuccess) return mxk::fail_nccl("ncclGetUniqueId", r);
    static_assert(sizeof(uid.internal) == 128, "unexpected ncclUniqueId size");
    std::memcpy(id, uid.internal, 128);
    return MXK_OK;
}

int mxk_comm_init(void** comm, int nranks, int rank, const unsigned char id[128]) {
    MXK_REQUIRE(comm && id && nranks >= 1 && rank >= 0 && rank < nranks, "comm_init: bad arguments");
    mxk::NcclApi& api = mxk::nccl();
    auto* c = new mxk::Comm();
    c->nranks = nranks;
    c->rank = rank;
    if (nranks > 1) {
        if (!api.ok) {
            delete c;
            return mxk::fail(MXK_ERR_COMM, "NCCL (libnccl.so.2) could not be loaded");
        }
        ncclUniqueId uid;
        std::memcpy(uid.internal, id, 128);
        ncclResult_t r = api.CommInitRank(&c->comm, nranks, uid, rank);
        if (r != ncclSuccess) {
            delete c;
            return mxk::fail_nccl("ncclCommInitRank", r);
        }
    }
    *comm = c;
    return MXK_OK;
}

int mxk_inject_rank_failure(int rank, int iteration) {
    mxk::g_inject_rank.store(rank);
    mxk::g_inject_iteration.store(iteration);
    return MXK_OK;
}

int mxk_comm_destroy(void* comm) {
    auto* c = static_cast<mxk::Comm*>(comm);
    if (!c) return MXK_OK;
    int st = MXK_OK;
    if (c->comm) {
        ncclResult_t r = mxk::nccl().CommDestroy(c->comm);
        if (r != ncclSuccess) st = mxk::fail_nccl("ncclCommDestroy", r);
    }
    delete c;
    return st;
}

int mxk_kmeans_mixed_sharded(void* comm, int64_t n_local, int d, int k, const float* points, float* centroids,
                             int* labels, const mxk_options* options, int* iterations, void* stream) {
    MXK_REQUIRE(comm != nullptr, "kmeans_mixed_sharded: null communicator");
    return mxk::run_lloyd(static_cast<mxk::Comm*>(comm), n_local, d, k, points, centroids, labels, options, iterations,
                          mxk::as_stream(stream));
}

}  // extern "C"
