// Host runtime of libmxkmeans: error reporting, launch accounting and kernel
// timing, the per-device error word, and tensor-map encoding.
#include <atomic>
#include <deque>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include <nvtx3/nvToolsExt.h>

#include "common.cuh"

namespace mxk {

namespace {
thread_local std::string g_last_error;
std::atomic<uint64_t> g_launches{0};
std::atomic<int> g_profiling{0};

struct PendingTiming {
    int device;
    const char* name;
    cudaEvent_t start, stop;
};

struct KernelStat {
    int device;
    std::string name;
    uint64_t launches = 0;
    double total_ms = 0.0;
};

std::mutex g_mutex;
std::deque<PendingTiming> g_pending;
std::vector<KernelStat> g_stats;
unsigned* g_error_words[64] = {};
// Timing events of finished launches, per device, reused by later launches:
// creating events can wait on driver locks that another process (an NVML
// client such as nvidia-smi) holds for milliseconds, which would stall the
// enqueueing thread on every launch while profiling.
std::vector<cudaEvent_t> g_event_pool[64];

bool take_events_locked(int device, cudaEvent_t* a, cudaEvent_t* b) {
    auto& pool = g_event_pool[device];
    for (cudaEvent_t* e : {a, b}) {
        if (!pool.empty()) {
            *e = pool.back();
            pool.pop_back();
        } else if (cudaEventCreate(e) != cudaSuccess) {
            cudaGetLastError();
            *e = nullptr;
        }
    }
    if (*a && *b) return true;
    if (*a) pool.push_back(*a);
    if (*b) pool.push_back(*b);
    *a = *b = nullptr;
    return false;
}

// Adds a finished launch's time to the statistics and recycles its events.
void account_locked(const PendingTiming& p) {
    float ms = 0.0f;
    if (cudaEventElapsedTime(&ms, p.start, p.stop) == cudaSuccess) {
        KernelStat* st = nullptr;
        for (auto& s : g_stats)
            if (s.device == p.device && s.name == p.name) st = &s;
        if (!st) {
            g_stats.push_back(KernelStat{p.device, p.name});
            st = &g_stats.back();
        }
        st->launches += 1;
        st->total_ms += ms;
        g_event_pool[p.device].push_back(p.start);
        g_event_pool[p.device].push_back(p.stop);
    } else {
        cudaGetLastError();
        cudaEventDestroy(p.start);
        cudaEventDestroy(p.stop);
    }
}

// Waits for every pending launch and accounts for it.
void drain_pending_locked() {
    for (auto& p : g_pending) {
        if (cudaEventSynchronize(p.stop) != cudaSuccess) cudaGetLastError();
        account_locked(p);
    }
    g_pending.clear();
}

// Accounts for the launches at the front of the queue that have finished
// (without waiting), so a long profiled run keeps reusing a bounded set of events.
void harvest_finished_locked() {
    while (!g_pending.empty()) {
        const cudaError_t e = cudaEventQuery(g_pending.front().stop);
        if (e == cudaErrorNotReady) break;
        if (e != cudaSuccess) cudaGetLastError();
        account_locked(g_pending.front());
        g_pending.pop_front();
    }
}
}  // namespace

int fail(int status, const std::string& message) {
    g_last_error = message;
    return status;
}

int fail_cuda(const char* what, cudaError_t err) {
    g_last_error = std::string(what) + ": " + cudaGetErrorString(err);
    return MXK_ERR_CUDA;
}

void clear_error() { g_last_error.clear(); }

LaunchScope::LaunchScope(const char* n, cudaStream_t s) : name(n), stream(s) {
    nvtxRangePushA(n);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    if (g_profiling.load(std::memory_order_relaxed)) {
        bool ok = cudaGetDevice(&device) == cudaSuccess && device >= 0 && device < 64;
        if (ok) {
            std::lock_guard<std::mutex> lock(g_mutex);
            if (g_event_pool[device].size() < 2) harvest_finished_locked();
            ok = take_events_locked(device, &start, &stop);
        }
        if (ok) cudaEventRecord(start, stream);
    }
}

LaunchScope::~LaunchScope() {
    if (start && stop) {
        cudaEventRecord(stop, stream);
        std::lock_guard<std::mutex> lock(g_mutex);
        g_pending.push_back(PendingTiming{device, name, start, stop});
    }
    nvtxRangePop();
}

PhaseRange::PhaseRange(const char* name) { nvtxRangePushA(name); }
PhaseRange::~PhaseRange() { nvtxRangePop(); }

unsigned* device_error_word() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(g_mutex);
    if (!g_error_words[dev]) {
        void* p = nullptr;
        if (cudaMalloc(&p, sizeof(unsigned)) != cudaSuccess) return nullptr;
        if (cudaMemset(p, 0, sizeof(unsigned)) != cudaSuccess) return nullptr;
        g_error_words[dev] = static_cast<unsigned*>(p);
    }
    return g_error_words[dev];
}

unsigned long long* device_tile_counter() {
    static unsigned long long* counters[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(g_mutex);
    if (!counters[dev]) {
        void* p = nullptr;
        if (cudaMalloc(&p, sizeof(unsigned long long)) != cudaSuccess) return nullptr;
        if (cudaMemset(p, 0, sizeof(unsigned long long)) != cudaSuccess) return nullptr;
        counters[dev] = static_cast<unsigned long long*>(p);
    }
    return counters[dev];
}

unsigned long long* device_row_counter() {
    static unsigned long long* counters[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(g_mutex);
    if (!counters[dev]) {
        void* p = nullptr;
        if (cudaMalloc(&p, sizeof(unsigned long long)) != cudaSuccess) return nullptr;
        if (cudaMemset(p, 0, sizeof(unsigned long long)) != cudaSuccess) return nullptr;
        counters[dev] = static_cast<unsigned long long*>(p);
    }
    return counters[dev];
}

int check_device_error(cudaStream_t stream) {
    unsigned* w = device_error_word();
    if (!w) return fail(MXK_ERR_CUDA, "cannot allocate the device error word");
    unsigned host = 0;
    MXK_CUDA(cudaMemcpyAsync(&host, w, sizeof(unsigned), cudaMemcpyDeviceToHost, stream));
    MXK_CUDA(cudaStreamSynchronize(stream));
    if (host) {
        MXK_CUDA(cudaMemsetAsync(w, 0, sizeof(unsigned), stream));
        if (host & (1u << MXK_ERR_TIMEOUT))
            return fail(MXK_ERR_TIMEOUT, "a device-side wait timed out; the kernel unwound without finishing");
        if (host & (1u << MXK_ERR_NONFINITE))
            return fail(MXK_ERR_NONFINITE,
                        "Non-finite distances: a label outside [0, k) (every distance +inf or NaN); check the input scale");
        return fail(MXK_ERR_CUDA, "device error word set: " + std::to_string(host));
    }
    return MXK_OK;
}

cudaMemPool_t workspace_pool() {
    static std::mutex mu;
    static cudaMemPool_t pools[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (!pools[dev]) {
        cudaMemPoolProps props{};
        props.allocType = cudaMemAllocationTypePinned;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = dev;
        cudaMemPool_t pool = nullptr;
        if (cudaMemPoolCreate(&pool, &props) != cudaSuccess) return nullptr;
        uint64_t keep = ~0ull;  // keep freed blocks mapped for the next call
        if (cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep) != cudaSuccess) {
            cudaMemPoolDestroy(pool);
            return nullptr;
        }
        pools[dev] = pool;
    }
    return pools[dev];
}

int sm_count() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
    return n;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int encode_tensor_map_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                         uint32_t box_inner, uint32_t box_outer, CUtensorMapDataType dtype,
                         CUtensorMapSwizzle swizzle) {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !p)
            return fail(MXK_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
        fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    if (reinterpret_cast<uintptr_t>(base) % 16 || row_bytes % 16)
        return fail(MXK_ERR_UNSUPPORTED, "TMA operand base and row pitch must be 16-byte aligned");
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(MXK_ERR_CUDA, "cuTensorMapEncodeTiled failed with code " + std::to_string(int(r)));
    return MXK_OK;
}

}  // namespace mxk

namespace mxk {
namespace {

// Self-check of the kernels' failure detection: warp 0 waits on an mbarrier
// that nothing arrives on, through dev::mbar_wait (the wait every pipelined
// kernel here uses) with the given limit, so it times out, records
// MXK_ERR_TIMEOUT in the error word and raises the CTA's abort flag; warp 1
// waits on the same barrier with the default limit and leaves through the
// abort flag, as the other roles of an aborted GEMM CTA do.
__global__ void wait_timeout_selftest_kernel(long long limit_cycles, unsigned* err, int* outcome) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        dev::mbar_init(&bar, 1);
        abort_flag = 0;
        dev::fence_barrier_init();
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) {
        volatile int* af = &abort_flag;
        const bool completed = warp == 0 ? dev::mbar_wait(&bar, 0, af, err, limit_cycles)
                                         : dev::mbar_wait(&bar, 0, af, err);
        outcome[warp] = completed ? 1 : 0;  // both must report "gave up"
    }
}

}  // namespace
}  // namespace mxk

extern "C" {

int mxk_check_wait_timeout(long long limit_cycles, int* outcome, void* stream) {
    MXK_REQUIRE(limit_cycles > 0 && limit_cycles <= mxk::dev::kWaitLimitCycles && outcome,
                "check_wait_timeout: limit must be in (0, the kernels' own limit] and outcome non-null");
    unsigned* err = mxk::device_error_word();
    if (!err) return mxk::fail(MXK_ERR_CUDA, "check_wait_timeout: cannot allocate the device error word");
    cudaStream_t s = mxk::as_stream(stream);
    {
        mxk::LaunchScope scope("wait_timeout_selftest", s);
        mxk::wait_timeout_selftest_kernel<<<1, 64, 0, s>>>(limit_cycles, err, outcome);
        MXK_CUDA(cudaGetLastError());
    }
    return mxk::check_device_error(s);
}

const char* mxk_last_error(void) { return mxk::g_last_error.c_str(); }

int mxk_version(void) { return 100; }

uint64_t mxk_launch_count(void) { return mxk::g_launches.load(); }

int mxk_gemm_tiles_multiplied(unsigned long long* count, int reset) {
    unsigned long long* c = mxk::device_tile_counter();
    if (!c) return mxk::fail(MXK_ERR_CUDA, "gemm_tiles_multiplied: no counter on the current device");
    MXK_CUDA(cudaDeviceSynchronize());
    MXK_CUDA(cudaMemcpy(count, c, sizeof(*count), cudaMemcpyDeviceToHost));
    if (reset) MXK_CUDA(cudaMemset(c, 0, sizeof(*c)));
    return MXK_OK;
}

int mxk_gemm_rows_processed(unsigned long long* count, int reset) {
    unsigned long long* c = mxk::device_row_counter();
    if (!c) return mxk::fail(MXK_ERR_CUDA, "gemm_rows_processed: no counter on the current device");
    MXK_CUDA(cudaDeviceSynchronize());
    MXK_CUDA(cudaMemcpy(count, c, sizeof(*count), cudaMemcpyDeviceToHost));
    if (reset) MXK_CUDA(cudaMemset(c, 0, sizeof(*c)));
    return MXK_OK;
}

int mxk_release_workspace(void) {
    cudaMemPool_t pool = mxk::workspace_pool();
    if (!pool) return mxk::fail(MXK_ERR_CUDA, "release_workspace: no workspace pool on the current device");
    MXK_CUDA(cudaDeviceSynchronize());
    MXK_CUDA(cudaMemPoolTrimTo(pool, 0));
    return MXK_OK;
}

int mxk_profile_enable(int on) {
    std::lock_guard<std::mutex> lock(mxk::g_mutex);
    mxk::drain_pending_locked();
    if (on) {
        mxk::g_stats.clear();
        // events for the first launches, created here rather than while timing
        int dev = 0;
        if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < 64) {
            auto& pool = mxk::g_event_pool[dev];
            while (pool.size() < 1024) {
                cudaEvent_t e = nullptr;
                if (cudaEventCreate(&e) != cudaSuccess) {
                    cudaGetLastError();
                    break;
                }
                pool.push_back(e);
            }
        } else {
            cudaGetLastError();
        }
    }
    mxk::g_profiling.store(on ? 1 : 0);
    return MXK_OK;
}

int mxk_profile_read(mxk_kernel_stat* out, int max, int* count) {
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mxk::g_mutex);
    mxk::drain_pending_locked();
    int n = 0;
    for (auto& s : mxk::g_stats) {
        if (s.device != dev) continue;
        if (out && n < max) {
            std::memset(&out[n], 0, sizeof(mxk_kernel_stat));
            std::strncpy(out[n].name, s.name.c_str(), sizeof(out[n].name) - 1);
            out[n].launches = s.launches;
            out[n].total_ms = s.total_ms;
        }
        ++n;
    }
    if (count) *count = n;
    return MXK_OK;
}

}  // extern "C"
