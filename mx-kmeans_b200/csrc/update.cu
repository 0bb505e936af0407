// K3: FP32 centroid update and convergence shift.
//
// Reference: ParCIS/MX-KMeans src/kernels/update.cu:7-61 -- per-cluster sums and
// counts by one global atomicAdd per (point, feature), divide, keep the previous
// center of an empty cluster, then sum((prev - cur)^2) by one atomicAdd per
// element into a single float.
//
// Here: (a) when the K x D sums fit in shared memory, every CTA accumulates a
// private copy with shared-memory atomics and flushes it once with vector
// reductions; (b) otherwise each warp walks a contiguous run of points with
// 128-bit loads, keeps a register sum while consecutive points share a label
// and flushes it with one red.global.add.v4.f32 per 4 features on label change.
// Counts are aggregated the same way.  The finalize kernel divides, applies the
// empty-cluster rule and reduces the shift in a fixed order (bit-reproducible).
#include "common.cuh"
#include "kernels.cuh"

namespace mxk {
namespace {

constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ void red_add_v4(float* addr, float4 v) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}

// Sums of the update are kept in float (the reference-facing update_centroids)
// or double (the Lloyd driver's running sums, which must survive clusters that
// lose most of their points without FP32 cancellation).  Acc4 is four of them.
template <class T>
struct Acc4 {
    T x, y, z, w;
};
template <class T>
__device__ __forceinline__ void acc_zero(Acc4<T>& a) { a.x = a.y = a.z = a.w = T(0); }
template <class T>
__device__ __forceinline__ void acc_add(Acc4<T>& a, float4 v) {
    a.x += (T)v.x, a.y += (T)v.y, a.z += (T)v.z, a.w += (T)v.w;
}
// *dst += a (four consecutive sums), one vector reduction for float
__device__ __forceinline__ void flush4(float* dst, const Acc4<float>& a) {
    red_add_v4(dst, make_float4(a.x, a.y, a.z, a.w));
}
__device__ __forceinline__ void flush4(double* dst, const Acc4<double>& a) {
    atomicAdd(dst, a.x), atomicAdd(dst + 1, a.y), atomicAdd(dst + 2, a.z), atomicAdd(dst + 3, a.w);
}

__device__ __forceinline__ float4 ldg_stream4(const float* p) {
    float4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}

// (b) global path.  Lane owns features 4*lane + 128*j, j < d/128 (d % 128 == 0).
// A label outside [0, k) -- the argmin's INT_MAX when every distance of a
// point is +inf or NaN -- is never used as an index: the point is skipped and
// the error word records MXK_ERR_NONFINITE for the host to report.
__device__ __forceinline__ bool bad_label(int lab, int k, unsigned* err) {
    if ((unsigned)lab < (unsigned)k) return false;
    if (err) atomicOr(err, 1u << MXK_ERR_NONFINITE);
    return true;
}

template <int NJ, class T>
__global__ void __launch_bounds__(256) accumulate_runs_kernel(int64_t n, int d, int k, const float* __restrict__ points,
                                                              const int* __restrict__ labels,
                                                              const int* __restrict__ order, T* __restrict__ sums,
                                                              int* __restrict__ counts, int64_t per_warp,
                                                              unsigned* __restrict__ err, const int* __restrict__ stop) {
    if (stop && *stop) return;  // the Lloyd loop has already converged
    const int lane = threadIdx.x & 31;
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t begin = warp * per_warp;
    if (begin >= n) return;
    const int64_t end = begin + per_warp < n ? begin + per_warp : n;
    Acc4<T> acc[NJ];
    int cur = -1;  // no open run
    int run = 0;
#pragma unroll
    for (int j = 0; j < NJ; ++j) acc_zero(acc[j]);
    // Rows are taken kBatch at a time: their ids, labels and feature vectors
    // are all requested before the first is added, so each warp keeps several
    // rows in flight; the additions stay in row order.
    constexpr int kBatch = NJ <= 2 ? 4 : (NJ <= 4 ? 2 : 1);
    for (int64_t i0 = begin; i0 < end; i0 += kBatch) {
        int64_t pnt[kBatch];
        int lab[kBatch];
        float4 xb[kBatch][NJ];
#pragma unroll
        for (int u = 0; u < kBatch; ++u)
            pnt[u] = i0 + u < end ? (order ? (int64_t)order[i0 + u] : i0 + u) : -1;
#pragma unroll
        for (int u = 0; u < kBatch; ++u) lab[u] = pnt[u] >= 0 ? labels[pnt[u]] : -1;
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            if (pnt[u] >= 0) {
                const float* src = points + pnt[u] * d + 4 * lane;
#pragma unroll
                for (int j = 0; j < NJ; ++j) xb[u][j] = ldg_stream4(src + 128 * j);
            }
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            if (pnt[u] < 0) break;
            if (bad_label(lab[u], k, lane == 0 ? err : nullptr)) continue;
            if (lab[u] != cur) {
                if (cur >= 0) {
                    T* dst = sums + (int64_t)cur * d + 4 * lane;
#pragma unroll
                    for (int j = 0; j < NJ; ++j) flush4(dst + 128 * j, acc[j]), acc_zero(acc[j]);
                    if (lane == 0) atomicAdd(counts + cur, run);
                }
                cur = lab[u];
                run = 0;
            }
#pragma unroll
            for (int j = 0; j < NJ; ++j) acc_add(acc[j], xb[u][j]);
            ++run;
        }
    }
    if (cur < 0) return;
    T* dst = sums + (int64_t)cur * d + 4 * lane;
#pragma unroll
    for (int j = 0; j < NJ; ++j) flush4(dst + 128 * j, acc[j]);
    if (lane == 0) atomicAdd(counts + cur, run);
}

// (a) privatized path: the CTA's copy of all K x D sums and K counts lives in
// shared memory; one warp per point, float4 per lane.
template <class T>
__global__ void __launch_bounds__(512) accumulate_private_kernel(int64_t n, int d, int k,
                                                                 const float* __restrict__ points,
                                                                 const int* __restrict__ labels,
                                                                 const int* __restrict__ order, T* __restrict__ sums,
                                                                 int* __restrict__ counts, unsigned* __restrict__ err,
                                                                 const int* __restrict__ stop) {
    if (stop && *stop) return;
    extern __shared__ __align__(16) unsigned char priv_raw[];
    T* priv = reinterpret_cast<T*>(priv_raw);  // k*d sums, then k counts
    int* pcount = reinterpret_cast<int*>(priv + (int64_t)k * d);
    const int kd = k * d;
    for (int i = threadIdx.x; i < kd; i += blockDim.x) priv[i] = T(0);
    for (int i = threadIdx.x; i < k; i += blockDim.x) pcount[i] = 0;
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int warps = blockDim.x >> 5;
    const int vec_per_row = d >> 2;
    for (int64_t i = (int64_t)blockIdx.x * warps + (threadIdx.x >> 5); i < n; i += (int64_t)gridDim.x * warps) {
        const int64_t pnt = order ? (int64_t)order[i] : i;
        const int lab = labels[pnt];
        if (bad_label(lab, k, lane == 0 ? err : nullptr)) continue;
        const float* src = points + pnt * d;
        T* dst = priv + (int64_t)lab * d;
        for (int v = lane; v < vec_per_row; v += 32) {
            const float4 x = ldg_stream4(src + 4 * v);
            atomicAdd(dst + 4 * v, (T)x.x);
            atomicAdd(dst + 4 * v + 1, (T)x.y);
            atomicAdd(dst + 4 * v + 2, (T)x.z);
            atomicAdd(dst + 4 * v + 3, (T)x.w);
        }
        if (lane == 0) atomicAdd(pcount + lab, 1);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < (kd >> 2); i += blockDim.x) {
        const Acc4<T> v{priv[4 * i], priv[4 * i + 1], priv[4 * i + 2], priv[4 * i + 3]};
        if (v.x != T(0) || v.y != T(0) || v.z != T(0) || v.w != T(0)) flush4(sums + 4 * i, v);
    }
    for (int i = threadIdx.x; i < k; i += blockDim.x)
        if (pcount[i]) atomicAdd(counts + i, pcount[i]);
}

// Generic fallback for d % 128 != 0 (API use with unpadded d).
template <class T>
__global__ void accumulate_scalar_kernel(int64_t n, int d, int k, const float* __restrict__ points,
                                         const int* __restrict__ labels, T* __restrict__ sums,
                                         int* __restrict__ counts, unsigned* __restrict__ err,
                                         const int* __restrict__ stop) {
    if (stop && *stop) return;
    const int64_t total = n * d;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = i / d;
        const int f = (int)(i - row * d);
        const int lab = labels[row];
        if (bad_label(lab, k, f == 0 ? err : nullptr)) continue;
        if (f == 0) atomicAdd(counts + lab, 1);
        atomicAdd(sums + (int64_t)lab * d + f, (T)points[i]);
    }
}

// Incremental update: each recorded label change (point, old, new) moves the
// point's row from cluster old's sum to cluster new's and its count.  A warp
// takes 32 consecutive records (one per lane), groups them by new label and by
// old label (the GEMM visits rows sorted by their previous label, so the old
// labels of neighbouring records mostly agree), sums each group's rows in FP64
// registers and flushes one FP64 reduction per group and feature, instead of
// one per record.  rec[i] = (point, old label, new label, 0), *count entries.
__global__ void __launch_bounds__(256) accumulate_changes_kernel(int d, int k, const float* __restrict__ points,
                                                                 const int4* __restrict__ rec,
                                                                 const int* __restrict__ count,
                                                                 double* __restrict__ sums, int* __restrict__ counts,
                                                                 unsigned* __restrict__ err,
                                                                 const int* __restrict__ stop) {
    if (stop && *stop) return;
    const int lane = threadIdx.x & 31;
    const int warps = (int)((gridDim.x * blockDim.x) >> 5);
    const int nrec = *count;
    for (int base = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5) * 32; base < nrec; base += warps * 32) {
        int4 c = base + lane < nrec ? rec[base + lane] : make_int4(0, -1, -1, 0);
        bool valid = base + lane < nrec;
        if (valid && (bad_label(c.z, k, err) || bad_label(c.y, k, err))) valid = false;
        const unsigned live = __ballot_sync(kFull, valid);
        if (!valid) c.y = c.z = -1;
        const int point = c.x;
#pragma unroll 1
        for (int side = 0; side < 2; ++side) {
            const int key = side ? c.y : c.z;
            const unsigned peers = __match_any_sync(kFull, key);
            if (valid && lane == __ffs(peers) - 1) atomicAdd(counts + key, side ? -__popc(peers) : __popc(peers));
            unsigned leads = __ballot_sync(kFull, valid && lane == __ffs(peers) - 1) & live;
            while (leads) {
                const int l = __ffs(leads) - 1;
                leads &= leads - 1;
                const unsigned members = __shfl_sync(kFull, peers, l);
                const int label = __shfl_sync(kFull, key, l);
                double* dst = sums + (int64_t)label * d;
                for (int f0 = 0; f0 < d; f0 += 128) {  // (warp-uniform trip count: the shuffles below)
                    const int f = f0 + 4 * lane;
                    Acc4<double> acc;
                    acc_zero(acc);
                    unsigned m = members;
                    while (m) {
                        const int j = __ffs(m) - 1;
                        m &= m - 1;
                        const int64_t row = __shfl_sync(kFull, point, j);
                        // (cached in L1: the other side's group reads the row again)
                        if (f < d) acc_add(acc, __ldg(reinterpret_cast<const float4*>(points + row * d + f)));
                    }
                    if (side) acc.x = -acc.x, acc.y = -acc.y, acc.z = -acc.z, acc.w = -acc.w;
                    if (f < d) flush4(dst + f, acc);
                }
            }
        }
    }
}

// Applies the stopping rule to the Lloyd driver's state words for shift s
// (kmeans.cu:62-67): counts the iteration and stops on a non-finite shift or
// one <= tolerance.
__device__ __forceinline__ void apply_stop_rule(int* loop, float s, float tolerance) {
    loop[1] += 1;
    if (!isfinite(s)) {
        loop[2] = 1;
        loop[0] = 1;
        loop[3] = 0;
    } else if (s <= tolerance) {
        loop[0] = 1;
        loop[3] = 0;
    }
}

// Divides, applies the empty-cluster rule, and writes this CTA's partial shift
// (sum of (old - new)^2 over its grid-stride elements, reduced in a fixed order)
// to partials[blockIdx.x].  The grid size is fixed by the shape, so the shift is
// bit-identical on every GPU that runs it -- all ranks of a sharded run stop on
// the same iteration without exchanging it.  With `loop` (the Lloyd driver's
// state words) the CTA that finishes last (a ticket on *done, which it resets
// to 0) also sums the partials in index order into *total_out and applies the
// stopping rule; once loop[0] is set the launch does nothing except publish
// the state.  Driver options: old may be centroids itself (each element is
// read, then written, by one thread); prev_out receives the old centroids;
// zero_sums leaves sums and counts zeroed for the next accumulation;
// host_state (host-mapped) receives the four state words.  With acc_sums /
// acc_counts (FP64 running sums and int counts kept across iterations), sums /
// counts are this iteration's additions: full replaces the running values with
// them (a fresh accumulation), otherwise they are added (label changes); the
// last CTA also zeroes *zero_word (the change list's count).  The
// centroid is the running sum rounded to FP32, divided by the count in FP32,
// as the reference divides its FP32 sums.
__device__ __forceinline__ void publish_state(const int* loop, int* host_state) {
    if (!host_state) return;
    volatile const int* src = loop;
    volatile int* dst = host_state;
    for (int i = 0; i < 4; ++i) dst[i] = src[i];
    __threadfence_system();
}

template <class T>
__global__ void __launch_bounds__(256) finalize_kernel(int d, int k, T* __restrict__ sums, int* __restrict__ counts,
                                                       const float* old, float* centroids, float* __restrict__ prev_out,
                                                       float* __restrict__ partials, int* __restrict__ loop,
                                                       unsigned* __restrict__ done, float* __restrict__ total_out,
                                                       float tolerance, int zero_sums, int* __restrict__ host_state,
                                                       double* __restrict__ acc_sums, int* __restrict__ acc_counts,
                                                       int full_host, int* __restrict__ zero_word,
                                                       const int* __restrict__ full_dev) {
    if (loop && *(volatile int*)loop) {  // converged: the centroids stay as they are
        if (blockIdx.x == 0 && threadIdx.x == 0) publish_state(loop, host_state);
        return;
    }
    const int full = full_dev ? *full_dev : full_host;
    __shared__ float warp_sum[8];
    const int64_t total = (int64_t)k * d;
    float local = 0.0f;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        int cnt = counts[i / d];
        float sum = (float)sums[i];
        if (acc_sums) {
            const double run = (full ? 0.0 : acc_sums[i]) + (double)sums[i];
            acc_sums[i] = run;
            sum = (float)run;
            if (!full) cnt += acc_counts[i / d];
        }
        const float o = old[i];
        // An empty cluster keeps its previous center (update.cu:26-29).
        const float v = cnt ? sum / (float)cnt : o;
        const float diff = o - v;
        if (prev_out) prev_out[i] = o;
        if (zero_sums) sums[i] = T(0);
        centroids[i] = v;
        local += diff * diff;
    }
    if (!partials) return;
    for (int o = 16; o; o >>= 1) local += __shfl_xor_sync(kFull, local, o);
    if ((threadIdx.x & 31) == 0) warp_sum[threadIdx.x >> 5] = local;
    __syncthreads();
    __shared__ bool last;
    if (threadIdx.x == 0) {
        float s = 0.0f;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += warp_sum[w];
        partials[blockIdx.x] = s;
        if (loop) {
            __threadfence();  // the partial is visible before the ticket is taken
            last = atomicAdd(done, 1u) == gridDim.x - 1;
        }
    }
    if (!loop) return;
    __syncthreads();
    if (!last) return;
    __threadfence();
    local = 0.0f;
    for (int i = threadIdx.x; i < (int)gridDim.x; i += blockDim.x) local += __ldcg(partials + i);
    for (int o = 16; o; o >>= 1) local += __shfl_xor_sync(kFull, local, o);
    if ((threadIdx.x & 31) == 0) warp_sum[threadIdx.x >> 5] = local;
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = 0.0f;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += warp_sum[w];
        *total_out = s;
        *done = 0u;
        if (zero_word) *zero_word = 0;
        apply_stop_rule(loop, s, tolerance);
        __threadfence();
        publish_state(loop, host_state);
    }
    if (zero_sums || acc_counts) {  // every CTA has read its counts (it took a ticket after its loop)
        __syncthreads();
        for (int c = threadIdx.x; c < k; c += blockDim.x) {
            if (acc_counts) acc_counts[c] = (full ? 0 : acc_counts[c]) + counts[c];
            if (zero_sums) counts[c] = 0;
        }
    }
}

// Sums the per-CTA partials in a fixed order into out[0].  With `loop` (the
// Lloyd driver's state words, see launch_finalize) it also applies the stopping
// rule, and does nothing once the loop has stopped.
__global__ void sum_partials_kernel(const float* __restrict__ partials, int count, float* __restrict__ out,
                                    int* __restrict__ loop, float tolerance) {
    if (loop && *(volatile int*)loop) return;  // read by every thread before thread 0 can write it
    __shared__ float warp_sum[32];
    float local = 0.0f;
    for (int i = threadIdx.x; i < count; i += blockDim.x) local += partials[i];
    for (int o = 16; o; o >>= 1) local += __shfl_xor_sync(kFull, local, o);
    if ((threadIdx.x & 31) == 0) warp_sum[threadIdx.x >> 5] = local;
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = 0.0f;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += warp_sum[w];
        out[0] = s;
        if (loop) apply_stop_rule(loop, s, tolerance);
    }
}

__global__ void __launch_bounds__(256) shift_kernel(int64_t elements, const float* __restrict__ prev,
                                                    const float* __restrict__ cur, float* __restrict__ partials) {
    __shared__ float warp_sum[8];
    float local = 0.0f;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < elements; i += (int64_t)gridDim.x * blockDim.x) {
        const float diff = prev[i] - cur[i];
        local += diff * diff;
    }
    for (int o = 16; o; o >>= 1) local += __shfl_xor_sync(kFull, local, o);
    if ((threadIdx.x & 31) == 0) warp_sum[threadIdx.x >> 5] = local;
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = 0.0f;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += warp_sum[w];
        partials[blockIdx.x] = s;
    }
}

constexpr int kShiftBlocks = 256;  // fixed grid of the shift reduction (<= partial slots)

template <class T>
int accumulate_impl(bool switched, int64_t n, int d, int k, const float* points, const int* labels, const int* order,
                    T* sums, int* counts, cudaStream_t stream, const int* stop) {
    if (n <= 0) return MXK_OK;
    MXK_REQUIRE(d > 0 && k > 0 && points && labels && sums && counts, "update_centroids: bad arguments");
    const int sms = sm_count();
    unsigned* err = device_error_word();
    if (!err) return fail(MXK_ERR_CUDA, "update_centroids: cannot allocate the device error word");
    const bool aligned = (reinterpret_cast<uintptr_t>(points) % 16 == 0) && (reinterpret_cast<uintptr_t>(sums) % 16 == 0);
    const int64_t priv_bytes = (int64_t)k * d * (int64_t)sizeof(T) + (int64_t)k * 4;
    int max_smem = 0, dev = 0;
    MXK_CUDA(cudaGetDevice(&dev));
    MXK_CUDA(cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    // A label-sorted visiting order makes the run kernel's flushes rare, which
    // beats per-element shared-memory atomics; without one, privatize when the
    // sums fit in shared memory.
    if (!order && aligned && d % 4 == 0 && priv_bytes <= max_smem && priv_bytes <= 200 * 1024 && n >= (int64_t)k * 64) {
        MXK_CUDA(cudaFuncSetAttribute(accumulate_private_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)priv_bytes));
        LaunchScope scope(switched ? "accumulate_private_switched" : "accumulate_private", stream);
        accumulate_private_kernel<T><<<sms, 512, (size_t)priv_bytes, stream>>>(n, d, k, points, labels, order, sums,
                                                                                counts, err, stop);
        MXK_CUDA(cudaGetLastError());
        return MXK_OK;
    }
    if (aligned && d % 128 == 0 && d <= 1024) {
        // one wave: as many warps as the SMs hold at once, each a contiguous
        // range of rows
        auto launch = [&](auto kernel) -> int {
            int per_sm = 0;
            MXK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, 256, 0));
            if (per_sm < 1) per_sm = 1;
            const int64_t warps_total = (int64_t)sms * per_sm * 8;
            int64_t per_warp = (n + warps_total - 1) / warps_total;
            if (per_warp < 16) per_warp = 16;
            const int64_t warps = (n + per_warp - 1) / per_warp;
            const int64_t blocks = (warps * 32 + 255) / 256;
            LaunchScope scope(switched ? "accumulate_runs_switched" : "accumulate_runs", stream);
            kernel<<<(unsigned)blocks, 256, 0, stream>>>(n, d, k, points, labels, order, sums, counts, per_warp, err,
                                                         stop);
            MXK_CUDA(cudaGetLastError());
            return MXK_OK;
        };
        switch (d / 128) {
            case 1: return launch(accumulate_runs_kernel<1, T>);
            case 2: return launch(accumulate_runs_kernel<2, T>);
            case 3: return launch(accumulate_runs_kernel<3, T>);
            case 4: return launch(accumulate_runs_kernel<4, T>);
            case 5: return launch(accumulate_runs_kernel<5, T>);
            case 6: return launch(accumulate_runs_kernel<6, T>);
            case 7: return launch(accumulate_runs_kernel<7, T>);
            default: return launch(accumulate_runs_kernel<8, T>);
        }
    }
    LaunchScope scope(switched ? "accumulate_scalar_switched" : "accumulate_scalar", stream);
    accumulate_scalar_kernel<T><<<sms * 8, 256, 0, stream>>>(n, d, k, points, labels, sums, counts, err, stop);
    MXK_CUDA(cudaGetLastError());
    return MXK_OK;
}

template <class T>
int finalize_impl(int d, int k, T* sums, int* counts, const float* old_centroids, float* centroids,
                  float* shift_scratch, cudaStream_t stream, int* loop, float tolerance, float* prev_out,
                  bool zero_sums, int* host_state, double* acc_sums, int* acc_counts, bool full, int* zero_word,
                  const int* full_dev) {
    MXK_REQUIRE(!(zero_sums || host_state || acc_sums) || loop,
                "finalize: zeroing, running sums and the host state need the loop words");
    MXK_REQUIRE(!acc_sums == !acc_counts, "finalize: running sums and counts go together");
    MXK_REQUIRE(!loop || shift_scratch, "finalize: the loop state needs the shift scratch");
    const int64_t total = (int64_t)k * d;
    int64_t blocks = (total + 255) / 256;
    if (blocks > kShiftBlocks) blocks = kShiftBlocks;
    {
        LaunchScope scope("finalize", stream);
        finalize_kernel<T><<<(unsigned)blocks, 256, 0, stream>>>(
            d, k, sums, counts, old_centroids, centroids, prev_out, shift_scratch, loop,
            loop ? reinterpret_cast<unsigned*>(shift_scratch + kShiftBlocks + 1) : nullptr,
            loop ? shift_scratch + kShiftBlocks : nullptr, tolerance, zero_sums ? 1 : 0, host_state, acc_sums,
            acc_counts, full ? 1 : 0, zero_word, full_dev);
        MXK_CUDA(cudaGetLastError());
    }
    if (shift_scratch && !loop) {  // (with loop the finalize kernel's last CTA sums the partials)
        LaunchScope scope("shift_total", stream);
        sum_partials_kernel<<<1, 1024, 0, stream>>>(shift_scratch, (int)blocks, shift_scratch + kShiftBlocks, loop,
                                                    tolerance);
        MXK_CUDA(cudaGetLastError());
    }
    return MXK_OK;
}

}  // namespace

int launch_accumulate(int64_t n, int d, int k, const float* points, const int* labels, const int* order, float* sums,
                      int* counts, cudaStream_t stream, const int* stop) {
    return accumulate_impl(false, n, d, k, points, labels, order, sums, counts, stream, stop);
}
int launch_accumulate(int64_t n, int d, int k, const float* points, const int* labels, const int* order, double* sums,
                      int* counts, cudaStream_t stream, const int* stop, bool switched) {
    return accumulate_impl(switched, n, d, k, points, labels, order, sums, counts, stream, stop);
}

namespace {
// w = (skip the incremental update, skip the fresh accumulation, fresh): the
// fresh accumulation of every point replaces the incremental one once more
// than `threshold` labels changed; both are skipped once the loop has stopped.
__global__ void update_gate_kernel(const int* __restrict__ stop, const int* __restrict__ changes, int threshold,
                                   int* __restrict__ w) {
    if (threadIdx.x != 0) return;
    const bool stopped = stop && *stop;
    const bool fresh = *changes > threshold;
    w[0] = stopped || fresh;
    w[1] = stopped || !fresh;
    w[2] = fresh;
}
}  // namespace

int launch_update_gate(const int* stop, const int* changes, int threshold, int* words, cudaStream_t stream) {
    MXK_REQUIRE(changes && words, "update_gate: bad arguments");
    LaunchScope scope("update_gate", stream);
    update_gate_kernel<<<1, 32, 0, stream>>>(stop, changes, threshold, words);
    MXK_CUDA(cudaGetLastError());
    return MXK_OK;
}

int launch_accumulate_changes(int d, int k, const float* points, const int4* rec, const int* count, double* sums,
                              int* counts, cudaStream_t stream, const int* stop) {
    MXK_REQUIRE(d > 0 && d % 4 == 0 && points && rec && count && sums && counts, "accumulate_changes: bad arguments");
    MXK_REQUIRE(reinterpret_cast<uintptr_t>(points) % 16 == 0 && reinterpret_cast<uintptr_t>(sums) % 16 == 0,
                "accumulate_changes: points and sums must be 16-byte aligned");
    unsigned* err = device_error_word();
    if (!err) return fail(MXK_ERR_CUDA, "accumulate_changes: cannot allocate the device error word");
    LaunchScope scope("accumulate_changes", stream);
    accumulate_changes_kernel<<<(unsigned)(sm_count() * 8), 256, 0, stream>>>(d, k, points, rec, count, sums, counts,
                                                                             err, stop);
    MXK_CUDA(cudaGetLastError());
    return MXK_OK;
}

// [0, kShiftBlocks): partials, [kShiftBlocks]: the total, [kShiftBlocks + 1]:
// the finalize kernel's ticket counter (zero between launches)
int64_t shift_scratch_floats() { return kShiftBlocks + 2; }
int64_t shift_total_index() { return kShiftBlocks; }

int launch_finalize(int d, int k, float* sums, int* counts, const float* old_centroids, float* centroids,
                    float* shift_scratch, cudaStream_t stream, int* loop, float tolerance, float* prev_out,
                    bool zero_sums, int* host_state, double* acc_sums, int* acc_counts, bool full, int* zero_word,
                    const int* full_dev) {
    return finalize_impl(d, k, sums, counts, old_centroids, centroids, shift_scratch, stream, loop, tolerance, prev_out,
                         zero_sums, host_state, acc_sums, acc_counts, full, zero_word, full_dev);
}
int launch_finalize(int d, int k, double* sums, int* counts, const float* old_centroids, float* centroids,
                    float* shift_scratch, cudaStream_t stream, int* loop, float tolerance, float* prev_out,
                    bool zero_sums, int* host_state, double* acc_sums, int* acc_counts, bool full, int* zero_word,
                    const int* full_dev) {
    return finalize_impl(d, k, sums, counts, old_centroids, centroids, shift_scratch, stream, loop, tolerance, prev_out,
                         zero_sums, host_state, acc_sums, acc_counts, full, zero_word, full_dev);
}

int launch_shift(int64_t elements, const float* previous, const float* current, float* shift_scratch,
                 cudaStream_t stream) {
    int64_t blocks = (elements + 255) / 256;
    if (blocks > kShiftBlocks) blocks = kShiftBlocks;
    if (blocks < 1) blocks = 1;
    {
        LaunchScope scope("shift", stream);
        shift_kernel<<<(unsigned)blocks, 256, 0, stream>>>(elements, previous, current, shift_scratch);
        MXK_CUDA(cudaGetLastError());
    }
    LaunchScope scope("shift_total", stream);
    sum_partials_kernel<<<1, 1024, 0, stream>>>(shift_scratch, (int)blocks, shift_scratch + kShiftBlocks, nullptr,
                                                0.0f);
    MXK_CUDA(cudaGetLastError());
    return MXK_OK;
}

}  // namespace mxk

extern "C" {

int mxk_update_centroids(int64_t n, int d, int k, const float* points, const int* labels, const float* old_centroids,
                         float* centroids, int* counts, void* stream) {
    cudaStream_t s = mxk::as_stream(stream);
    MXK_REQUIRE(d > 0 && k > 0, "update_centroids: bad arguments");
    MXK_REQUIRE(centroids != old_centroids, "update_centroids: centroids and old_centroids must differ");
    MXK_CUDA(cudaMemsetAsync(centroids, 0, sizeof(float) * (size_t)k * d, s));
    MXK_CUDA(cudaMemsetAsync(counts, 0, sizeof(int) * (size_t)k, s));
    MXK_CHECK(mxk::launch_accumulate(n, d, k, points, labels, nullptr, centroids, counts, s));
    MXK_CHECK(mxk::launch_finalize(d, k, centroids, counts, old_centroids, centroids, nullptr, s));
    // Reports labels outside [0, k) (skipped above) instead of writing past the
    // sums as an unchecked index would.
    return mxk::check_device_error(s);
}

int mxk_centroid_shift(int64_t elements, const float* previous, const float* current, float* device_sum,
                       float* host_result, void* stream) {
    cudaStream_t s = mxk::as_stream(stream);
    MXK_REQUIRE(device_sum != nullptr, "centroid_shift: null device_sum");
    float h = 0.0f;
    if (elements > 0) {
        float* scratch = nullptr;
        MXK_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&scratch), sizeof(float) * mxk::shift_scratch_floats(), s));
        int st = mxk::launch_shift(elements, previous, current, scratch, s);
        if (st == MXK_OK) {
            cudaError_t e = cudaMemcpyAsync(device_sum, scratch + mxk::shift_total_index(), sizeof(float),
                                            cudaMemcpyDeviceToDevice, s);
            if (e != cudaSuccess) st = mxk::fail_cuda("cudaMemcpyAsync", e);
        }
        cudaFreeAsync(scratch, s);
        if (st != MXK_OK) return st;
    } else {
        MXK_CUDA(cudaMemsetAsync(device_sum, 0, sizeof(float), s));
    }
    MXK_CUDA(cudaMemcpyAsync(&h, device_sum, sizeof(float), cudaMemcpyDeviceToHost, s));
    MXK_CUDA(cudaStreamSynchronize(s));
    if (host_result) *host_result = h;
    return MXK_OK;
}

}  // extern "C"
