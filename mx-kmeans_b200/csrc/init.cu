// Centroid initialisation on the GPU, bit-identical to the reference's host code.
//
// Reference: ParCIS/MX-KMeans include/host_utils.hpp:80-119 (init_centroids,
// D^2-sampling K-Means++: std::mt19937, double squared distances accumulated
// feature by feature, a sequential double running sum, uniform_real_distribution
// target) and :121-141 (init_centroids_farthest: float squared distances, the
// first maximum).  The reference runs both on one host thread, O(N*D) per
// center -- hours at N = 8M, K = 2048.
//
// Here every per-point distance is one GPU thread evaluating exactly the
// reference's expression (same operation order, no contraction: __f*_rn /
// __d*_rn), so distances and minima are bit-identical.  The parts that are
// order-dependent in the reference are handled so that the choice is the same:
//   * farthest-first: the first maximum is an exact parallel reduction
//     (value, then lowest index; std::max_element never moves off a NaN at
//     index 0 and never onto a NaN elsewhere).
//   * K-Means++: the reference draws against a running double sum whose
//     rounding depends on the order.  The GPU computes a parallel prefix sum P
//     (block sums, scanned block offsets, in-block scans) and locates the first
//     point whose P exceeds the target.  The sequential sums S the reference
//     would form differ from the exact sums T by at most gamma_n T, and so do
//     the parallel ones, so |S - P| <= 2 gamma_n T_n / (1 - gamma_n) for every
//     prefix (nonnegative terms; gamma_n = n u / (1 - n u), u = 2^-53).  When
//     the target, bounded the same way, lies clear of both P values around the
//     candidate, the sequential search would pick the same point; otherwise
//     (a few percent of centers at N = 8M, never at small N) the host repeats
//     the reference's sequential loop on the distances exactly.  The random
//     draw itself stays on the host (std::generate_canonical, the call
//     uniform_real_distribution makes), one per center as in the reference.
#include <cmath>
#include <cstring>
#include <limits>
#include <random>
#include <vector>

#include "common.cuh"
#include "kernels.cuh"

namespace mxk {
namespace {

constexpr int kInitBlock = 256;  // points per block (one per thread)

__device__ __forceinline__ float4 ldg4f(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

// ---- farthest-first ---------------------------------------------------------

// dist[p] = min(dist[p], sum_j (x_pj - c_j)^2) in float, features in order; the
// center's own entry becomes -1 (host_utils.hpp:130-137).  Each block reports
// its first maximum (NaN never wins).
__global__ void __launch_bounds__(kInitBlock) far_dist_kernel(int64_t n, int d, const float* __restrict__ points,
                                                              const int64_t* __restrict__ pick, float* __restrict__ dist,
                                                              float* __restrict__ best_val,
                                                              int64_t* __restrict__ best_idx) {
    extern __shared__ float cs[];  // the center row
    const int64_t c = *pick;
    for (int j = threadIdx.x; j < d; j += blockDim.x) cs[j] = points[c * d + j];
    __syncthreads();
    const int64_t p = (int64_t)blockIdx.x * kInitBlock + threadIdx.x;
    float v = __int_as_float(0x7fc00000);  // NaN: never the maximum
    int64_t vi = INT64_MAX;
    if (p < n) {
        const float* row = points + p * d;
        float s = 0.0f;
        for (int j = 0; j < d; j += 4) {
            const float4 x = ldg4f(row + j);
            float t = __fsub_rn(x.x, cs[j]);
            s = __fadd_rn(s, __fmul_rn(t, t));
            t = __fsub_rn(x.y, cs[j + 1]);
            s = __fadd_rn(s, __fmul_rn(t, t));
            t = __fsub_rn(x.z, cs[j + 2]);
            s = __fadd_rn(s, __fmul_rn(t, t));
            t = __fsub_rn(x.w, cs[j + 3]);
            s = __fadd_rn(s, __fmul_rn(t, t));
        }
        const float old = dist[p];
        v = s < old ? s : old;  // std::min(old, s)
        if (p == c) v = -1.0f;
        dist[p] = v;
        vi = p;
    }
    // first maximum: larger value wins, equal values keep the lower index
    auto better = [](float a, int64_t ai, float b, int64_t bi) {
        if (b != b) return false;
        if (a != a) return true;
        return b > a || (b == a && bi < ai);
    };
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int64_t oi = __shfl_xor_sync(0xffffffffu, vi, o);
        if (better(v, vi, ov, oi)) v = ov, vi = oi;
    }
    __shared__ float wv[kInitBlock / 32];
    __shared__ int64_t wi[kInitBlock / 32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) wv[warp] = v, wi[warp] = vi;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < kInitBlock / 32; ++w)
            if (better(v, vi, wv[w], wi[w])) v = wv[w], vi = wi[w];
        best_val[blockIdx.x] = v;
        best_idx[blockIdx.x] = vi;
    }
}

// Reduces the block maxima to the next center (std::max_element: the first
// maximum, or index 0 when dist[0] is NaN) and copies its row to out_row.
__global__ void __launch_bounds__(1024) far_select_kernel(int nblocks, int d, const float* __restrict__ points,
                                                          const float* __restrict__ dist,
                                                          const float* __restrict__ best_val,
                                                          const int64_t* __restrict__ best_idx,
                                                          int64_t* __restrict__ pick, float* __restrict__ out_row) {
    float v = __int_as_float(0x7fc00000);
    int64_t vi = INT64_MAX;
    auto better = [](float a, int64_t ai, float b, int64_t bi) {
        if (b != b) return false;
        if (a != a) return true;
        return b > a || (b == a && bi < ai);
    };
    for (int b = threadIdx.x; b < nblocks; b += blockDim.x)
        if (better(v, vi, best_val[b], best_idx[b])) v = best_val[b], vi = best_idx[b];
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int64_t oi = __shfl_xor_sync(0xffffffffu, vi, o);
        if (better(v, vi, ov, oi)) v = ov, vi = oi;
    }
    __shared__ float wv[32];
    __shared__ int64_t wi[32];
    __shared__ int64_t chosen;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) wv[warp] = v, wi[warp] = vi;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
            if (better(v, vi, wv[w], wi[w])) v = wv[w], vi = wi[w];
        const float d0 = dist[0];
        if (d0 != d0 || vi == INT64_MAX) vi = 0;  // max_element stays on a NaN first element
        *pick = vi;
        chosen = vi;
    }
    __syncthreads();
    if (out_row)
        for (int j = threadIdx.x; j < d; j += blockDim.x) out_row[j] = points[chosen * d + j];
}

// ---- K-Means++ ----------------------------------------------------------------

// dist[p] = selected[p] ? 0 : min(dist[p], sum_j (double(x_pj) - c_j)^2), the
// sum in double, features in order (host_utils.hpp:88-97); block sums for the
// prefix sums (any order).
__global__ void __launch_bounds__(kInitBlock) kpp_dist_kernel(int64_t n, int d, const float* __restrict__ points,
                                                              const float* __restrict__ center,
                                                              const uint8_t* __restrict__ selected,
                                                              double* __restrict__ dist, double* __restrict__ block_sums) {
    extern __shared__ double cd[];  // the center row in double
    for (int j = threadIdx.x; j < d; j += blockDim.x) cd[j] = (double)center[j];
    __syncthreads();
    const int64_t p = (int64_t)blockIdx.x * kInitBlock + threadIdx.x;
    double v = 0.0;
    if (p < n) {
        const float* row = points + p * d;
        double s = 0.0;
        for (int j = 0; j < d; j += 4) {
            const float4 x = ldg4f(row + j);
            double t = __dsub_rn((double)x.x, cd[j]);
            s = __dadd_rn(s, __dmul_rn(t, t));
            t = __dsub_rn((double)x.y, cd[j + 1]);
            s = __dadd_rn(s, __dmul_rn(t, t));
            t = __dsub_rn((double)x.z, cd[j + 2]);
            s = __dadd_rn(s, __dmul_rn(t, t));
            t = __dsub_rn((double)x.w, cd[j + 3]);
            s = __dadd_rn(s, __dmul_rn(t, t));
        }
        const double old = dist[p];
        v = selected[p] ? 0.0 : (s < old ? s : old);  // std::min(old, s)
        dist[p] = v;
    }
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __shared__ double ws[kInitBlock / 32];
    if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int w = 0; w < kInitBlock / 32; ++w) t += ws[w];
        block_sums[blockIdx.x] = t;
    }
}

// Exclusive scan of the block sums (one block): offsets[b]; out[0] = the total.
__global__ void __launch_bounds__(1024) kpp_scan_kernel(int nblocks, const double* __restrict__ block_sums,
                                                        double* __restrict__ offsets, double* __restrict__ out) {
    __shared__ double carry;
    __shared__ double wsum[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) carry = 0.0;
    __syncthreads();
    for (int base = 0; base < nblocks; base += blockDim.x) {
        const int b = base + threadIdx.x;
        const double x = b < nblocks ? block_sums[b] : 0.0;
        double incl = x;
        for (int o = 1; o < 32; o <<= 1) {
            const double t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
        }
        if (lane == 31) wsum[warp] = incl;
        __syncthreads();
        if (warp == 0) {
            double w = lane < (int)(blockDim.x >> 5) ? wsum[lane] : 0.0;
            double wi = w;
            for (int o = 1; o < 32; o <<= 1) {
                const double t = __shfl_up_sync(0xffffffffu, wi, o);
                if (lane >= o) wi += t;
            }
            wsum[lane] = wi - w;
        }
        __syncthreads();
        if (b < nblocks) offsets[b] = carry + (wsum[warp] + (incl - x));
        __syncthreads();
        if (threadIdx.x == blockDim.x - 1) carry += wsum[warp] + incl;
        __syncthreads();
    }
    if (threadIdx.x == 0) out[0] = carry;
}

// First point whose parallel prefix sum P exceeds t.  Each block scans its own
// distances on top of its offset; the block holding a crossing records the
// prefix sums just before and at it.  out_idx: atomic minimum (start INT64_MAX).
__global__ void __launch_bounds__(kInitBlock) kpp_find_kernel(int64_t n, const double* __restrict__ dist,
                                                              const double* __restrict__ offsets, double t,
                                                              unsigned long long* __restrict__ out_idx,
                                                              double2* __restrict__ slots) {
    const int64_t p = (int64_t)blockIdx.x * kInitBlock + threadIdx.x;
    const double x = p < n ? dist[p] : 0.0;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    double incl = x;
    for (int o = 1; o < 32; o <<= 1) {
        const double v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    __shared__ double wsum[kInitBlock / 32];
    __shared__ int first;
    if (lane == 31) wsum[warp] = incl;
    if (threadIdx.x == 0) first = INT32_MAX;
    __syncthreads();
    double wofs = 0.0;
    for (int w = 0; w < warp; ++w) wofs += wsum[w];
    const double off = offsets[blockIdx.x];
    const double pe = off + (wofs + (incl - x));  // prefix before p
    const double pi = off + (wofs + incl);        // prefix through p
    if (p < n && pi > t) atomicMin(&first, (int)threadIdx.x);
    __syncthreads();
    if ((int)threadIdx.x == first) {
        slots[blockIdx.x] = make_double2(threadIdx.x == 0 ? off : pe, pi);
        atomicMin(out_idx, (unsigned long long)p);
    }
}

// First point not yet chosen (the reference's fallback, host_utils.hpp:112-115).
__global__ void kpp_first_free_kernel(int64_t n, const uint8_t* __restrict__ selected,
                                      unsigned long long* __restrict__ out_idx) {
    for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < n; p += (int64_t)gridDim.x * blockDim.x)
        if (!selected[p]) {
            atomicMin(out_idx, (unsigned long long)p);
            return;
        }
}

template <typename T>
__global__ void fill_kernel(T* __restrict__ out, int64_t n, T value) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = value;
}

struct DeviceScratch {
    std::vector<void*> ptrs;
    cudaStream_t stream;
    explicit DeviceScratch(cudaStream_t s) : stream(s) {}
    ~DeviceScratch() {
        for (void* p : ptrs) cudaFreeAsync(p, stream);
    }
    template <typename T>
    int alloc(T** out, int64_t count) {
        void* p = nullptr;
        cudaMemPool_t pool = workspace_pool();
        if (!pool) return fail(MXK_ERR_CUDA, "init: cannot create the memory pool");
        cudaError_t e = cudaMallocFromPoolAsync(&p, sizeof(T) * (size_t)(count > 0 ? count : 1), pool, stream);
        if (e != cudaSuccess) return fail_cuda("cudaMallocFromPoolAsync (init workspace)", e);
        ptrs.push_back(p);
        *out = static_cast<T*>(p);
        return MXK_OK;
    }
};

int check_init_args(int64_t n, int d, int k, const float* points, const float* centroids) {
    MXK_REQUIRE(n > 0 && n <= INT32_MAX, "init: n must be in 1..2^31-1");
    MXK_REQUIRE(k > 0 && k <= n, "init: k must be in 1..n");
    MXK_REQUIRE(d > 0 && d % 4 == 0 && d <= 4096, "init: d must be a positive multiple of 4 (at most 4096)");
    MXK_REQUIRE(points && centroids, "init: null points or centroids");
    MXK_REQUIRE(reinterpret_cast<uintptr_t>(points) % 16 == 0, "init: points must be 16-byte aligned");
    return MXK_OK;
}

}  // namespace

int run_init_farthest(int64_t n, int d, int k, const float* points, float* centroids, cudaStream_t stream) {
    MXK_CHECK(check_init_args(n, d, k, points, centroids));
    const int64_t nb = (n + kInitBlock - 1) / kInitBlock;
    DeviceScratch ws(stream);
    float *dist = nullptr, *best_val = nullptr;
    int64_t *best_idx = nullptr, *pick = nullptr;
    MXK_CHECK(ws.alloc(&dist, n));
    MXK_CHECK(ws.alloc(&best_val, nb));
    MXK_CHECK(ws.alloc(&best_idx, nb));
    MXK_CHECK(ws.alloc(&pick, 1));
    // dist = FLT_MAX, first center = row 0 (host_utils.hpp:124-127)
    fill_kernel<float><<<(unsigned)std::min<int64_t>(nb, 4096), kInitBlock, 0, stream>>>(
        dist, n, std::numeric_limits<float>::max());
    MXK_CUDA(cudaGetLastError());
    MXK_CUDA(cudaMemsetAsync(pick, 0, sizeof(int64_t), stream));
    MXK_CUDA(cudaMemcpyAsync(centroids, points, sizeof(float) * (size_t)d, cudaMemcpyDeviceToDevice, stream));
    const size_t smem = sizeof(float) * (size_t)d;
    for (int c = 0; c < k; ++c) {
        {
            LaunchScope scope("init_farthest_dist", stream);
            far_dist_kernel<<<(unsigned)nb, kInitBlock, smem, stream>>>(n, d, points, pick, dist, best_val, best_idx);
            MXK_CUDA(cudaGetLastError());
        }
        LaunchScope scope("init_farthest_select", stream);
        far_select_kernel<<<1, 1024, 0, stream>>>((int)nb, d, points, dist, best_val, best_idx, pick,
                                                  c + 1 < k ? centroids + (size_t)(c + 1) * d : nullptr);
        MXK_CUDA(cudaGetLastError());
    }
    MXK_CUDA(cudaStreamSynchronize(stream));
    return MXK_OK;
}

int run_init_kmeanspp(int64_t n, int d, int k, const float* points, float* centroids, uint32_t seed,
                      cudaStream_t stream) {
    MXK_CHECK(check_init_args(n, d, k, points, centroids));
    const int64_t nb = (n + kInitBlock - 1) / kInitBlock;
    DeviceScratch ws(stream);
    double *dist = nullptr, *block_sums = nullptr, *offsets = nullptr, *total_dev = nullptr;
    uint8_t* selected = nullptr;
    unsigned long long* idx_dev = nullptr;
    double2* slots = nullptr;
    MXK_CHECK(ws.alloc(&dist, n));
    MXK_CHECK(ws.alloc(&block_sums, nb));
    MXK_CHECK(ws.alloc(&offsets, nb));
    MXK_CHECK(ws.alloc(&total_dev, 1));
    MXK_CHECK(ws.alloc(&selected, n));
    MXK_CHECK(ws.alloc(&idx_dev, 1));
    MXK_CHECK(ws.alloc(&slots, nb));
    fill_kernel<double><<<(unsigned)std::min<int64_t>(nb, 4096), kInitBlock, 0, stream>>>(
        dist, n, std::numeric_limits<double>::infinity());
    MXK_CUDA(cudaGetLastError());
    MXK_CUDA(cudaMemsetAsync(selected, 0, (size_t)n, stream));

    std::mt19937 generator(seed);
    int64_t next = std::uniform_int_distribution<int>(0, (int)(n - 1))(generator);
    // gamma_m for m = n + 64 roundings along any prefix (sequential: n - 1; the
    // parallel scan: far fewer nonzero additions, plus one subtraction)
    const double u = std::ldexp(1.0, -53);
    const double m = (double)n + 64.0;
    const double gamma = m * u / (1.0 - m * u);
    std::vector<double> host_dist;  // only for the exact fallback
    const size_t smem = sizeof(double) * (size_t)d;
    for (int c = 0; c < k; ++c) {
        float* crow = centroids + (size_t)c * d;
        MXK_CUDA(cudaMemcpyAsync(crow, points + next * d, sizeof(float) * (size_t)d, cudaMemcpyDeviceToDevice, stream));
        MXK_CUDA(cudaMemsetAsync(selected + next, 1, 1, stream));
        {
            LaunchScope scope("init_kmeanspp_dist", stream);
            kpp_dist_kernel<<<(unsigned)nb, kInitBlock, smem, stream>>>(n, d, points, crow, selected, dist, block_sums);
            MXK_CUDA(cudaGetLastError());
        }
        if (c + 1 == k) break;
        {
            LaunchScope scope("init_kmeanspp_scan", stream);
            kpp_scan_kernel<<<1, 1024, 0, stream>>>((int)nb, block_sums, offsets, total_dev);
            MXK_CUDA(cudaGetLastError());
        }
        double total_p = 0.0;
        MXK_CUDA(cudaMemcpyAsync(&total_p, total_dev, sizeof(double), cudaMemcpyDeviceToHost, stream));
        MXK_CUDA(cudaStreamSynchronize(stream));
        // total > 0 exactly when some distance is > 0, for the parallel sum as for
        // the sequential one (nonnegative terms)
        next = -1;
        bool exact = !std::isfinite(total_p);
        double draw = 0.0;
        if (total_p > 0.0) {
            draw = std::generate_canonical<double, std::numeric_limits<double>::digits>(generator);
            if (!exact) {
                const double delta = 2.02 * gamma * total_p;      // bound on |S - P| for every prefix
                const double lo_t = draw * (total_p - delta) * (1.0 - 4 * u);
                const double hi_t = draw * (total_p + delta) * (1.0 + 4 * u);
                const double t_mid = draw * total_p;
                const unsigned long long none = ~0ull;
                MXK_CUDA(cudaMemcpyAsync(idx_dev, &none, sizeof(none), cudaMemcpyHostToDevice, stream));
                {
                    LaunchScope scope("init_kmeanspp_find", stream);
                    kpp_find_kernel<<<(unsigned)nb, kInitBlock, 0, stream>>>(n, dist, offsets, t_mid, idx_dev, slots);
                    MXK_CUDA(cudaGetLastError());
                }
                unsigned long long cand = none;
                MXK_CUDA(cudaMemcpyAsync(&cand, idx_dev, sizeof(cand), cudaMemcpyDeviceToHost, stream));
                MXK_CUDA(cudaStreamSynchronize(stream));
                if (cand != none) {
                    double2 pv;
                    MXK_CUDA(cudaMemcpyAsync(&pv, slots + cand / kInitBlock, sizeof(pv), cudaMemcpyDeviceToHost,
                                             stream));
                    MXK_CUDA(cudaStreamSynchronize(stream));
                    // The sequential sum crosses the target exactly here if the prefix
                    // before the candidate stays at or below it and the one through it
                    // stays above it, for every admissible sum and target (outward
                    // rounding margins on both sides).
                    const double above = pv.y * (1.0 - 4 * u) - delta * (1.0 + 4 * u);
                    const double below = (pv.x + delta) * (1.0 + 4 * u);
                    if (above > hi_t && (cand == 0 || below <= lo_t)) next = (int64_t)cand;
                    else exact = true;
                } else {
                    exact = true;
                }
            }
            if (exact) {
                // the reference's sequential loop on the same distances
                host_dist.resize((size_t)n);
                MXK_CUDA(cudaMemcpyAsync(host_dist.data(), dist, sizeof(double) * (size_t)n, cudaMemcpyDeviceToHost,
                                         stream));
                MXK_CUDA(cudaStreamSynchronize(stream));
                double total = 0.0;
                for (int64_t p = 0; p < n; ++p) total += host_dist[(size_t)p];
                const double target = draw * (total - 0.0) + 0.0;
                double cumulative = 0.0;
                for (int64_t p = 0; p < n; ++p) {
                    cumulative += host_dist[(size_t)p];
                    // selected points have distance 0, so "distance > 0" implies "not selected"
                    if (host_dist[(size_t)p] > 0.0 && cumulative > target) {
                        next = p;
                        break;
                    }
                }
            }
        }
        if (next < 0) {  // every remaining point duplicates a center, or rounding at the end of the sum
            const unsigned long long none = ~0ull;
            MXK_CUDA(cudaMemcpyAsync(idx_dev, &none, sizeof(none), cudaMemcpyHostToDevice, stream));
            kpp_first_free_kernel<<<(unsigned)std::min<int64_t>(nb, 4096), kInitBlock, 0, stream>>>(n, selected,
                                                                                                   idx_dev);
            MXK_CUDA(cudaGetLastError());
            unsigned long long cand = none;
            MXK_CUDA(cudaMemcpyAsync(&cand, idx_dev, sizeof(cand), cudaMemcpyDeviceToHost, stream));
            MXK_CUDA(cudaStreamSynchronize(stream));
            if (cand == none) return fail(MXK_ERR_INVALID, "init: no point left to choose");
            next = (int64_t)cand;
        }
    }
    MXK_CUDA(cudaStreamSynchronize(stream));
    return MXK_OK;
}

}  // namespace mxk

extern "C" {

int mxk_init_farthest(int64_t n, int d, int k, const float* points, float* centroids, void* stream) {
    mxk::clear_error();
    return mxk::run_init_farthest(n, d, k, points, centroids, mxk::as_stream(stream));
}

int mxk_init_kmeanspp(int64_t n, int d, int k, const float* points, float* centroids, uint32_t seed, void* stream) {
    mxk::clear_error();
    return mxk::run_init_kmeanspp(n, d, k, points, centroids, seed, mxk::as_stream(stream));
}

}  // extern "C"
