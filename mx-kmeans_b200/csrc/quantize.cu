// K1: MX quantization of point and centroid rows, plus the per-run point error
// bounds, the precision policy and the per-precision compaction of point ids.
//
// Reference: ParCIS/MX-KMeans src/kernels/quantize.cu (quantize_kernel :13-72,
// point_bounds_kernel :74-98, precision_kernel :100-108, launchers :111-134),
// src/kernels/assignment.cu:7-16 (norms) and src/kmeans.cu:36-52 (centroid
// statistics and group compaction).
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"
#include "mx_codec.cuh"
#include "precision.hpp"

namespace mxk {
namespace {

constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ float4 ldg4(const float* p) {
    float4 v;
    asm volatile("ld.global.nc.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
    return v;
}

// One thread owns 16 consecutive features of one output row: four 128-bit loads
// in, one 128-bit (MXFP8), 96-bit (MXFP6) or 64-bit (MXFP4) store out.  The two
// threads of a 32-feature block combine their maxima with one shuffle, derive the
// UE8M0 scale exactly as the reference (Scale(amax/qmax) or 1 when amax == 0),
// and multiply by the exact reciprocal of the scale.
template <int BITS>
__device__ __forceinline__ void quantize_chunk(int64_t g, int64_t total, int chunks, int d,
                                               const float* __restrict__ points, const int* __restrict__ pid,
                                               uint8_t* __restrict__ values, uint8_t* __restrict__ scales,
                                               float* __restrict__ errors, int atom_rows) {
    const bool valid = g < total;
    const int64_t row = valid ? g / chunks : 0;
    const int chunk = valid ? (int)(g - row * chunks) : 0;
    float x[16];
    if (valid) {
        const int64_t src = pid ? (int64_t)pid[row] : row;
        const float* p = points + src * d + chunk * 16;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float4 v = ldg4(p + 4 * i);
            x[4 * i] = v.x, x[4 * i + 1] = v.y, x[4 * i + 2] = v.z, x[4 * i + 3] = v.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) x[i] = 0.0f;
    }
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(x[i]));
    amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, 1));
    constexpr float qmax = BITS == 8 ? 448.0f : (BITS == 6 ? 7.5f : 6.0f);
    const uint32_t s = dev::ue8m0_encode(amax > 0.0f ? amax / qmax : 1.0f);
    const float rcp = dev::ue8m0_reciprocal(s);
    const float sval = dev::ue8m0_value(s);

    uint32_t code[16];
    if constexpr (BITS == 8) {
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
            const uint32_t two = dev::e4m3x2_encode(x[i] * rcp, x[i + 1] * rcp);
            code[i] = two & 0xffu;
            code[i + 1] = two >> 8;
        }
    } else if constexpr (BITS == 6) {
#pragma unroll
        for (int i = 0; i < 16; ++i) code[i] = dev::e2m3_encode(x[i] * rcp);
    } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) code[i] = dev::e2m1_encode(x[i] * rcp);
    }

    float err = 0.0f;
    if (errors) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            float q;
            if constexpr (BITS == 8)
                q = dev::e4m3_decode(code[i]);
            else if constexpr (BITS == 6)
                q = dev::e2m3_decode(code[i]);
            else
                q = dev::e2m1_decode(code[i]);
            const float diff = x[i] - q * sval;
            err = fmaxf(err, diff * diff);
        }
        err = fmaxf(err, __shfl_xor_sync(kFull, err, 1));
    }
    if (!valid) return;

    const int64_t elem = row * d + chunk * 16;
    if constexpr (BITS == 8) {
        uint4 w;
        w.x = code[0] | (code[1] << 8) | (code[2] << 16) | (code[3] << 24);
        w.y = code[4] | (code[5] << 8) | (code[6] << 16) | (code[7] << 24);
        w.z = code[8] | (code[9] << 8) | (code[10] << 16) | (code[11] << 24);
        w.w = code[12] | (code[13] << 8) | (code[14] << 16) | (code[15] << 24);
        *reinterpret_cast<uint4*>(values + elem) = w;
    } else if constexpr (BITS == 6) {
        // Four 6-bit codes in three bytes, least significant bit first
        // (quantize.cu:53-62): a 24-bit group c0 | c1<<6 | c2<<12 | c3<<18.
        uint32_t g24[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
            g24[j] = (code[4 * j] & 63u) | ((code[4 * j + 1] & 63u) << 6) | ((code[4 * j + 2] & 63u) << 12) |
                     ((code[4 * j + 3] & 63u) << 18);
        uint32_t* out = reinterpret_cast<uint32_t*>(values + (elem / 4) * 3);
        out[0] = g24[0] | (g24[1] << 24);
        out[1] = (g24[1] >> 8) | (g24[2] << 16);
        out[2] = (g24[2] >> 16) | (g24[3] << 8);
    } else {
        // Low nibble = even feature (quantize.cu:48-51).
        uint2 w;
        w.x = (code[0] & 15u) | ((code[1] & 15u) << 4) | ((code[2] & 15u) << 8) | ((code[3] & 15u) << 12) |
              ((code[4] & 15u) << 16) | ((code[5] & 15u) << 20) | ((code[6] & 15u) << 24) | ((code[7] & 15u) << 28);
        w.y = (code[8] & 15u) | ((code[9] & 15u) << 4) | ((code[10] & 15u) << 8) | ((code[11] & 15u) << 12) |
              ((code[12] & 15u) << 16) | ((code[13] & 15u) << 20) | ((code[14] & 15u) << 24) |
              ((code[15] & 15u) << 28);
        *reinterpret_cast<uint2*>(values + elem / 2) = w;
    }
    if ((chunk & 1) == 0) {
        if (atom_rows)
            scales[dev::scale_atom_offset(row, chunk >> 1, d >> 7, atom_rows)] = (uint8_t)s;
        else
            scales[row * (d >> 5) + (chunk >> 1)] = (uint8_t)s;
        // Squared errors are non-negative, so integer order equals float order.
        if (errors) atomicMax(reinterpret_cast<unsigned*>(errors + row), __float_as_uint(err));
    }
}

template <int BITS>
__global__ void __launch_bounds__(256) quantize_kernel(int64_t rows, int d, const float* __restrict__ points,
                                                       const int* __restrict__ pid, uint8_t* __restrict__ values,
                                                       uint8_t* __restrict__ scales, float* __restrict__ errors,
                                                       const int* __restrict__ rows_dev, int atom_rows) {
    const int64_t nrows = rows_dev ? (int64_t)*rows_dev : rows;
    const int chunks = d >> 4;
    const int64_t total = nrows * chunks;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;  // multiple of 32: block pairs stay in one warp
    for (int64_t base = (int64_t)blockIdx.x * blockDim.x; base < total; base += stride) {
        quantize_chunk<BITS>(base + threadIdx.x, total, chunks, d, points, pid, values, scales, errors, atom_rows);
    }
}

// Sequential FMA sum of squares per row (assignment.cu:7-16: nvcc contracts
// `sum += x * x`), staged through shared memory so global loads coalesce.
__global__ void __launch_bounds__(256) l2_norm_kernel(int64_t rows, int d, const float* __restrict__ x,
                                                      float* __restrict__ norms) {
    __shared__ float tile[8][32][33];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row0 = ((int64_t)blockIdx.x * 8 + warp) * 32;
    if (row0 >= rows) return;
    float sum = 0.0f;
    for (int f0 = 0; f0 < d; f0 += 32) {
        const int f = f0 + lane;
#pragma unroll 8
        for (int r = 0; r < 32; ++r) {
            const int64_t row = row0 + r;
            tile[warp][r][lane] = (row < rows && f < d) ? x[row * d + f] : 0.0f;
        }
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 32; ++j) sum = fmaf(tile[warp][lane][j], tile[warp][lane][j], sum);
        __syncwarp();
    }
    if (row0 + lane < rows) norms[row0 + lane] = sum;
}

// The same sums for many rows of d % 128 == 0 features, 16-byte aligned: a warp
// stages 32 consecutive rows, 128 features at a time (one 512-byte row chunk
// per load, all 32 in flight), in shared memory with a 528-byte row pitch
// (16-byte stores and loads both conflict-free), then each lane walks its own
// row in feature order.
constexpr int kNormPitch = 132;  // floats per staged row
__global__ void __launch_bounds__(64) norm_rows_staged_kernel(int64_t rows, int d, const float* __restrict__ x,
                                                              float* __restrict__ norms) {
    __shared__ __align__(16) float tile[2][32][kNormPitch];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row0 = ((int64_t)blockIdx.x * 2 + w) * 32;
    if (row0 >= rows) return;
    float(*t)[kNormPitch] = tile[w];
    float sum = 0.0f;
    for (int c = 0; c < d; c += 128) {
#pragma unroll
        for (int r = 0; r < 32; ++r) {
            const int64_t row = row0 + r;
            const float4 v = row < rows ? __ldg(reinterpret_cast<const float4*>(x + row * d + c) + lane)
                                        : make_float4(0.f, 0.f, 0.f, 0.f);
            *reinterpret_cast<float4*>(&t[r][4 * lane]) = v;
        }
        __syncwarp();
        const float4* own = reinterpret_cast<const float4*>(t[lane]);
#pragma unroll 8
        for (int q = 0; q < 32; ++q) {
            const float4 v = own[q];
            sum = fmaf(v.x, v.x, sum);
            sum = fmaf(v.y, v.y, sum);
            sum = fmaf(v.z, v.z, sum);
            sum = fmaf(v.w, v.w, sum);
        }
        __syncwarp();
    }
    const int64_t my = row0 + lane;
    if (my < rows) norms[my] = sum;
}

// The same sums for a few rows (the centroids, every iteration): one thread per
// row, its features read as 128-bit loads, all in flight at once, and
// accumulated in feature order as above.  d % 4 == 0, rows 16-byte aligned.
__global__ void __launch_bounds__(64) l2_norm_rows_kernel(int64_t rows, int d, const float* __restrict__ x,
                                                          float* __restrict__ norms) {
    const int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= rows) return;
    const float4* xr = reinterpret_cast<const float4*>(x + row * d);
    float sum = 0.0f;
#pragma unroll 8
    for (int f = 0; f < d / 4; ++f) {
        const float4 v = __ldg(xr + f);
        sum = fmaf(v.x, v.x, sum);
        sum = fmaf(v.y, v.y, sum);
        sum = fmaf(v.z, v.z, sum);
        sum = fmaf(v.w, v.w, sum);
    }
    norms[row] = sum;
}

// One thread per point, one 32-feature block at a time (eight 128-bit loads of
// the block's contiguous 128 bytes): block maximum, the FP4 (E2M1) and FP6 (E3M2,
// as the reference) scales, and the reconstruction errors of features 1..31
// (quantize.cu:74-98: feature 0 of each block is skipped, an exact max either way).
__global__ void __launch_bounds__(256) point_bounds_kernel(int64_t n, int d, const float* __restrict__ points,
                                                           const float* __restrict__ norms, float* __restrict__ upper) {
    const int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (p >= n) return;
    const float* row = points + p * d;
    float e4 = 0.0f, e6 = 0.0f;
    for (int base = 0; base < d; base += 32) {
        float x[32];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 v = ldg4(row + base + 4 * i);
            x[4 * i] = v.x, x[4 * i + 1] = v.y, x[4 * i + 2] = v.z, x[4 * i + 3] = v.w;
        }
        float amax = 0.0f;
#pragma unroll
        for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(x[j]));
        const uint32_t s4 = dev::ue8m0_encode(amax > 0.0f ? amax / 6.0f : 1.0f);
        const uint32_t s6 = dev::ue8m0_encode(amax > 0.0f ? amax / 7.5f : 1.0f);
        const float r4 = dev::ue8m0_reciprocal(s4), r6 = dev::ue8m0_reciprocal(s6);
        const float v4 = dev::ue8m0_value(s4), v6 = dev::ue8m0_value(s6);
#pragma unroll
        for (int j = 1; j < 32; ++j) {
            const float q4 = dev::e2m1_round_trip(x[j] * r4);
            const float q6 = dev::e3m2_round_trip(x[j] * r6);
            e4 = fmaxf(e4, fabsf(fmaf(q4, v4, -x[j])));
            e6 = fmaxf(e6, fabsf(fmaf(q6, v6, -x[j])));
        }
    }
    const size_t tile = (size_t)(p / 32) * 96;
    const int slot = (int)(p % 32);
    const float nrm = norms[p];
    upper[tile + slot] = nrm;
    upper[tile + 32 + slot] = fmaf((float)d * e6, e6, nrm);
    upper[tile + 64 + slot] = fmaf((float)d * e4, e4, nrm);
}

__global__ void __launch_bounds__(256) precision_kernel(int64_t n, int d, const float* __restrict__ upper,
                                                        const float* __restrict__ gaps, float lc, float ec,
                                                        const float* __restrict__ lc_ec_dev, int* __restrict__ precision,
                                                        int* __restrict__ group_counts, int policy) {
    const int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (lc_ec_dev) {
        ec = lc_ec_dev[0];
        lc = lc_ec_dev[1];
    }
    int prec = 0;
    if (p < n) {
        const size_t tile = (size_t)(p / 32) * 96;
        const int slot = (int)(p % 32);
        // policy 0: the reference's select_precision; 1: the candidate it discards
        prec = policy ? precision_candidate(upper[tile + 64 + slot], upper[tile + 32 + slot], lc, d, gaps[p])
                      : select_precision(upper[tile + 64 + slot], upper[tile + 32 + slot], lc, ec, d, gaps[p]);
        precision[p] = prec;
    }
    if (group_counts) {
        const int lane = threadIdx.x & 31;
#pragma unroll
        for (int g = 0; g < 3; ++g) {
            const unsigned m = __ballot_sync(kFull, p < n && prec == 4 + 2 * g);
            if (m && lane == __ffs(m) - 1) atomicAdd(group_counts + g, __popc(m));
        }
    }
}

__global__ void centroid_stats_kernel(int k, const float* __restrict__ errors, const float* __restrict__ norms,
                                      float* __restrict__ stats) {
    __shared__ float se[32], sn[32];
    float me = 0.0f, mn = 0.0f;
    for (int i = threadIdx.x; i < k; i += blockDim.x) {
        me = fmaxf(me, errors[i]);
        mn = fmaxf(mn, norms[i]);
    }
    for (int o = 16; o; o >>= 1) {
        me = fmaxf(me, __shfl_xor_sync(kFull, me, o));
        mn = fmaxf(mn, __shfl_xor_sync(kFull, mn, o));
    }
    if ((threadIdx.x & 31) == 0) se[threadIdx.x >> 5] = me, sn[threadIdx.x >> 5] = mn;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) me = fmaxf(me, se[w]), mn = fmaxf(mn, sn[w]);
        stats[0] = sqrtf(me);
        stats[1] = sqrtf(mn);
    }
}

// ---- stable three-way compaction (thrust::copy_if per group, kmeans.cu:46-50)
constexpr int kCompactBlock = 1024;  // elements per block (256 threads x 4)

// Element i of the sequence is point order[i] (or i without an order), so the
// groups come out in the sequence's order -- ascending point index like the
// reference's copy_if, or label-sorted when the driver passes that order.
__global__ void __launch_bounds__(256) group_block_count_kernel(int64_t n, const int* __restrict__ precision,
                                                                const int* __restrict__ order,
                                                                int* __restrict__ block_counts, int nblocks,
                                                                const int* __restrict__ stop) {
    if (stop && *stop) return;  // the Lloyd loop has already converged
    __shared__ int cnt[3];
    if (threadIdx.x < 3) cnt[threadIdx.x] = 0;
    __syncthreads();
    int local[3] = {0, 0, 0};
    const int64_t base = (int64_t)blockIdx.x * kCompactBlock;
    for (int i = threadIdx.x; i < kCompactBlock; i += blockDim.x) {
        const int64_t i_seq = base + i;
        if (i_seq < n) {
            const int v = precision[order ? (int64_t)order[i_seq] : i_seq];
            local[0] += v == 4, local[1] += v == 6, local[2] += v == 8;
        }
    }
    for (int g = 0; g < 3; ++g) {
        int v = local[g];
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
        if ((threadIdx.x & 31) == 0 && v) atomicAdd(&cnt[g], v);
    }
    __syncthreads();
    if (threadIdx.x < 3) block_counts[threadIdx.x * nblocks + blockIdx.x] = cnt[threadIdx.x];
}

// Exclusive scan of per-block counts for each group (one block, three warps).
__global__ void group_scan_kernel(int* __restrict__ block_counts, int nblocks, int* __restrict__ group_counts,
                                  const int* __restrict__ stop) {
    const int g = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (g >= 3) return;
    if (stop && *stop) {  // converged: empty groups, so the quantize and GEMM launches that read them do nothing
        if (lane == 0) group_counts[g] = 0;
        return;
    }
    int* c = block_counts + (size_t)g * nblocks;
    int carry = 0;
    for (int b0 = 0; b0 < nblocks; b0 += 32) {
        const int b = b0 + lane;
        const int v = b < nblocks ? c[b] : 0;
        int incl = v;
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(kFull, incl, o);
            if (lane >= o) incl += t;
        }
        if (b < nblocks) c[b] = carry + incl - v;
        carry += __shfl_sync(kFull, incl, 31);
    }
    if (lane == 0) group_counts[g] = carry;
}

__global__ void __launch_bounds__(256) group_scatter_kernel(int64_t n, const int* __restrict__ precision,
                                                            const int* __restrict__ order,
                                                            const int* __restrict__ block_offsets, int nblocks,
                                                            int* __restrict__ ids, const int* __restrict__ stop) {
    if (stop && *stop) return;
    __shared__ int warp_tot[3][8];
    __shared__ int running[3];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x < 3) running[threadIdx.x] = block_offsets[threadIdx.x * nblocks + blockIdx.x];
    __syncthreads();
    const int64_t base = (int64_t)blockIdx.x * kCompactBlock;
    for (int i0 = 0; i0 < kCompactBlock; i0 += 256) {
        const int64_t i_seq = base + i0 + threadIdx.x;
        const int64_t p = i_seq < n ? (order ? (int64_t)order[i_seq] : i_seq) : 0;
        const int v = i_seq < n ? precision[p] : 0;
        unsigned m[3];
        for (int g = 0; g < 3; ++g) {
            m[g] = __ballot_sync(kFull, v == 4 + 2 * g);
            if (lane == 0) warp_tot[g][warp] = __popc(m[g]);
        }
        __syncthreads();
        for (int g = 0; g < 3; ++g) {
            if (v == 4 + 2 * g) {
                int off = running[g];
                for (int w = 0; w < warp; ++w) off += warp_tot[g][w];
                off += __popc(m[g] & ((1u << lane) - 1u));
                ids[(int64_t)g * n + off] = (int)p;
            }
        }
        __syncthreads();
        if (threadIdx.x < 3) {
            int t = 0;
            for (int w = 0; w < 8; ++w) t += warp_tot[threadIdx.x][w];
            running[threadIdx.x] += t;
        }
        __syncthreads();
    }
}

bool aligned(const void* p, int bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) == 0; }

}  // namespace

int launch_quantize(int bits, int64_t rows, int d, const float* points, const int* pid, void* values,
                    uint8_t* scales, float* max_errors, const int* rows_dev, cudaStream_t stream, int atom_rows,
                    const char* name) {
    if (bits != 4 && bits != 6 && bits != 8) return fail(MXK_ERR_INVALID, "Precision must be 4, 6, or 8");
    if (rows <= 0) return MXK_OK;
    MXK_REQUIRE(d > 0 && d % 32 == 0, "quantize_rows: d must be a positive multiple of 32");
    MXK_REQUIRE(atom_rows >= 0, "quantize_rows: negative atom tile height");
    MXK_REQUIRE(!atom_rows || d % 128 == 0, "quantize_rows: the scale-atom layout needs d % 128 == 0");
    MXK_REQUIRE(points && values && scales, "quantize_rows: null pointer");
    MXK_REQUIRE(aligned(points, 16), "quantize_rows: points must be 16-byte aligned");
    MXK_REQUIRE(aligned(values, bits == 8 ? 16 : (bits == 4 ? 8 : 4)),
                "quantize_rows: values must be aligned to the packed store width");
    const int64_t threads = rows * (d / 16);
    int64_t blocks = (threads + 255) / 256;
    const int64_t cap = (int64_t)sm_count() * 16;  // grid-stride beyond 16 CTAs per SM
    if (blocks > cap) blocks = cap;
    auto* out = static_cast<uint8_t*>(values);
    LaunchScope scope(name, stream);
    switch (bits) {
        case 8: quantize_kernel<8><<<(unsigned)blocks, 256, 0, stream>>>(rows, d, points, pid, out, scales, max_errors, rows_dev, atom_rows); break;
        case 6: quantize_kernel<6><<<(unsigned)blocks, 256, 0, stream>>>(rows, d, points, pid, out, scales, max_errors, rows_dev, atom_rows); break;
        default: quantize_kernel<4><<<(unsigned)blocks, 256, 0, stream>>>(rows, d, points, pid, out, scales, max_errors, rows_dev, atom_rows); break;
    }
    MXK_CUDA(cudaGetLastError());
    return MXK_OK;
}

int launch_l2_norm(int64_t rows, int d, const float* x, float* norms, cudaStream_t stream) {
    if (rows <= 0) return MXK_OK;
    MXK_REQUIRE(d > 0 && x && norms, "compute_l2_norm: bad arguments");
    LaunchScope scope("l2_norm", stream);
    const bool aligned = reinterpret_cast<uintptr_t>(x) % 16 == 0;
    if (rows <= 65536 && d % 4 == 0 && aligned) {
        // few rows: spread them over the SMs, one per thread
        l2_norm_rows_kernel<<<(unsigned)((rows + 63) / 64), 64, 0, stream>>>(rows, d, x, norms);
    } else if (d % 128 == 0 && aligned) {
        norm_rows_staged_kernel<<<(unsigned)((rows + 63) / 64), 64, 0, stream>>>(rows, d, x, norms);
    } else {
        const int64_t blocks = (rows + 255) / 256;
        l2_norm_kernel<<<(unsigned)blocks, 256, 0, stream>>>(rows, d, x, norms);
    }
    MXK_CUDA(cudaGetLastError());
    return MXK_OK;
}

int launch_point_bounds(int64_t n, int d, const float* points, const float* norms, float* upper,
                        cudaStream_t stream) {
    if (n <= 0) return MXK_OK;
    MXK_REQUIRE(d > 0 && d % 32 == 0, "precompute_point_bounds: d must be a multiple of 32");
    MXK_REQUIRE(reinterpret_cast<uintptr_t>(points) % 16 == 0, "precompute_point_bounds: points must be 16-byte aligned");
    const int64_t blocks = (n + 255) / 256;
    LaunchScope scope("point_bounds", stream);
    point_bounds_kernel<<<(unsigned)blocks, 256, 0, stream>>>(n, d, points, norms, upper);
    MXK_CUDA(cudaGetLastError());
    return MXK_OK;
}

int launch_assign_precisions(int64_t n, int d, const float* upper, const float* gaps, float lc, float ec,
                             const float* lc_ec_dev, int* precision, int* group_counts, cudaStream_t stream,
                             int policy) {
    if (n <= 0) return MXK_OK;
    const int64_t blocks = (n + 255) / 256;
    LaunchScope scope("assign_precisions", stream);
    precision_kernel<<<(unsigned)blocks, 256, 0, stream>>>(n, d, upper, gaps, lc, ec, lc_ec_dev, precision,
                                                          group_counts, policy);
    MXK_CUDA(cudaGetLastError());
    return MXK_OK;
}

int launch_centroid_stats(int k, const float* errors, const float* norms, float* stats, cudaStream_t stream) {
    LaunchScope scope("centroid_stats", stream);
    centroid_stats_kernel<<<1, 1024, 0, stream>>>(k, errors, norms, stats);
    MXK_CUDA(cudaGetLastError());
    return MXK_OK;
}

int64_t compaction_scratch_ints(int64_t n) { return 3 * ((n + kCompactBlock - 1) / kCompactBlock) + 3; }

int launch_group_compaction(int64_t n, const int* precision, const int* order, int* ids, int* group_counts,
                            int* scratch, cudaStream_t stream, const int* stop) {
    if (n <= 0) return MXK_OK;
    const int64_t nb = (n + kCompactBlock - 1) / kCompactBlock;
    MXK_REQUIRE(nb < (1ll << 31), "compaction: too many points");
    {
        LaunchScope scope("group_count", stream);
        group_block_count_kernel<<<(unsigned)nb, 256, 0, stream>>>(n, precision, order, scratch, (int)nb, stop);
        MXK_CUDA(cudaGetLastError());
    }
    {
        LaunchScope scope("group_scan", stream);
        group_scan_kernel<<<1, 96, 0, stream>>>(scratch, (int)nb, group_counts, stop);
        MXK_CUDA(cudaGetLastError());
    }
    {
        LaunchScope scope("group_scatter", stream);
        group_scatter_kernel<<<(unsigned)nb, 256, 0, stream>>>(n, precision, order, scratch, (int)nb, ids, stop);
        MXK_CUDA(cudaGetLastError());
    }
    return MXK_OK;
}

// Rows of an MXFP8 matrix (packed values, row-major scales) copied in the order
// pid into contiguous rows, with the scales rewritten in the atom layout of
// kPointTileRows-row tiles (what the GEMM bulk-copies).  One thread per 16
// bytes of values; the first d / 128 threads of a row also move its scale words.
__global__ void __launch_bounds__(256) gather_mxfp8_rows_kernel(int64_t rows, int d, const uint8_t* __restrict__ src,
                                                                const uint8_t* __restrict__ src_scales,
                                                                const int* __restrict__ pid,
                                                                uint8_t* __restrict__ dst,
                                                                uint8_t* __restrict__ dst_scales,
                                                                const int* __restrict__ stop) {
    if (stop && *stop) return;
    const int pieces = d >> 4;
    const int64_t total = rows * pieces;
    for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = g / pieces;
        const int piece = (int)(g - row * pieces);
        const int64_t from = pid ? (int64_t)pid[row] : row;
        reinterpret_cast<uint4*>(dst + row * d)[piece] = reinterpret_cast<const uint4*>(src + from * d)[piece];
        if (piece < (d >> 7)) {  // the four block scales of 128-feature chunk `piece`
            const uint32_t w = reinterpret_cast<const uint32_t*>(src_scales + from * (d >> 5))[piece];
            *reinterpret_cast<uint32_t*>(dst_scales + dev::scale_atom_offset(row, 4 * piece, d >> 7, kPointTileRows)) = w;
        }
    }
}

int launch_gather_mxfp8_rows(int64_t rows, int d, const uint8_t* src, const uint8_t* src_scales, const int* pid,
                             uint8_t* dst, uint8_t* dst_scales, const int* stop, cudaStream_t stream) {
    if (rows <= 0) return MXK_OK;
    MXK_REQUIRE(d % 128 == 0, "gather_mxfp8_rows: d must be a multiple of 128");
    const int64_t total = rows * (d >> 4);
    const int64_t blocks = std::min<int64_t>((total + 255) / 256, (int64_t)sm_count() * 32);
    LaunchScope scope("gather_mxfp8_rows", stream);
    gather_mxfp8_rows_kernel<<<(unsigned)blocks, 256, 0, stream>>>(rows, d, src, src_scales, pid, dst, dst_scales,
                                                                   stop);
    MXK_CUDA(cudaGetLastError());
    return MXK_OK;
}

// Every float32 bit pattern through the division-free MXFP8 scale codec of the
// fused assignment's in-kernel quantizer and through the IEEE division it
// replaces (the rule quantize_rows applies); result[0] counts disagreements,
// result[1] keeps the smallest disagreeing pattern (all ones when none).
__global__ void __launch_bounds__(256) scale_codec_check_kernel(unsigned long long* __restrict__ result) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    unsigned long long bad = 0, first = ~0ull;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (1ull << 32); i += stride) {
        const float a = __uint_as_float((uint32_t)i);
        const uint32_t want = dev::ue8m0_encode(a > 0.0f ? a / 448.0f : 1.0f);
        if (dev::ue8m0_mxfp8_scale(a) != want) {
            ++bad;
            first = first < i ? first : i;
        }
    }
    if (bad) {
        atomicAdd(result, bad);
        atomicMin(result + 1, first);
    }
}

int launch_scale_codec_check(unsigned long long* result, cudaStream_t stream) {
    MXK_REQUIRE(result != nullptr, "check_mxfp8_scale_codec: result must not be null");
    MXK_CUDA(cudaMemsetAsync(result, 0, sizeof(unsigned long long), stream));
    MXK_CUDA(cudaMemsetAsync(result + 1, 0xff, sizeof(unsigned long long), stream));
    int sms = 0, dev = 0;
    MXK_CUDA(cudaGetDevice(&dev));
    MXK_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    LaunchScope scope("scale_codec_check", stream);
    scale_codec_check_kernel<<<(unsigned)(sms * 8), 256, 0, stream>>>(result);
    MXK_CUDA(cudaGetLastError());
    return MXK_OK;
}

}  // namespace mxk

extern "C" {

int mxk_compute_l2_norm(int64_t rows, int d, const float* points, float* norms, void* stream) {
    return mxk::launch_l2_norm(rows, d, points, norms, mxk::as_stream(stream));
}

int mxk_quantize_rows(int bits, int64_t rows, int d, const float* points, const int* pid, void* values,
                      uint8_t* scales, float* max_errors, void* stream) {
    return mxk::launch_quantize(bits, rows, d, points, pid, values, scales, max_errors, nullptr,
                                mxk::as_stream(stream), false);
}

int mxk_precompute_point_bounds(int64_t n, int d, const float* points, const float* norms, float* upper,
                                void* stream) {
    return mxk::launch_point_bounds(n, d, points, norms, upper, mxk::as_stream(stream));
}

int mxk_assign_precisions(int64_t n, int d, const float* upper, const float* gaps, float lc, float ec,
                          int* precision, void* stream) {
    return mxk::launch_assign_precisions(n, d, upper, gaps, lc, ec, nullptr, precision, nullptr,
                                         mxk::as_stream(stream));
}

int mxk_check_mxfp8_scale_codec(unsigned long long* result, void* stream) {
    return mxk::launch_scale_codec_check(result, mxk::as_stream(stream));
}

}  // extern "C"
