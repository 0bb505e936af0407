// Exact pruning of centroid tiles for the fused assignment GEMM.
//
// A Lloyd iteration assigns each point x to argmin_c d(x, c), where d is the
// MX distance fmaf(-2, D(x, c), |x|^2 + |c|^2) and D the tensor-core product of
// the MXFP8-quantized rows x^ and c^.  The GEMM need not multiply a
// 192-centroid tile against a 128-point tile when no point of the point tile can
// have its minimum there.  The test proves that from the previous iteration,
// working in the quantized space where the tensor core works:
//
// * d(x, c) = |x^ - c^|^2 + alpha_x + beta_c + rho, with the per-row constants
//   alpha_x = |x|^2 - |x^|^2 and beta_c = |c|^2 - |c^|^2 (the norms the GEMM
//   adds are those of the unquantized rows) and a rounding term
//   |rho| <= kappa (|x|^2 + |c|^2 + |x^|^2 + |c^|^2 + 2 |x^| |c^|) covering the
//   tensor core's FP32 accumulation (taken as <= 1.5e-5 of sum |x^_i c^_i|), the
//   fmaf, and the FP32 evaluation of alpha and beta.
// * Upper bound.  x's previous label a and previous distance d_prev (written by
//   the previous GEMM against c_a_old) give |x^ - c^_a_old| <= sqrt(d_prev -
//   alpha_x - beta_a_old + rho_old); with the quantized centroid's move
//   delta_a = |c^_a - c^_a_old|, r = that + delta_a >= |x^ - c^_a| and
//   U = r^2 + alpha_x + beta_a + rho >= d(x, c_a) >= the new minimum.
// * Lower bound.  For c in tile T, |x^ - c^| >= |c^ - c^_a| - r >= dmin(a, T) -
//   r (dmin: the smallest quantized distance from c^_a into T), so d(x, c) >=
//   max(0, dmin(a, T) - r)^2 + alpha_x + min_T beta - rho_T.  When that exceeds
//   U, no centroid of T can be x's nearest (nor tie with it): T is skipped.
//
// * Second-nearest bound (Hamerly's bound, in the same space).  The GEMM also
//   writes, per point, sec <= d(x, c_old) - beta_c_old for every centroid c
//   other than the label it chose (from its screened chunk minima, the exact
//   chunks, each less the largest beta of its 32 centroids, and the bounds of
//   the tiles the row's mask excluded).  So |x^ - c^_old|^2 >= sec - alpha_x -
//   rho_old, |x^ - c^| >= that root - max delta, and d(x, c) >= (that)^2 +
//   alpha_x + min beta - rho for every c != a: when that exceeds U the row
//   keeps its label without the per-tile test.  A row that leaves the GEMM gets
//   the smallest of its tiles' lower bounds (less beta) as its next sec.  Kept
//   free of beta, the bound loses only the centroids' movement and rounding
//   margins from one iteration to the next.
//
// A point tile computes the union of its rows' tiles (each row's own tile
// always among them).  Every bound is evaluated with outward margins well above
// the FP32 rounding of its own arithmetic, and any non-finite input keeps every
// tile.  The labels are those of the unpruned computation, bit for bit (tested
// by replaying iterations without a mask).
#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "kernels.cuh"
#include "mx_codec.cuh"

namespace mxk {
namespace {

constexpr int kMaxPruneTiles = 64;
// Pair-bound kernel: a CTA covers 64 centroids a against one 192-centroid
// tile T; 128 threads, each 8 rows x 12 columns of the FP32 Gram block,
// feature chunks of 32 staged in shared memory.
constexpr int kPairRows = 64;
constexpr int kPairCols = kCentroidTileRows;  // 192
constexpr int kPairChunk = 32;
constexpr int kPairThreads = 128;

// MXFP8 round trip of 4 consecutive features held by one lane; the 8 lanes of
// each 32-feature block share its scale (quantize_rows' arithmetic, the values
// the tensor core multiplies).
__device__ __forceinline__ float4 mxfp8_round_trip4(float4 x, int lane) {
    float amax = fmaxf(fmaxf(fmaxf(0.0f, fabsf(x.x)), fmaxf(fabsf(x.y), fabsf(x.z))), fabsf(x.w));
    for (int o = 1; o < 8; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    (void)lane;
    const uint32_t sc = dev::ue8m0_mxfp8_scale(amax);
    const float rcp = dev::ue8m0_reciprocal(sc), scale = dev::ue8m0_value(sc);
    auto rt = [&](float v) { return dev::e4m3_decode(dev::e4m3x2_encode(v * rcp, 0.0f) & 0xffu) * scale; };
    return make_float4(rt(x.x), rt(x.y), rt(x.z), rt(x.w));
}

__device__ __forceinline__ float warp_sum(float v) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Per centroid (one warp per row), in one pass over its row: the row's squared
// norm |c|^2 (the reference's sequential FP32 sum, compute_l2_norm: features in
// order, carried from lane to lane), its MXFP8 codes and UE8M0 scales (the
// bytes quantize_rows writes, scales in the GEMM's atom layout for 192-row
// tiles), the dequantized row c^ into chat, stats cst[a] = (beta = |c|^2 -
// |c^|^2, |c^|^2, |c|^2, |c^|), and delta[a] >= |c^_a - c^_a_old| (the previous
// centroids' round trip; +inf without prev).
__global__ void __launch_bounds__(256) centroid_prep_kernel(int k, int d, const float* __restrict__ c,
                                                            const float* __restrict__ prev, float* __restrict__ cn,
                                                            float* __restrict__ chat, float4* __restrict__ cst,
                                                            float* __restrict__ delta, uint8_t* __restrict__ qcent,
                                                            uint8_t* __restrict__ cscales,
                                                            const int* __restrict__ stop) {
    if (stop && *stop) return;
    const int lane = threadIdx.x & 31;
    const int a = (int)(((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    if (a >= k) return;  // warp-uniform
    const int kchunks = d >> 7;
    float norm = 0.0f, h = 0.0f, mv = 0.0f;
    for (int j = 4 * lane; j < d; j += 128) {
        const float4 x = __ldg(reinterpret_cast<const float4*>(c + (int64_t)a * d + j));
        // features j - 4 lane .. + 127 in order: lane L applies its four, then
        // hands the running sum to lane L + 1
#pragma unroll
        for (int L = 0; L < 32; ++L) {
            const float t = fmaf(x.w, x.w, fmaf(x.z, x.z, fmaf(x.y, x.y, fmaf(x.x, x.x, norm))));
            norm = __shfl_sync(0xffffffffu, t, L);
        }
        float amax = fmaxf(fmaxf(fmaxf(0.0f, fabsf(x.x)), fmaxf(fabsf(x.y), fabsf(x.z))), fabsf(x.w));
        for (int o = 1; o < 8; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const uint32_t sc = dev::ue8m0_mxfp8_scale(amax);
        const float rcp = dev::ue8m0_reciprocal(sc), scale = dev::ue8m0_value(sc);
        const uint32_t lo = dev::e4m3x2_encode(x.x * rcp, x.y * rcp);
        const uint32_t hi = dev::e4m3x2_encode(x.z * rcp, x.w * rcp);
        *reinterpret_cast<uint32_t*>(qcent + (int64_t)a * d + j) = (lo & 0xffffu) | (hi << 16);
        if ((lane & 7) == 0) cscales[dev::scale_atom_offset(a, j >> 5, kchunks, kCentroidTileRows)] = (uint8_t)sc;
        const float4 ch = make_float4(dev::e4m3_decode(lo & 0xffu) * scale, dev::e4m3_decode((lo >> 8) & 0xffu) * scale,
                                      dev::e4m3_decode(hi & 0xffu) * scale, dev::e4m3_decode((hi >> 8) & 0xffu) * scale);
        *reinterpret_cast<float4*>(chat + (int64_t)a * d + j) = ch;
        h = fmaf(ch.x, ch.x, fmaf(ch.y, ch.y, fmaf(ch.z, ch.z, fmaf(ch.w, ch.w, h))));
        if (prev) {
            const float4 oh =
                mxfp8_round_trip4(__ldg(reinterpret_cast<const float4*>(prev + (int64_t)a * d + j)), lane);
            const float t0 = ch.x - oh.x, t1 = ch.y - oh.y, t2 = ch.z - oh.z, t3 = ch.w - oh.w;
            mv = fmaf(t0, t0, fmaf(t1, t1, fmaf(t2, t2, fmaf(t3, t3, mv))));
        }
    }
    h = warp_sum(h);
    mv = warp_sum(mv);
    if (lane == 0) {
        const float rel = 1.0f + (float)(d + 8) * 1.2e-7f;  // rounding of an FP32 sum of d squares
        delta[a] = prev ? sqrtf(mv * rel) * (1.0f + 1e-6f) : __int_as_float(0x7f800000);
        cn[a] = norm;
        cst[a] = make_float4(norm - h, h, norm, sqrtf(h));
    }
}

// The stats of tile t over its centroids, by one whole block of kPairThreads
// threads: tst[t] = (min beta, max |c^|^2, max |c|^2, non-finite flag),
// tst[tiles + t] = (max beta, max delta (+inf for a non-finite one), the root of
// max |c^|^2, 0) and
// bmax32[c / 32] = the largest beta of each 32 consecutive centroids.
__device__ void tile_stats_block(int k, int t, int tiles, const float4* __restrict__ cst,
                                 const float* __restrict__ delta, float4* __restrict__ tst,
                                 float* __restrict__ bmax32) {
    static_assert(kPairCols % 32 == 0 && kPairThreads % 32 == 0, "32-centroid groups inside one warp");
    __shared__ float4 part[kPairThreads / 32];
    __shared__ float2 part2[kPairThreads / 32];
    const float inf = __int_as_float(0x7f800000);
    float4 m = make_float4(inf, 0.0f, 0.0f, 0.0f);
    float bmax = -inf, dmax = 0.0f;
    for (int j0 = 0; j0 < kPairCols; j0 += kPairThreads) {
        const int j = j0 + (int)threadIdx.x;
        const int b = t * kPairCols + j;
        const bool valid = j < kPairCols && b < k;
        float b32 = -inf;
        if (valid) {
            const float4 v = cst[b];
            m.x = fminf(m.x, v.x), m.y = fmaxf(m.y, v.y), m.z = fmaxf(m.z, v.z);
            if (!(fabsf(v.x) < inf && v.y < inf && v.z < inf)) m.w = 1.0f;  // a non-finite centroid: no pruning
            bmax = fmaxf(bmax, v.x);
            b32 = v.x;
            const float dv = delta[b];
            dmax = dv < inf ? fmaxf(dmax, dv) : inf;  // (NaN counts as infinite)
        }
        for (int o = 16; o; o >>= 1) b32 = fmaxf(b32, __shfl_xor_sync(0xffffffffu, b32, o));
        const int b0 = b - (int)(threadIdx.x & 31);  // the warp's first centroid
        if ((threadIdx.x & 31) == 0 && j < kPairCols && b0 < k) bmax32[b0 >> 5] = b32;
    }
    for (int o = 16; o; o >>= 1) {
        m.x = fminf(m.x, __shfl_xor_sync(0xffffffffu, m.x, o));
        m.y = fmaxf(m.y, __shfl_xor_sync(0xffffffffu, m.y, o));
        m.z = fmaxf(m.z, __shfl_xor_sync(0xffffffffu, m.z, o));
        m.w = fmaxf(m.w, __shfl_xor_sync(0xffffffffu, m.w, o));
        bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, o));
        dmax = fmaxf(dmax, __shfl_xor_sync(0xffffffffu, dmax, o));
    }
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = m, part2[threadIdx.x >> 5] = make_float2(bmax, dmax);
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < kPairThreads / 32; ++w) {
            const float4 o = part[w];
            m.x = fminf(m.x, o.x), m.y = fmaxf(m.y, o.y), m.z = fmaxf(m.z, o.z), m.w = fmaxf(m.w, o.w);
            bmax = fmaxf(bmax, part2[w].x), dmax = fmaxf(dmax, part2[w].y);
        }
        tst[t] = m;
        tst[tiles + t] = make_float4(bmax, dmax, sqrtf(m.y), 0.0f);
    }
}

// dmin[a * tiles + T]: a lower bound of min over c in T, c != a, of |c^ - c^_a|,
// from the Gram entries G_ab = <c^_a, c^_b> (FP32, each accumulated by fmaf in
// increasing feature order) and the quantized squared norms h = cst[].y:
// |c^_a - c^_b|^2 = h_a + h_b - 2 G_ab, less (d + 16) u' (h_a + h_b + 2 |c^_a|
// |c^_b|) for the rounding of the product, the norms and this sum; 0 when no
// finite bound exists.  The Gram block is reduced to its per-row minima in
// registers, so no K x K product is stored.  The first block of each tile
// column also writes the tile's stats (tile_stats_block).
__global__ void __launch_bounds__(kPairThreads) pair_bounds_kernel(int k, int d, int tiles, const float* __restrict__ chat,
                                                                   const float4* __restrict__ cst,
                                                                   const float* __restrict__ delta,
                                                                   float* __restrict__ dmin, float4* __restrict__ tst,
                                                                   float* __restrict__ bmax32,
                                                                   const int* __restrict__ stop) {
    if (stop && *stop) return;
    if (blockIdx.x == 0) tile_stats_block(k, blockIdx.y, tiles, cst, delta, tst, bmax32);
    __shared__ __align__(16) float As[kPairChunk][kPairRows];
    __shared__ __align__(16) float Bs[kPairChunk][kPairCols];
    __shared__ float hb_s[kPairCols], sb_s[kPairCols];
    const int tid = threadIdx.x;
    const int a0 = blockIdx.x * kPairRows, tile = blockIdx.y, b0 = tile * kPairCols;
    const int ty = tid >> 4, tx = tid & 15;  // rows 8 ty .. +8, columns 12 tx .. +12
    for (int j = tid; j < kPairCols; j += kPairThreads) {
        const int b = b0 + j;
        const float h = b < k ? cst[b].y : 0.0f;
        hb_s[j] = h;
        sb_s[j] = sqrtf(h);
    }
    float acc[8][12];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 12; ++j) acc[i][j] = 0.0f;
    for (int k0 = 0; k0 < d; k0 += kPairChunk) {
        __syncthreads();
        // rows fastest: consecutive threads store consecutive rows of a k line
        for (int idx = tid; idx < kPairRows * (kPairChunk / 4); idx += kPairThreads) {
            const int r = idx % kPairRows, q = idx / kPairRows;
            const int a = a0 + r;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (a < k) v = __ldg(reinterpret_cast<const float4*>(chat + (int64_t)a * d + k0 + 4 * q));
            As[4 * q][r] = v.x, As[4 * q + 1][r] = v.y, As[4 * q + 2][r] = v.z, As[4 * q + 3][r] = v.w;
        }
        for (int idx = tid; idx < kPairCols * (kPairChunk / 4); idx += kPairThreads) {
            const int r = idx % kPairCols, q = idx / kPairCols;
            const int b = b0 + r;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (b < k) v = __ldg(reinterpret_cast<const float4*>(chat + (int64_t)b * d + k0 + 4 * q));
            Bs[4 * q][r] = v.x, Bs[4 * q + 1][r] = v.y, Bs[4 * q + 2][r] = v.z, Bs[4 * q + 3][r] = v.w;
        }
        __syncthreads();
#pragma unroll 4
        for (int kk = 0; kk < kPairChunk; ++kk) {
            const float4 a_lo = *reinterpret_cast<const float4*>(&As[kk][8 * ty]);
            const float4 a_hi = *reinterpret_cast<const float4*>(&As[kk][8 * ty + 4]);
            const float4 b_0 = *reinterpret_cast<const float4*>(&Bs[kk][12 * tx]);
            const float4 b_1 = *reinterpret_cast<const float4*>(&Bs[kk][12 * tx + 4]);
            const float4 b_2 = *reinterpret_cast<const float4*>(&Bs[kk][12 * tx + 8]);
            const float av[8] = {a_lo.x, a_lo.y, a_lo.z, a_lo.w, a_hi.x, a_hi.y, a_hi.z, a_hi.w};
            const float bv[12] = {b_0.x, b_0.y, b_0.z, b_0.w, b_1.x, b_1.y, b_1.z, b_1.w, b_2.x, b_2.y, b_2.z, b_2.w};
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 12; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
    }
    const float rel = (float)(d + 16) * 1.2e-7f;
    const float inf = __int_as_float(0x7f800000);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int a = a0 + 8 * ty + i;
        const float ha = a < k ? cst[a].y : 0.0f;
        const float sa = sqrtf(ha);
        float m = inf;  // fminf skips NaN entries; all NaN leaves no bound
#pragma unroll
        for (int j = 0; j < 12; ++j) {
            const int c = 12 * tx + j, b = b0 + c;
            if (b < k && b != a) {
                const float hb = hb_s[c];
                const float d2 = ha + hb - 2.0f * acc[i][j];
                m = fminf(m, d2 - rel * (ha + hb + 2.0f * sa * sb_s[c]));
            }
        }
        for (int o = 8; o; o >>= 1) m = fminf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (tx == 0 && a < k) dmin[(int64_t)a * tiles + tile] = m < inf ? sqrtf(fmaxf(m, 0.0f)) * (1.0f - 1e-6f) : 0.0f;
    }
}

// Drift update of the pair bounds between two full computations: the quantized
// centroids moved by at most delta (|c^_new - c^_old|), so by the triangle
// inequality min over b in T of |c^_a - c^_b| shrinks by at most delta_a +
// max over b in T of delta_b.  dmin[a][T] is lowered by that (with a margin
// above the rounding of the two FP32 subtractions) and clamped at 0; a
// non-finite delta leaves no bound.  Blocks [0, tiles) write the tile stats.
__global__ void __launch_bounds__(kPairThreads) pair_drift_kernel(int k, int tiles, const float* __restrict__ delta,
                                                                  const float4* __restrict__ cst,
                                                                  float* __restrict__ dmin, float4* __restrict__ tst,
                                                                  float* __restrict__ bmax32,
                                                                  const int* __restrict__ stop) {
    if (stop && *stop) return;
    if ((int)blockIdx.x < tiles) {
        tile_stats_block(k, blockIdx.x, tiles, cst, delta, tst, bmax32);
        return;
    }
    __shared__ unsigned tmax[kMaxPruneTiles];  // per tile max delta (non-negative: integer order)
    for (int t = threadIdx.x; t < tiles; t += blockDim.x) tmax[t] = 0u;
    __syncthreads();
    for (int b = threadIdx.x; b < k; b += blockDim.x) {
        const float v = delta[b];
        atomicMax(&tmax[b / kPairCols], v == v ? __float_as_uint(v) : 0x7f800000u);  // NaN counts as infinite
    }
    __syncthreads();
    const int a = (blockIdx.x - tiles) * blockDim.x + threadIdx.x;
    if (a >= k) return;
    const float da = delta[a];
    const float inf = __int_as_float(0x7f800000);
    for (int t = 0; t < tiles; ++t) {
        float* p = dmin + (int64_t)a * tiles + t;
        const float x = *p, y = da, z = __uint_as_float(tmax[t]);
        const float v = (x - y - z) - 4e-7f * (x + y + z);
        *p = (v < inf && y < inf && z < inf) ? fmaxf(v, 0.0f) : 0.0f;  // (false for NaN: no bound)
    }
}

// The rounding term rho of the header comment for squared norms px, pc (of x and
// c) and hx2, hc2 (of x^ and c^), from pxh = px + hx2 and the roots shx =
// |x^|, shc = |c^|.
__device__ __forceinline__ float rho_bound(float pxh, float shx, float pc, float hc2, float shc, float kappa) {
    return kappa * (pxh + pc + hc2 + 2.0f * shx * shc);
}

// Square root by the hardware approximation (PTX sqrt.approx.f32, relative
// error a few units of 2^-23); every use below widens it by 4e-6, outward.
__device__ __forceinline__ float sqrt_approx(float x) {
    float r;
    asm("sqrt.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

// Whole-centroid-set terms of the second-nearest test, gathered from the tile
// stats: min beta, max |c^|^2, max |c|^2, max delta of the current centroids,
// max |c^|^2 and max |c|^2 of the previous ones, and the roots of the two
// max |c^|^2.
struct SetTerms {
    float bmin, hc2, pc, dmax, hc2_old, pc_old, shc, shc_old;
};

// One row of tile_mask_kernel: its centroid-tile mask m, whether it must stay
// in the GEMM (need), its GEMM record rb, and (compact, proven rows) its pinfo
// bounds for the next iteration.
__device__ __forceinline__ void row_tile_mask(int64_t row, int64_t rows, int k, int tiles, uint64_t all, float kappa,
                                              bool second, bool fresh, const SetTerms& gs,
                                              const int* __restrict__ prev_label,
                                              float4* __restrict__ pinfo, const float4* __restrict__ cst,
                                              const float4* __restrict__ cst_old, const float4* tcs,
                                              const float* __restrict__ delta, const float* __restrict__ dmin,
                                              float4* __restrict__ row_bound, int compact, uint64_t& m, bool& need) {
    const float inf = __int_as_float(0x7f800000);
    m = 0;
    need = false;
    if (row >= rows) return;
    // (bound on the row's nearest distance, its previous label, beta-free lower
    // bound of the tiles its mask excludes, the row's position as int bits) for
    // the GEMM's screen: (inf, label, inf, row) when no finite bound holds,
    // (inf, -1, inf, row) without a valid previous label
    float4 rb = make_float4(inf, __int_as_float(-1), inf, __int_as_float((int)row));
    const int a = prev_label[row];
    m = all;
    need = true;
    if ((unsigned)a < (unsigned)k) {
        rb.y = __int_as_float(a);  // the previous label, with or without a finite bound
        const float4 pi = pinfo[row];  // (previous distance, second-nearest bound, alpha_x, |x^|)
        const float dp = pi.x, sec = pi.y, al = pi.z, shx = pi.w;
        const float hx2 = shx * shx * (1.0f + 1e-6f);  // >= |x^|^2
        // px + hx2 with px = |x|^2 <= fl(alpha + hx2) (1 + 1e-6) (alpha = |x|^2 - |x^|^2 in FP32)
        const float pxh = fabsf(al + hx2) * (1.0f + 1e-6f) + hx2;
        // (fresh: dp bounds the distance to the current centroid, which has
        // not moved since)
        const float4 now = cst[a], old = fresh ? now : cst_old[a];  // (beta, |c^|^2, |c|^2, |c^|)
        const float r0 = dp - al - old.x + rho_bound(pxh, shx, old.z, old.y, old.w, kappa);
        const float r = (sqrt_approx(fmaxf(r0, 0.0f)) * (1.0f + 4e-6f) + (fresh ? 0.0f : delta[a])) * (1.0f + 1e-6f);
        const float u = r * r * (1.0f + 1e-6f) + al + now.x + rho_bound(pxh, shx, now.z, now.y, now.w, kappa);
        const float um = u + 1e-4f * (fabsf(u) + fabsf(al) + fabsf(now.x)) + 1e-30f;
        if (fabsf(um) < inf && fabsf(r0) < inf && fabsf(al) < inf) {  // false for NaN too: keep every tile
            m = 1ull << (a / kCentroidTileRows);  // its own tile
            need = false;
            // The screen only needs some upper bound: a wider margin costs
            // nothing measurable and keeps it far from the rounding terms.
            const float us = um + 1e-3f * (fabsf(um) + fabsf(al) + fabsf(now.x));
            if (fabsf(us) < inf) rb.x = us;
            // second-nearest bound: every centroid other than a, from the
            // previous GEMM's sec (free of beta) moved by at most max delta;
            // hl bounds d(x, c), hf the beta-free d(x, c) - beta_c
            float hl = -inf, hf = -inf;
            if (second) {
                const float g = sec - al - rho_bound(pxh, shx, gs.pc_old, gs.hc2_old, gs.shc_old, kappa) -
                                1e-4f * (fabsf(sec) + fabsf(al));
                const float sx =
                    fmaxf(sqrt_approx(fmaxf(g, 0.0f)) * (1.0f - 4e-6f) - gs.dmax * (1.0f + 1e-6f), 0.0f);
                const float s2 = sx * sx * (1.0f - 1e-6f);
                const float rn = rho_bound(pxh, shx, gs.pc, gs.hc2, gs.shc, kappa);
                const float lb = s2 + al + gs.bmin - rn;
                const float l = lb - 1e-4f * (fabsf(lb) + fabsf(al) + fabsf(gs.bmin));
                const float f = s2 + al - rn;
                const float lf = f - 1e-4f * (fabsf(f) + fabsf(al));
                if (l == l && lf == lf) hl = l, hf = lf;
            }
            float excl = inf;  // min over the tiles this row excludes of their beta-free lower bounds
            if (hl > um) {
                excl = hf;  // every other centroid strictly farther: no per-tile test
            } else {
                const float* dm = dmin + (int64_t)a * tiles;
                // rho of each tile's worst centroid: kp + tc.x + shx tc.y (the
                // per-tile terms of rho_bound, scaled up by 2e-6 to cover the
                // re-associated sum)
                const float kp = kappa * (1.0f + 2e-6f) * pxh;
                const float aal = fabsf(al);
#pragma unroll 8
                for (int t = 0; t < tiles; ++t) {  // (unrolled: the tiles' loads issue together)
                    const float4 tc = tcs[t];
                    const float gt = fmaxf(dm[t] - r, 0.0f);
                    const float g2 = gt * gt * (1.0f - 1e-6f);
                    const float rt = fmaf(shx, tc.y, kp + tc.x);
                    const float lb = g2 + al + tc.z - rt;
                    const float lbm = lb - 1e-4f * (fabsf(lb) + aal + tc.w);
                    if (!(lbm > um)) {  // (false for a non-finite tile: tc.z is NaN)
                        m |= 1ull << t;
                        need = true;
                    } else {
                        const float f = g2 + al - rt;
                        excl = fminf(excl, fmaxf(f - 1e-4f * (fabsf(f) + aal), hf));
                    }
                }
            }
            rb.z = excl;
            if (compact && !need)  // the label stands; its distance bounds for next time
                *reinterpret_cast<float2*>(pinfo + row) = make_float2(um, excl);
        }
    }
    if (compact && !need) m = 0;
    if (row_bound && (need || !compact)) row_bound[row] = rb;  // (compaction copies only the kept rows' records)
}

// Each row's pruning record, from the rows themselves: pinfo[g] = (an upper
// bound on d(x, c_a) for its label a's current centroid, 0, alpha_x, |x^|).
// The bound is |x^ - c^_a|^2 summed in FP32 over the MXFP8 round trip x^ of
// the point's row (quantize_rows' arithmetic: UE8M0 scale of each 32-feature
// block, E4M3 round to nearest even) and the dequantized centroid chat[a], plus
// the rounding of that sum, alpha_x + beta_a and rho (+inf for a row without
// a valid label); alpha_x = |x|^2 - |x^|^2 with |x|^2 summed as compute_l2_norm
// does.  A warp stages 32 rows, 128 features at a time (one 512-byte chunk per
// load, all 32 in flight), in shared memory with a 528-byte pitch; then each
// lane walks its own row.  tile_mask_kernel's `fresh` mode takes the bound on
// d(x, c_a) for the current centroids, with no centroid move added.
constexpr int kRowPitch = 132;  // floats per staged row
__global__ void __launch_bounds__(64) row_distance_bound_kernel(int64_t rows, int k, int d, const int* __restrict__ pid,
                                                                const int* __restrict__ label,
                                                                float4* __restrict__ pinfo,
                                                                const float* __restrict__ chat,
                                                                const float4* __restrict__ cst,
                                                                const float* __restrict__ points,
                                                                const int* __restrict__ stop) {
    if (stop && *stop) return;
    __shared__ __align__(16) float tile[2][32][kRowPitch];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row0 = ((int64_t)blockIdx.x * 2 + w) * 32;
    if (row0 >= rows) return;
    float(*t)[kRowPitch] = tile[w];
    const float inf = __int_as_float(0x7f800000);
    const int64_t g = row0 + lane;
    const int a = g < rows ? label[g] : -1;
    const bool valid = (unsigned)a < (unsigned)k;
    const float* c = chat + (int64_t)(valid ? a : 0) * d;
    const int my_point = g < rows ? (pid ? pid[g] : (int)g) : -1;  // (point ids are below 2^31)
    float sq = 0.0f, norm = 0.0f, h = 0.0f;
    for (int c0 = 0; c0 < d; c0 += 128) {
#pragma unroll
        for (int r = 0; r < 32; ++r) {
            const int x = __shfl_sync(0xffffffffu, my_point, r);
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (x >= 0) v = __ldg(reinterpret_cast<const float4*>(points + (int64_t)x * d + c0) + lane);
            *reinterpret_cast<float4*>(&t[r][4 * lane]) = v;
        }
        __syncwarp();
        const float4* own = reinterpret_cast<const float4*>(t[lane]);
#pragma unroll 1
        for (int b = 0; b < 4; ++b) {
            float amax = 0.0f;  // fmaxf drops NaN, as the quantizer's maximum does
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const float4 v = own[8 * b + q];
                amax = fmaxf(fmaxf(amax, fmaxf(fabsf(v.x), fabsf(v.y))), fmaxf(fabsf(v.z), fabsf(v.w)));
                norm = fmaf(v.w, v.w, fmaf(v.z, v.z, fmaf(v.y, v.y, fmaf(v.x, v.x, norm))));  // feature order
            }
            const uint32_t sc = dev::ue8m0_mxfp8_scale(amax);
            const float rcp = dev::ue8m0_reciprocal(sc), scale = dev::ue8m0_value(sc);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const float4 v = own[8 * b + q];
                const float4 cv = __ldg(reinterpret_cast<const float4*>(c + c0 + 32 * b + 4 * q));
                const float2 lo = dev::e4m3x2_decode(dev::e4m3x2_encode(v.x * rcp, v.y * rcp));
                const float2 hi = dev::e4m3x2_decode(dev::e4m3x2_encode(v.z * rcp, v.w * rcp));
                const float x0 = lo.x * scale, x1 = lo.y * scale, x2 = hi.x * scale, x3 = hi.y * scale;
                h = fmaf(x0, x0, fmaf(x1, x1, fmaf(x2, x2, fmaf(x3, x3, h))));
                const float t0 = x0 - cv.x, t1 = x1 - cv.y, t2 = x2 - cv.z, t3 = x3 - cv.w;
                sq = fmaf(t0, t0, fmaf(t1, t1, fmaf(t2, t2, fmaf(t3, t3, sq))));
            }
        }
        __syncwarp();
    }
    if (g >= rows) return;
    const float al = norm - h, shx = sqrtf(h);
    if (!valid) {
        pinfo[g] = make_float4(inf, 0.0f, al, shx);
        return;
    }
    const float kappa = 3e-5f + (float)(d + 8) * 1.2e-7f;
    const float hx2 = shx * shx * (1.0f + 1e-6f);
    const float pxh = fabsf(al + hx2) * (1.0f + 1e-6f) + hx2;
    const float4 cs = cst[a];  // (beta, |c^|^2, |c|^2, |c^|)
    const float geo = sq * (1.0f + (float)(d + 8) * 1.2e-7f) * (1.0f + 1e-6f);
    const float u = geo + al + cs.x + rho_bound(pxh, shx, cs.z, cs.y, cs.w, kappa);
    const float um = u + 1e-4f * (fabsf(u) + fabsf(al) + fabsf(cs.x));
    pinfo[g] = make_float4(um == um ? um : inf, 0.0f, al, shx);
}

// Per 128-row point tile (one warp; lane l takes rows l, l + 32, l + 64 and
// l + 96): the union over its rows of the centroid tiles the bounds cannot
// exclude.  With `compact` (the fused path's row compaction) a row whose every
// other centroid -- its own tile's included, through dmin[a][own], which
// leaves a out -- lies strictly beyond its upper bound keeps its label: it is
// left out of the GEMM (need_bits, counts), its distance for the next
// iteration's bounds becomes that upper bound and its second-nearest bound the
// smallest lower bound of its tiles, and the tile's mask is the union over the
// rows that remain; cmask[tile] is zeroed for the compacted masks of
// work_scatter_kernel.  tst / tst_old: 2 x tiles stats of the current and
// (optional) previous centroids; without tst_old or with a non-finite centroid
// the second-nearest bounds are not used.  prev_label and pinfo are per row,
// in the visiting order.  fresh: pinfo's distances bound the distance to the
// rows' current centroids (row_distance_bound_kernel).  Warps loop over point
// tiles.
__global__ void __launch_bounds__(128) tile_mask_kernel(
    int64_t rows, int k, int d, int tiles,
    const int* __restrict__ prev_label, float4* __restrict__ pinfo, const float4* __restrict__ cst,
    const float4* __restrict__ cst_old, const float4* __restrict__ tst, const float4* __restrict__ tst_old,
    const float* __restrict__ delta, const float* __restrict__ dmin, uint64_t* __restrict__ mask,
    float4* __restrict__ row_bound, int compact, int fresh, uint4* __restrict__ need_bits, int* __restrict__ tile_count,
    uint64_t* __restrict__ cmask, const int* __restrict__ stop) {
    if (stop && *stop) return;
    const float inf = __int_as_float(0x7f800000);
    __shared__ SetTerms gs_s;
    __shared__ int g_ok;
    const float kappa = 3e-5f + (float)(d + 8) * 1.2e-7f;
    // per centroid tile: (kappa' (max |c|^2 + max |c^|^2), 2 kappa' max |c^|,
    // min beta -- NaN for a tile with a non-finite centroid --, |min beta|),
    // kappa' = kappa (1 + 2e-6)
    __shared__ float4 tcs[kMaxPruneTiles];
    for (int t = threadIdx.x; t < tiles; t += blockDim.x) {
        const float4 ts = tst[t];  // (min beta, max |c^|^2, max |c|^2, non-finite)
        const float kq = kappa * (1.0f + 2e-6f);
        const float bmin = ts.w != 0.0f ? __int_as_float(0x7fc00000) : ts.x;
        tcs[t] = make_float4(kq * (ts.z + ts.y), 2.0f * kq * tst[tiles + t].z, bmin, fabsf(bmin));
    }
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        // v = (min beta, max |c^|^2, max |c|^2, max delta; previous: max |c^|^2, max |c|^2)
        float v[6] = {inf, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
        float bad = tst_old ? 0.0f : 1.0f;
        if (tst_old) {
            for (int t = lane; t < tiles; t += 32) {
                const float4 a = tst[t], b = tst[tiles + t], c = tst_old[t];
                v[0] = fminf(v[0], a.x), v[1] = fmaxf(v[1], a.y), v[2] = fmaxf(v[2], a.z), v[3] = fmaxf(v[3], b.y);
                v[4] = fmaxf(v[4], c.y), v[5] = fmaxf(v[5], c.z);
                bad = fmaxf(bad, fmaxf(a.w, c.w));
            }
        }
        for (int o = 16; o; o >>= 1) {
            v[0] = fminf(v[0], __shfl_xor_sync(0xffffffffu, v[0], o));
#pragma unroll
            for (int i = 1; i < 6; ++i) v[i] = fmaxf(v[i], __shfl_xor_sync(0xffffffffu, v[i], o));
            bad = fmaxf(bad, __shfl_xor_sync(0xffffffffu, bad, o));
        }
        if (lane == 0) {
            gs_s = SetTerms{v[0], v[1], v[2], v[3], v[4], v[5], sqrtf(v[1]), sqrtf(v[4])};
            g_ok = bad == 0.0f;
        }
    }
    __syncthreads();
    const SetTerms gs = gs_s;
    const bool second = g_ok != 0;
    const uint64_t all = tiles >= 64 ? ~0ull : ((1ull << tiles) - 1ull);
    const int64_t ntiles = (rows + 127) / 128;
    const int lane = threadIdx.x & 31;
    for (int64_t tile = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5); tile < ntiles; tile += (int64_t)gridDim.x * 4) {
        uint64_t m = 0;
        unsigned nb[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            uint64_t mr;
            bool need;
            row_tile_mask(tile * 128 + q * 32 + lane, rows, k, tiles, all, kappa, second, fresh != 0, gs, prev_label,
                          pinfo, cst, cst_old, tcs, delta, dmin, row_bound, compact, mr, need);
            m |= mr;
            nb[q] = __ballot_sync(0xffffffffu, need);
        }
        // union over the 128 rows
        m = __reduce_or_sync(0xffffffffu, (unsigned)m) |
            ((uint64_t)__reduce_or_sync(0xffffffffu, (unsigned)(m >> 32)) << 32);
        if (lane == 0) {
            mask[tile] = m;
            if (compact) {
                need_bits[tile] = make_uint4(nb[0], nb[1], nb[2], nb[3]);
                tile_count[tile] = __popc(nb[0]) + __popc(nb[1]) + __popc(nb[2]) + __popc(nb[3]);
                cmask[tile] = 0ull;
            }
        }
    }
}

// Segmented exclusive prefix sum of the per-tile counts of rows that stay in
// the GEMM: block s scans tiles [1024 s, 1024 s + 1024) into offsets[] (local
// to the segment) and writes the segment's total to seg_total[s];
// work_scatter_kernel adds the totals of the segments before its own.
constexpr int kScanSeg = 1024;
__global__ void __launch_bounds__(kScanSeg) work_scan_kernel(int ntiles, const int* __restrict__ counts,
                                                             int* __restrict__ offsets, int* __restrict__ seg_total,
                                                             const int* __restrict__ stop) {
    if (stop && *stop) return;
    __shared__ int warp_tot[32];
    const int i = blockIdx.x * kScanSeg + threadIdx.x;
    const int c = i < ntiles ? counts[i] : 0;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    int incl = c;
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31) warp_tot[w] = incl;
    __syncthreads();
    if (w == 0) {
        int t = warp_tot[lane];
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, t, o);
            if (lane >= o) t += v;
        }
        warp_tot[lane] = t;  // inclusive over warps
    }
    __syncthreads();
    if (i < ntiles) offsets[i] = incl - c + (w > 0 ? warp_tot[w - 1] : 0);
    if (threadIdx.x == 0) seg_total[blockIdx.x] = warp_tot[31];
}

// One block per 128-row point tile: the rows that stay in the GEMM, in order,
// to work_pid / work_rb at the tile's offset; the tile's mask ORed into the
// (at most two) compacted 128-row tiles its rows land in.
// Block 0 also writes *work_rows, the number of rows that stay (0 once the loop
// has stopped, so that the GEMM launches of later iterations do nothing).
constexpr int kScatterTiles = 8;  // point tiles per work_scatter block (kScanSeg is a multiple)
__global__ void __launch_bounds__(128) work_scatter_kernel(int64_t rows, const int* __restrict__ pid,
                                                           const float4* __restrict__ row_bound,
                                                           const uint4* __restrict__ need_bits,
                                                           const int* __restrict__ offsets,
                                                           const int* __restrict__ counts,
                                                           const int* __restrict__ seg_total, int nseg,
                                                           const uint64_t* __restrict__ mask,
                                                           int* __restrict__ work_pid, float4* __restrict__ work_rb,
                                                           unsigned long long* __restrict__ cmask,
                                                           int* __restrict__ work_rows, const int* __restrict__ stop) {
    static_assert(kScanSeg % kScatterTiles == 0, "a block's tiles share one scan segment");
    const bool stopped = stop && *stop;
    const int64_t tile0 = (int64_t)blockIdx.x * kScatterTiles;
    __shared__ int seg_base;
    if (threadIdx.x < 32) {  // the totals of the segments before this block's (all of them for block 0)
        const int seg = (int)(tile0 / kScanSeg);
        const int upto = blockIdx.x == 0 ? nseg : seg;
        int acc = 0, mine = 0;
        if (!stopped)
            for (int s2 = threadIdx.x; s2 < upto; s2 += 32) {
                const int v = seg_total[s2];
                acc += v;
                if (s2 < seg) mine += v;
            }
        for (int o = 16; o; o >>= 1) {
            acc += __shfl_xor_sync(0xffffffffu, acc, o);
            mine += __shfl_xor_sync(0xffffffffu, mine, o);
        }
        if (threadIdx.x == 0) {
            seg_base = mine;
            if (blockIdx.x == 0) *work_rows = stopped ? 0 : acc;
        }
    }
    if (stopped) return;
    __syncthreads();
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int64_t tile = tile0; tile < tile0 + kScatterTiles && tile * 128 < rows; ++tile) {
        const int cnt = counts[tile];
        if (cnt == 0) continue;
        const int64_t row = tile * 128 + threadIdx.x;
        const uint4 nb = need_bits[tile];
        const unsigned words[4] = {nb.x, nb.y, nb.z, nb.w};
        const int off = seg_base + offsets[tile];
        if ((words[w] >> lane) & 1u) {
            int before = __popc(words[w] & ((1u << lane) - 1u));
            for (int v = 0; v < w; ++v) before += __popc(words[v]);
            const int pos = off + before;
            work_pid[pos] = pid ? pid[row] : (int)row;
            work_rb[pos] = row_bound[row];
        }
        if (threadIdx.x == 0) {
            const uint64_t m = mask[tile];
            const int j0 = off >> 7, j1 = (off + cnt - 1) >> 7;
            atomicOr(cmask + j0, (unsigned long long)m);
            if (j1 != j0) atomicOr(cmask + j1, (unsigned long long)m);
        }
    }
}

}  // namespace

bool prune_supported(int64_t k, int d) {
    return (k + kCentroidTileRows - 1) / kCentroidTileRows <= kMaxPruneTiles && d % 128 == 0 && d <= 1024;
}

int launch_centroid_prep(int k, int d, const float* centroids, const float* prev, float* cn, float* chat,
                         float4* cst, float* delta, uint8_t* qcent, uint8_t* cscales, const int* stop,
                         cudaStream_t stream) {
    MXK_REQUIRE(prune_supported(k, d), "centroid prep: unsupported shape");
    LaunchScope scope("centroid_prep", stream);
    centroid_prep_kernel<<<(unsigned)(((int64_t)k * 32 + 255) / 256), 256, 0, stream>>>(k, d, centroids, prev, cn, chat,
                                                                                       cst, delta, qcent, cscales,
                                                                                       stop);
    MXK_CUDA(cudaGetLastError());
    return MXK_OK;
}

int launch_centroid_pairs(int k, int d, const float* chat, const float4* cst, const float* delta, float* dmin,
                          float4* tst, float* bmax32, const int* stop, cudaStream_t stream) {
    MXK_REQUIRE(prune_supported(k, d), "centroid pairs: unsupported shape");
    const int tiles = (k + kCentroidTileRows - 1) / kCentroidTileRows;
    LaunchScope scope("centroid_pairs", stream);
    pair_bounds_kernel<<<dim3((unsigned)((k + kPairRows - 1) / kPairRows), (unsigned)tiles), kPairThreads, 0, stream>>>(
        k, d, tiles, chat, cst, delta, dmin, tst, bmax32, stop);
    MXK_CUDA(cudaGetLastError());
    return MXK_OK;
}

int launch_centroid_pairs_drift(int k, int d, const float* delta, const float4* cst, float* dmin, float4* tst,
                                float* bmax32, const int* stop, cudaStream_t stream) {
    MXK_REQUIRE(prune_supported(k, d), "centroid pairs: unsupported shape");
    const int tiles = (k + kCentroidTileRows - 1) / kCentroidTileRows;
    LaunchScope scope("centroid_pairs_drift", stream);
    pair_drift_kernel<<<(unsigned)(tiles + (k + kPairThreads - 1) / kPairThreads), kPairThreads, 0, stream>>>(
        k, tiles, delta, cst, dmin, tst, bmax32, stop);
    MXK_CUDA(cudaGetLastError());
    return MXK_OK;
}

int launch_row_distance_bound(int64_t rows, int k, int d, const int* pid, const int* label, float4* pinfo,
                              const float* chat, const float4* cst, const float* points, const int* stop,
                              cudaStream_t stream) {
    if (rows <= 0) return MXK_OK;
    MXK_REQUIRE(prune_supported(k, d) && label && pinfo && chat && cst && points, "row distance bound: bad arguments");
    MXK_REQUIRE((rows + 63) / 64 < (1ll << 31), "row distance bound: too many rows");
    LaunchScope scope("row_distance_bound", stream);
    row_distance_bound_kernel<<<(unsigned)((rows + 63) / 64), 64, 0, stream>>>(rows, k, d, pid, label, pinfo, chat,
                                                                               cst, points, stop);
    MXK_CUDA(cudaGetLastError());
    return MXK_OK;
}

int launch_tile_mask(int64_t rows, int k, int d, const int* pid, const int* prev_label, float4* pinfo,
                     const float4* cst, const float4* cst_old, const float4* tst, const float4* tst_old,
                     const float* delta, const float* dmin, uint64_t* mask, float4* row_bound, const int* stop,
                     cudaStream_t stream, WorkRows* work, bool fresh) {
    if (rows <= 0 && !work) return MXK_OK;
    const int tiles = (k + kCentroidTileRows - 1) / kCentroidTileRows;
    MXK_REQUIRE(tiles <= kMaxPruneTiles, "tile mask: at most 64 centroid tiles");
    MXK_REQUIRE(!work || (row_bound && work->pid && work->rb && work->need_bits && work->counts && work->offsets &&
                          work->seg_total && work->cmask && work->rows),
                "tile mask: incomplete row-compaction buffers");
    const int64_t blocks = (rows + kPointTileRows - 1) / kPointTileRows;
    MXK_REQUIRE(blocks < (1ll << 31), "tile mask: too many rows");
    if (blocks > 0) {
        LaunchScope scope("tile_mask", stream);
        // one resident wave of blocks (four point tiles at a time), looping over the point tiles
        static int per_sm = 0;
        if (per_sm <= 0) {
            MXK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, tile_mask_kernel, 128, 0));
            per_sm = std::max(per_sm, 1);
        }
        tile_mask_kernel<<<(unsigned)std::min<int64_t>((blocks + 3) / 4, (int64_t)sm_count() * per_sm), 128, 0,
                           stream>>>(
            rows, k, d, tiles, prev_label, pinfo, cst, cst_old, tst, tst_old, delta, dmin, mask,
            row_bound, work ? 1 : 0, fresh ? 1 : 0, work ? work->need_bits : nullptr, work ? work->counts : nullptr,
            work ? reinterpret_cast<uint64_t*>(work->cmask) : nullptr, stop);
        MXK_CUDA(cudaGetLastError());
    }
    if (!work) return MXK_OK;
    const int nseg = (int)((blocks + kScanSeg - 1) / kScanSeg);
    if (nseg > 0) {
        LaunchScope scope("work_scan", stream);
        work_scan_kernel<<<(unsigned)nseg, kScanSeg, 0, stream>>>((int)blocks, work->counts, work->offsets,
                                                                   work->seg_total, stop);
        MXK_CUDA(cudaGetLastError());
    }
    {  // (at least one block: it writes the row count)
        LaunchScope scope("work_scatter", stream);
        work_scatter_kernel<<<(unsigned)std::max<int64_t>((blocks + kScatterTiles - 1) / kScatterTiles, 1), 128, 0,
                              stream>>>(
            rows, pid, row_bound, work->need_bits, work->offsets, work->counts, work->seg_total, nseg, mask,
            work->pid, work->rb, work->cmask, work->rows, stop);
        MXK_CUDA(cudaGetLastError());
    }
    return MXK_OK;
}

}  // namespace mxk
