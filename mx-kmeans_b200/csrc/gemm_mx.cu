// K2: block-scaled MX GEMM on 5th-generation tensor cores (tcgen05, sm_100a).
//
//   D[m x n] = A[m x k] . B[n x k]^T,  A = quantized points (MXFP8; MXFP6/MXFP4
//   re-encoded to E4M3 on the way into shared memory), B = MXFP8 centroids, one
//   UE8M0 scale per 32 features of each row.
//
// Reference: ParCIS/MX-KMeans src/kernels/gemm.cu:32-363 (CUTLASS SM120
// collective, dense FP32 output) followed by src/kernels/assignment.cu:19-57
// (nearest_kernel over the dense product).  Here the same product feeds either
// a dense store (gemm_mx API) or, fused, the distance fmaf(-2,dot,pn+cn) and the
// lowest-index argmin (+ optional two-largest gap) so that no N x K buffer exists.
//
// Structure (one persistent CTA per SM, 320 threads):
//   warp 0      producer: TMA (SWIZZLE_128B) of a 128-row point tile (all K,
//               resident while every centroid tile streams past) and of 128-row
//               x 128-byte centroid chunks through a ring as deep as shared
//               memory allows; 1-D bulk copies of the matching 512-byte
//               tcgen05 scale atoms (the quantizer writes scales in that layout;
//               row-major API scales are converted once per call).
//   warp 1      TMEM allocator and the single MMA-issuing thread: tcgen05.cp of
//               the scale atoms into TMEM, tcgen05.mma kind::mxf8f6f4
//               block_scale (M=128, N=128, K=32) into a double-buffered TMEM
//               accumulator, tcgen05.commit to release smem stages / publish tiles.
//   warps 2-17  epilogue: tcgen05.ld of the accumulator (warp w reads TMEM lane
//               quadrant w%4, 32-column quarter (w-2)/4), then dense store or
//               argmin: packed f32x2 distances, a 3-input-min tree per 32
//               columns and an index search only when that chunk improves the
//               row's running minimum.
#include <cstring>

#include "common.cuh"
#include "kernels.cuh"
#include "mx_codec.cuh"

namespace mxk {
namespace {

constexpr int kBM = 128;           // points per tile = TMEM lanes
constexpr int kBN = 128;           // centroids per accumulator tile
constexpr int kChunk = 128;        // K bytes per chunk = one SWIZZLE_128B row
constexpr int kTileBytes = kBM * kChunk;  // 16 KB
constexpr int kSfAtom = 512;       // 128 rows x 4 scale bytes
constexpr int kMaxBStages = 12;   // centroid-chunk ring depth: as many as shared memory holds
constexpr int kAccStages = 2;
constexpr int kEpiWarps = 16;     // 4 per TMEM lane quadrant, one 32-column quarter each
constexpr int kThreads = (2 + kEpiWarps) * 32;
constexpr int kMaxSmemNorms = 8192;  // centroid norms staged in shared memory up to this k
constexpr int kMaxChunks = 8;      // K <= 1024
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kSfaCol = 256;  // 4 columns per K chunk
constexpr uint32_t kSfbCol = 320;

struct GemmParams {
    int64_t m;
    const int* m_dev;
    int64_t n;
    int kdim;
    int kchunks;
    int a_bits;
    int a_stages;
    const uint8_t* a;  // packed source rows (only read directly when a_bits != 8)
    const uint8_t* a_scales;
    const uint8_t* b_scales;
    float* out;  // dense mode
    int out_vec;  // out is 16-byte aligned and n % 4 == 0 (vector stores)
    int cn_smem;  // number of centroid norms staged in shared memory (0 = read from global)
    int b_stages; // depth of the centroid-chunk ring (<= kMaxBStages)
    const float* pn;
    const float* cn;
    const int* pid;
    int* labels;
    float* gaps;
    const int* start_hint;  // optional: a label per point; each tile's sweep starts at its first row's tile
    unsigned* err;
};

struct SmemLayout {
    uint32_t a_off, b_off, sfa_off, sfb_off, merge_off, cn_off, bar_off, total;
};

// cn_floats: centroid norms staged in shared memory (0 when read from global).
__host__ __device__ inline SmemLayout smem_layout(int kchunks, int a_stages, int cn_floats, int b_stages) {
    SmemLayout s;
    s.a_off = 0;
    s.b_off = s.a_off + a_stages * kchunks * kTileBytes;
    s.sfa_off = s.b_off + b_stages * kTileBytes;
    s.sfb_off = s.sfa_off + a_stages * kchunks * kSfAtom;
    s.merge_off = s.sfb_off + b_stages * kSfAtom;                  // 3 quarters x 128 rows x 16 B
    s.cn_off = s.merge_off + 3 * kBM * 16;
    s.bar_off = s.cn_off + (uint32_t)((cn_floats * 4 + 15) / 16 * 16);
    s.total = s.bar_off + 40 * 8 + 64;  // 4 + 2*12 + 2*2 + 3 barriers, then the TMEM slot
    return s;
}

// Byte offset of (row, k-byte) inside a 128-row x 128-byte SWIZZLE_128B tile:
// the 16-byte chunk index is XOR-ed with row % 8 (the layout TMA writes).
__device__ __forceinline__ uint32_t sw128_offset(int row, int kbyte) {
    return (uint32_t)row * 128u + ((((uint32_t)kbyte >> 4) ^ ((uint32_t)row & 7u)) << 4) + ((uint32_t)kbyte & 15u);
}

// Fill one 128 x 128-byte A chunk from packed MXFP6 / MXFP4 rows, re-encoding
// every code as the E4M3 code of the same value (exact), in SWIZZLE_128B order.
__device__ void fill_a_subbyte(uint8_t* dst, const GemmParams& p, int64_t row0, int kc, int64_t mrows, int lane) {
    for (int i = 0; i < 4; ++i) {
        const int r = lane + 32 * i;
        const int64_t grow = row0 + r;
        for (int f = 0; f < kChunk; f += 4) {
            uint32_t word = 0;
            if (grow < mrows) {
                const int64_t feat = (int64_t)kc * kChunk + f;
                uint32_t c0, c1, c2, c3;
                if (p.a_bits == 6) {
                    const uint8_t* src = p.a + ((grow * p.kdim + feat) / 4) * 3;
                    const uint32_t g = (uint32_t)src[0] | ((uint32_t)src[1] << 8) | ((uint32_t)src[2] << 16);
                    c0 = dev::e2m3_to_e4m3(g & 63u);
                    c1 = dev::e2m3_to_e4m3((g >> 6) & 63u);
                    c2 = dev::e2m3_to_e4m3((g >> 12) & 63u);
                    c3 = dev::e2m3_to_e4m3((g >> 18) & 63u);
                } else {
                    const uint8_t* src = p.a + (grow * p.kdim + feat) / 2;
                    const uint32_t g = (uint32_t)src[0] | ((uint32_t)src[1] << 8);
                    c0 = dev::e2m1_to_e4m3(g & 15u);
                    c1 = dev::e2m1_to_e4m3((g >> 4) & 15u);
                    c2 = dev::e2m1_to_e4m3((g >> 8) & 15u);
                    c3 = dev::e2m1_to_e4m3((g >> 12) & 15u);
                }
                word = c0 | (c1 << 8) | (c2 << 16) | (c3 << 24);
            }
            *reinterpret_cast<uint32_t*>(dst + sw128_offset(r, f)) = word;
        }
    }
}

// Row-major scales [rows][k/32] -> tcgen05 scale atoms: one 512-byte atom per
// (128-row tile, 128-feature chunk), tile-major, row r's four block scales at
// (r % 32) * 16 + (r / 32) * 4 + block % 4; rows past `rows` get 0 (2^-127).
__global__ void __launch_bounds__(256) scales_to_atoms_kernel(int64_t rows, int kchunks, const uint8_t* __restrict__ src,
                                                              uint8_t* __restrict__ atoms, int64_t n_words) {
    for (int64_t w = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; w < n_words; w += (int64_t)gridDim.x * blockDim.x) {
        // word w = atom a, 32-bit slot (lane l, row group i): rows r = l + 32 i
        const int64_t a = w >> 7;
        const int slot = (int)(w & 127);
        const int l = slot >> 2, i = slot & 3;
        const int64_t tile = a / kchunks;
        const int kc = (int)(a - tile * kchunks);
        const int64_t row = tile * 128 + l + 32 * i;
        uint32_t v = 0;
        if (row < rows) v = *reinterpret_cast<const uint32_t*>(src + row * (int64_t)kchunks * 4 + 4 * kc);
        reinterpret_cast<uint32_t*>(atoms)[w] = v;
    }
}

// First centroid tile of the sweep for point tile `tile`: the tile holding the
// hint label of the tile's first row (the driver passes the previous
// iteration's labels, and rows are ordered by them, so that tile usually holds
// every row's nearest centroid and later chunks rarely improve a row).  Any
// start gives the same result: ties are broken by index, not by sweep order.
__device__ __forceinline__ int sweep_start(const GemmParams& p, int64_t tile, int64_t mrows, int tiles_n) {
    if (!p.start_hint) return 0;
    const int64_t row0 = tile * kBM;
    if (row0 >= mrows) return 0;
    const int64_t point = p.pid ? (int64_t)p.pid[row0] : row0;
    const int lab = p.start_hint[point];
    if (lab < 0 || (int64_t)lab >= p.n) return 0;
    return lab / kBN;
}

template <bool kArgmin, bool kGaps>
__global__ void __launch_bounds__(kThreads, 1)
    mx_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                   const GemmParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const SmemLayout L = smem_layout(p.kchunks, p.a_stages, p.cn_smem, p.b_stages);
    const int kBStages = p.b_stages;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bar_off);
    uint64_t* a_full = bars;                // [2]
    uint64_t* a_empty = bars + 2;           // [2]
    uint64_t* b_full = bars + 4;            // [kMaxBStages]
    uint64_t* b_empty = bars + 4 + kMaxBStages;
    uint64_t* acc_full = bars + 4 + 2 * kMaxBStages;
    uint64_t* acc_empty = acc_full + kAccStages;
    uint64_t* drain = acc_empty + kAccStages;
    uint64_t* merge_full = drain + 1;   // column-half hand-off of the argmin epilogue
    uint64_t* merge_empty = drain + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 40);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 40) + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t mrows = p.m_dev ? (int64_t)*p.m_dev : p.m;
    const int64_t tiles_m = (mrows + kBM - 1) / kBM;
    const int tiles_n = (int)((p.n + kBN - 1) / kBN);

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) dev::mbar_init(&a_full[i], 1), dev::mbar_init(&a_empty[i], 1);
        for (int i = 0; i < kBStages; ++i) dev::mbar_init(&b_full[i], 1), dev::mbar_init(&b_empty[i], 1);
        for (int i = 0; i < kAccStages; ++i) dev::mbar_init(&acc_full[i], 1), dev::mbar_init(&acc_empty[i], kEpiWarps);
        dev::mbar_init(drain, 1);
        dev::mbar_init(merge_full, 3 * kEpiWarps / 4);   // quarters 1..3 deposit
        dev::mbar_init(merge_empty, kEpiWarps / 4);      // quarter 0 has read
        *abort_flag = 0;
        dev::fence_barrier_init();
    }
    if (warp == 1) dev::tmem_alloc(tmem_slot, kTmemCols);
    if (kArgmin && p.cn_smem) {
        float* cn_s = reinterpret_cast<float*>(smem + L.cn_off);
        for (int i = threadIdx.x; i < p.cn_smem; i += blockDim.x) cn_s[i] = p.cn[i];
    }
    if (warp == 0 && lane == 0) {
        if (p.a_bits == 8) dev::prefetch_tensor_map(&tmap_a);
        dev::prefetch_tensor_map(&tmap_b);
    }
    dev::tc_fence_before();
    __syncthreads();
    dev::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        uint32_t bcount = 0;
        int it = 0;
        bool ok = true;
        for (int64_t tile = blockIdx.x; tile < tiles_m && ok; tile += gridDim.x, ++it) {
            const int as = it % p.a_stages;
            const uint32_t aph = (uint32_t)(it / p.a_stages) & 1u;
            if (!dev::mbar_wait(&a_empty[as], aph ^ 1u, abort_flag, p.err)) { ok = false; break; }
            uint8_t* a_smem = smem + L.a_off + (uint32_t)as * p.kchunks * kTileBytes;
            uint8_t* sfa = smem + L.sfa_off + (uint32_t)as * p.kchunks * kSfAtom;
            if (lane == 0) {
                const uint32_t bytes = (p.a_bits == 8 ? p.kchunks * kTileBytes : 0) + p.kchunks * kSfAtom;
                if (bytes)
                    asm volatile("mbarrier.expect_tx.shared::cta.b64 [%0], %1;" ::"r"(dev::smem_addr(&a_full[as])),
                                 "r"(bytes));
                if (p.a_bits == 8)
                    for (int kc = 0; kc < p.kchunks; ++kc)
                        dev::tma_load_2d(a_smem + kc * kTileBytes, &tmap_a, kc * kChunk, (int32_t)(tile * kBM), &a_full[as]);
                dev::bulk_load(sfa, p.a_scales + tile * p.kchunks * kSfAtom, (uint32_t)(p.kchunks * kSfAtom),
                               &a_full[as]);
            }
            if (p.a_bits != 8)
                for (int kc = 0; kc < p.kchunks; ++kc)
                    fill_a_subbyte(a_smem + kc * kTileBytes, p, tile * kBM, kc, mrows, lane);
            dev::fence_proxy_async();
            __syncwarp();
            if (lane == 0) dev::mbar_arrive(&a_full[as]);
            const int ct0 = sweep_start(p, tile, mrows, tiles_n);
            for (int i = 0; i < tiles_n && ok; ++i) {
                const int ct = ct0 + i < tiles_n ? ct0 + i : ct0 + i - tiles_n;
                for (int kc = 0; kc < p.kchunks; ++kc, ++bcount) {
                    const int bs = (int)(bcount % kBStages);
                    const uint32_t bph = (bcount / kBStages) & 1u;
                    if (!dev::mbar_wait(&b_empty[bs], bph ^ 1u, abort_flag, p.err)) { ok = false; break; }
                    if (lane == 0) {
                        asm volatile("mbarrier.expect_tx.shared::cta.b64 [%0], %1;" ::"r"(dev::smem_addr(&b_full[bs])),
                                     "r"((uint32_t)(kTileBytes + kSfAtom)));
                        dev::tma_load_2d(smem + L.b_off + bs * kTileBytes, &tmap_b, kc * kChunk, ct * kBN, &b_full[bs]);
                        dev::bulk_load(smem + L.sfb_off + bs * kSfAtom,
                                       p.b_scales + ((int64_t)ct * p.kchunks + kc) * kSfAtom, kSfAtom, &b_full[bs]);
                    }
                    __syncwarp();
                    if (lane == 0) dev::mbar_arrive(&b_full[bs]);
                }
            }
        }
        // Unwinding after an abort: wait (bounded) for the copies this warp
        // issued, so no TMA write lands in shared memory after the CTA exits.
        if (!ok && lane == 0) {
            volatile int no_abort = 0;
            for (uint32_t c = bcount > kBStages ? bcount - kBStages : 0; c < bcount; ++c)
                dev::mbar_wait(&b_full[c % kBStages], (c / kBStages) & 1u, &no_abort, nullptr);
            for (int j = it > p.a_stages ? it - p.a_stages : 0; j <= it; ++j)
                dev::mbar_wait(&a_full[j % p.a_stages], (uint32_t)(j / p.a_stages) & 1u, &no_abort, nullptr);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            uint32_t bcount = 0, acount = 0;
            int it = 0;
            bool ok = true;
            for (int64_t tile = blockIdx.x; tile < tiles_m && ok; tile += gridDim.x, ++it) {
                const int as = it % p.a_stages;
                const uint32_t aph = (uint32_t)(it / p.a_stages) & 1u;
                if (!dev::mbar_wait(&a_full[as], aph, abort_flag, p.err)) { ok = false; break; }
                dev::tc_fence_after();
                const uint32_t a_base = dev::smem_addr(smem + L.a_off + (uint32_t)as * p.kchunks * kTileBytes);
                const uint32_t sfa_base = dev::smem_addr(smem + L.sfa_off + (uint32_t)as * p.kchunks * kSfAtom);
                for (int kc = 0; kc < p.kchunks; ++kc)
                    dev::tc_copy_32x128b_x4(tmem + kSfaCol + 4 * kc,
                                            dev::smem_desc(sfa_base + kc * kSfAtom, 16, 128, dev::kLayoutNone));
                for (int ct = 0; ct < tiles_n && ok; ++ct, ++acount) {
                    const int accs = (int)(acount % kAccStages);
                    const uint32_t accph = (acount / kAccStages) & 1u;
                    if (!dev::mbar_wait(&acc_empty[accs], accph ^ 1u, abort_flag, p.err)) { ok = false; break; }
                    dev::tc_fence_after();
                    const uint32_t d_tmem = tmem + accs * kBN;
                    for (int kc = 0; kc < p.kchunks; ++kc, ++bcount) {
                        const int bs = (int)(bcount % kBStages);
                        const uint32_t bph = (bcount / kBStages) & 1u;
                        if (!dev::mbar_wait(&b_full[bs], bph, abort_flag, p.err)) { ok = false; break; }
                        dev::tc_fence_after();
                        const uint32_t b_addr = dev::smem_addr(smem + L.b_off + bs * kTileBytes);
                        dev::tc_copy_32x128b_x4(tmem + kSfbCol,
                                                dev::smem_desc(dev::smem_addr(smem + L.sfb_off + bs * kSfAtom), 16, 128,
                                                               dev::kLayoutNone));
#pragma unroll
                        for (int kb = 0; kb < 4; ++kb) {
                            const uint64_t adesc =
                                dev::smem_desc(a_base + kc * kTileBytes + kb * 32, 16, 1024, dev::kLayoutSwizzle128);
                            const uint64_t bdesc = dev::smem_desc(b_addr + kb * 32, 16, 1024, dev::kLayoutSwizzle128);
                            const uint32_t idesc = dev::mx_idesc(dev::kFmtE4M3, dev::kFmtE4M3, kBM, kBN, (uint32_t)kb);
                            dev::tc_mma_mx(d_tmem, adesc, bdesc, idesc, (tmem + kSfaCol + 4 * kc) | ((uint32_t)kb << 30),
                                           (tmem + kSfbCol) | ((uint32_t)kb << 30), (kc | kb) != 0);
                        }
                        dev::tc_commit(&b_empty[bs]);
                    }
                    if (ok) dev::tc_commit(&acc_full[accs]);
                }
                if (ok) dev::tc_commit(&a_empty[as]);
            }
            // Make sure every issued MMA/copy has finished before TMEM is freed.
            dev::tc_commit(drain);
            volatile int no_abort = 0;
            dev::mbar_wait(drain, 0, &no_abort, p.err);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------ epilogue
        const int q = warp & 3;          // TMEM lane quadrant this warp may access
        const int h = (warp - 2) >> 2;   // 32-column quarter of each accumulator tile
        const int r = q * 32 + lane;     // row within the point tile
        float4* merge = reinterpret_cast<float4*>(smem + L.merge_off);
        const float* cn_s = reinterpret_cast<const float*>(smem + L.cn_off);
        uint32_t acount = 0, merge_count = 0;
        bool ok = true;
        for (int64_t tile = blockIdx.x; tile < tiles_m && ok; tile += gridDim.x) {
            const int64_t grow = tile * kBM + r;
            const bool valid = grow < mrows;
            int64_t point = grow;
            float pn = 0.0f;
            if (kArgmin && valid) {
                point = p.pid ? (int64_t)p.pid[grow] : grow;
                pn = p.pn[point];
            }
            const uint64_t pn2 = dev::pack2(pn, pn);
            float first = __int_as_float(0x7f800000), largest = -1e38f, next = -1e38f;
            int best = 0x7fffffff;
            const int ct0 = sweep_start(p, tile, mrows, tiles_n);
            for (int i = 0; i < tiles_n; ++i, ++acount) {
                const int ct = ct0 + i < tiles_n ? ct0 + i : ct0 + i - tiles_n;
                const int accs = (int)(acount % kAccStages);
                const uint32_t accph = (acount / kAccStages) & 1u;
                if (!dev::mbar_wait(&acc_full[accs], accph, abort_flag, p.err)) { ok = false; break; }
                dev::tc_fence_after();
                uint32_t v[32];
                dev::tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + accs * kBN + h * 32, v);
                dev::tmem_wait_ld();
                dev::tc_fence_before();
                __syncwarp();
                if (lane == 0) dev::mbar_arrive(&acc_empty[accs]);
                const int64_t c0 = (int64_t)ct * kBN + h * 32;
                if constexpr (!kArgmin) {
                    if (valid) {
                        float* orow = p.out + grow * p.n;
                        if (c0 + 32 <= p.n && p.out_vec) {
#pragma unroll
                            for (int j = 0; j < 32; j += 4)
                                *reinterpret_cast<float4*>(orow + c0 + j) =
                                    make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]),
                                                __uint_as_float(v[j + 2]), __uint_as_float(v[j + 3]));
                        } else {
#pragma unroll
                            for (int j = 0; j < 32; ++j)
                                if (c0 + j < p.n) orow[c0 + j] = __uint_as_float(v[j]);
                        }
                    }
                } else if (c0 + 32 <= p.n) {
                    // distances fmaf(-2, dot, pn + cn) two at a time (add/fma .f32x2, each
                    // lane rounded exactly like the scalar operation)
                    float dist[32];
#pragma unroll
                    for (int j = 0; j < 32; j += 4) {
                        const float4 cv = p.cn_smem ? *reinterpret_cast<const float4*>(cn_s + c0 + j)
                                                    : __ldg(reinterpret_cast<const float4*>(p.cn + c0 + j));
                        dev::dist2(v[j], v[j + 1], pn2, cv.x, cv.y, dist[j], dist[j + 1]);
                        dev::dist2(v[j + 2], v[j + 3], pn2, cv.z, cv.w, dist[j + 2], dist[j + 3]);
                    }
                    if constexpr (kGaps) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            next = fmaxf(next, fminf(largest, dist[j]));
                            largest = fmaxf(largest, dist[j]);
                        }
                    }
                    // Chunk minimum with 3-input mins.  The index search runs only
                    // when the chunk can change the row's (distance, index) minimum:
                    // a smaller distance, or an equal one (a tie resolved by the
                    // lower index, as insert_distance does; rare after the first
                    // chunk).  NaN distances never compare, as in the reference.
                    float m3[11];
#pragma unroll
                    for (int t = 0; t < 10; ++t) m3[t] = dev::min3f(dist[3 * t], dist[3 * t + 1], dist[3 * t + 2]);
                    m3[10] = fminf(dist[30], dist[31]);
                    const float ma = dev::min3f(m3[0], m3[1], m3[2]);
                    const float mb = dev::min3f(m3[3], m3[4], m3[5]);
                    const float mc = dev::min3f(m3[6], m3[7], m3[8]);
                    const float cm = fminf(dev::min3f(ma, mb, mc), fminf(m3[9], m3[10]));
                    if (cm <= first) {
                        int idx = 31;
#pragma unroll
                        for (int j = 30; j >= 0; --j) idx = dist[j] == cm ? j : idx;
                        const int cand = (int)c0 + idx;
                        if (cm < first || cand < best) {
                            first = cm;
                            best = cand;
                        }
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        if (c0 + j < p.n) {
                            const float cnv = p.cn_smem ? cn_s[c0 + j] : __ldg(p.cn + c0 + j);
                            const float dist = fmaf(-2.0f, __uint_as_float(v[j]), pn + cnv);
                            if (dist < first || (dist == first && (int)(c0 + j) < best)) {
                                first = dist;
                                best = (int)(c0 + j);
                            }
                            if constexpr (kGaps) {
                                next = fmaxf(next, fminf(largest, dist));
                                largest = fmaxf(largest, dist);
                            }
                        }
                    }
                }
            }
            if constexpr (kArgmin) {
                if (!ok) break;
                // Combine the four column quarters of each row: lexicographic
                // (distance, index) minimum and the two-largest merge.  The hand-off
                // uses mbarriers with bounded waits (never an unbounded bar.sync).
                const uint32_t mph = (uint32_t)(merge_count++) & 1u;
                if (h != 0) {
                    if (!dev::mbar_wait(merge_empty, mph ^ 1u, abort_flag, p.err)) { ok = false; break; }
                    merge[(h - 1) * kBM + r] = make_float4(first, __int_as_float(best), largest, next);
                    __syncwarp();
                    if (lane == 0) dev::mbar_arrive(merge_full);
                } else {
                    if (!dev::mbar_wait(merge_full, mph, abort_flag, p.err)) { ok = false; break; }
                    float4 o[3];
#pragma unroll
                    for (int t = 0; t < 3; ++t) o[t] = merge[t * kBM + r];
                    __syncwarp();
                    if (lane == 0) dev::mbar_arrive(merge_empty);
                    if (valid) {
#pragma unroll
                        for (int t = 0; t < 3; ++t) {
                            const int ob = __float_as_int(o[t].y);
                            if (o[t].x < first || (o[t].x == first && ob < best)) first = o[t].x, best = ob;
                            if constexpr (kGaps) {
                                next = fmaxf(fminf(largest, o[t].z), fmaxf(next, o[t].w));
                                largest = fmaxf(largest, o[t].z);
                            }
                        }
                        p.labels[point] = best;
                        if constexpr (kGaps) p.gaps[point] = largest - next;
                    }
                }
            }
        }
    }

    dev::tc_fence_before();
    __syncthreads();
    dev::tc_fence_after();
    if (warp == 1) dev::tmem_dealloc(tmem, kTmemCols);
}

bool aligned(const void* p, int bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) == 0; }

}  // namespace

int launch_gemm_mx(int bits, int64_t m, int64_t n, int k, const void* a, const uint8_t* a_scales, const uint8_t* b,
                   const uint8_t* b_scales, float* out, const MxArgmin* argmin, const int* rows_dev,
                   cudaStream_t stream, bool scale_atoms) {
    if (bits != 4 && bits != 6 && bits != 8) return fail(MXK_ERR_INVALID, "Precision must be 4, 6, or 8");
    if (m <= 0 || n <= 0) return MXK_OK;
    MXK_REQUIRE(k > 0 && k % kChunk == 0, "gemm_mx: k must be a positive multiple of 128");
    if (k / kChunk > kMaxChunks) return fail(MXK_ERR_UNSUPPORTED, "gemm_mx: k > 1024 is not supported");
    MXK_REQUIRE(a && b && a_scales && b_scales, "gemm_mx: null operand");
    MXK_REQUIRE(aligned(a, 16) && aligned(b, 16), "gemm_mx: operands must be 16-byte aligned");
    MXK_REQUIRE(aligned(a_scales, scale_atoms ? 16 : 4) && aligned(b_scales, scale_atoms ? 16 : 4),
                "gemm_mx: scales must be 4-byte aligned (16 for the atom layout)");
    MXK_REQUIRE(n < (1ll << 31) && m < (1ll << 31), "gemm_mx: m and n must be below 2^31 (TMA coordinates)");
    if (argmin) {
        MXK_REQUIRE(argmin->point_norms && argmin->centroid_norms && argmin->labels, "assign: null pointer");
        MXK_REQUIRE(aligned(argmin->centroid_norms, 16), "assign: centroid norms must be 16-byte aligned");
    } else {
        MXK_REQUIRE(out != nullptr, "gemm_mx: null output");
    }

    CUtensorMap tmap_a, tmap_b;
    std::memset(&tmap_a, 0, sizeof(tmap_a));
    if (bits == 8)
        MXK_CHECK(encode_tensor_map_2d(&tmap_a, a, (uint64_t)k, (uint64_t)m, (uint64_t)k, kChunk, kBM,
                                       CU_TENSOR_MAP_DATA_TYPE_UINT8, CU_TENSOR_MAP_SWIZZLE_128B));
    MXK_CHECK(encode_tensor_map_2d(&tmap_b, b, (uint64_t)k, (uint64_t)n, (uint64_t)k, kChunk, kBN,
                                   CU_TENSOR_MAP_DATA_TYPE_UINT8, CU_TENSOR_MAP_SWIZZLE_128B));

    GemmParams p{};
    p.m = m;
    p.m_dev = rows_dev;
    p.n = n;
    p.kdim = k;
    p.kchunks = k / kChunk;
    p.a_bits = bits;
    p.a = static_cast<const uint8_t*>(a);
    p.a_scales = a_scales;
    p.b_scales = b_scales;
    p.out = out;
    p.out_vec = out && aligned(out, 16) && (n % 4 == 0);
    if (argmin) {
        p.pn = argmin->point_norms;
        p.cn = argmin->centroid_norms;
        p.pid = argmin->pid;
        p.labels = argmin->labels;
        p.gaps = argmin->gaps;
        p.start_hint = argmin->start_hint;
    }
    p.err = device_error_word();
    if (!p.err) return fail(MXK_ERR_CUDA, "gemm_mx: cannot allocate the device error word");

    int max_smem = 0, dev = 0;
    MXK_CUDA(cudaGetDevice(&dev));
    MXK_CUDA(cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    // Shared-memory plan: two point-tile stages when they fit, the centroid norms
    // when they fit, then as deep a centroid-chunk ring as the rest allows
    // (deeper rings keep more TMA bytes in flight per SM).
    auto fits = [&](int as, int cn, int bs) { return (int)smem_layout(p.kchunks, as, cn, bs).total + 1024 <= max_smem; };
    p.cn_smem = (argmin && n <= kMaxSmemNorms) ? (int)n : 0;
    p.a_stages = fits(2, p.cn_smem, 4) ? 2 : 1;
    if (!fits(p.a_stages, p.cn_smem, 4)) p.cn_smem = 0;
    if (!fits(p.a_stages, p.cn_smem, 2)) return fail(MXK_ERR_UNSUPPORTED, "gemm_mx: shared memory budget exceeded");
    p.b_stages = 2;
    while (p.b_stages < kMaxBStages && fits(p.a_stages, p.cn_smem, p.b_stages + 1)) ++p.b_stages;
    // At least 116 KB so that no second CTA shares the SM (each CTA holds all
    // 512 TMEM columns while it runs).
    const uint32_t smem_bytes =
        std::max<uint32_t>(smem_layout(p.kchunks, p.a_stages, p.cn_smem, p.b_stages).total + 1024, 116u * 1024u);
    if ((int)smem_bytes > max_smem) return fail(MXK_ERR_UNSUPPORTED, "gemm_mx: shared memory budget exceeded");

    const int64_t tiles_m = (m + kBM - 1) / kBM;
    const int grid = (int)std::min<int64_t>(tiles_m, sm_count());

    // Row-major scales (the API layout) are converted once per call into the
    // atom layout the kernel bulk-copies; the temporaries are stream-ordered.
    uint8_t* tmp_atoms = nullptr;
    if (!scale_atoms) {
        MXK_REQUIRE(!rows_dev, "gemm_mx: device-side row counts need atom-layout scales");
        const int64_t a_bytes = (m + 127) / 128 * p.kchunks * kSfAtom;
        const int64_t b_bytes = (n + 127) / 128 * p.kchunks * kSfAtom;
        MXK_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&tmp_atoms), (size_t)(a_bytes + b_bytes), stream));
        const int sms = sm_count();
        {
            LaunchScope scope("scales_to_atoms", stream);
            scales_to_atoms_kernel<<<sms * 4, 256, 0, stream>>>(m, p.kchunks, a_scales, tmp_atoms, a_bytes / 4);
            scales_to_atoms_kernel<<<sms * 4, 256, 0, stream>>>(n, p.kchunks, b_scales, tmp_atoms + a_bytes, b_bytes / 4);
        }
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) {
            cudaFreeAsync(tmp_atoms, stream);
            return fail_cuda("scales_to_atoms_kernel", e);
        }
        p.a_scales = tmp_atoms;
        p.b_scales = tmp_atoms + a_bytes;
    }

    auto launch = [&](auto kernel, const char* name) -> int {
        MXK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bytes));
        LaunchScope scope(name, stream);
        kernel<<<grid, kThreads, smem_bytes, stream>>>(tmap_a, tmap_b, p);
        MXK_CUDA(cudaGetLastError());
        return MXK_OK;
    };
    int st;
    if (!argmin)
        st = launch(mx_gemm_kernel<false, false>, "mx_gemm_dense");
    else if (argmin->gaps)
        st = launch(mx_gemm_kernel<true, true>, "mx_gemm_argmin_gap");
    else
        st = launch(mx_gemm_kernel<true, false>, "mx_gemm_argmin");
    if (tmp_atoms) cudaFreeAsync(tmp_atoms, stream);
    return st;
}

}  // namespace mxk

extern "C" {

int mxk_gemm_mx(int bits, int64_t m, int64_t n, int k, const void* a, const uint8_t* a_scales, const uint8_t* b,
                const uint8_t* b_scales, float* out, void* stream) {
    return mxk::launch_gemm_mx(bits, m, n, k, a, a_scales, b, b_scales, out, nullptr, nullptr,
                               mxk::as_stream(stream));
}

int mxk_assign_mx_fused(int bits, int64_t rows, int k, int d, const void* a, const uint8_t* a_scales,
                        const uint8_t* b, const uint8_t* b_scales, const float* point_norms,
                        const float* centroid_norms, const int* pid, int* labels, float* gaps,
                        const int* start_hint, void* stream) {
    mxk::MxArgmin am;
    am.point_norms = point_norms;
    am.centroid_norms = centroid_norms;
    am.pid = pid;
    am.labels = labels;
    am.gaps = gaps;
    am.start_hint = start_hint;
    return mxk::launch_gemm_mx(bits, rows, k, d, a, a_scales, b, b_scales, nullptr, &am, nullptr,
                               mxk::as_stream(stream));
}

}  // extern "C"
