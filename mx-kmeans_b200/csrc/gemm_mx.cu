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
// Structure (one persistent CTA per SM, 512 threads = 4 warpgroups):
//   warp 0      producer: TMA (SWIZZLE_128B) of a 128-row point tile (all K,
//               resident while every centroid tile streams past) and of
//               192-row x 128-byte centroid chunks through a ring as deep as
//               shared memory allows; 1-D bulk copies of the matching tcgen05
//               scale atoms (the quantizer writes scales in that layout;
//               row-major API scales are converted once per call).  The
//               centroid scales of small problems are copied into TMEM once.
//   warp 1      TMEM allocator and the single MMA-issuing thread:
//               tcgen05.mma kind::mxf8f6f4 block_scale (M=128, N=192, K=32)
//               into a two-stage TMEM accumulator ring (columns 0-383, scale
//               factors in 384-511), one tcgen05.commit per tile.
//   warps 2-3   idle (their warpgroup gives registers to the epilogue).
//   warps 4-15  epilogue, warp (q = w % 4, j = (w - 4) / 4): TMEM lane quadrant
//               q, columns [64 j, 64 j + 64) of every tile.  Dense store, or
//               argmin: a cheap key fmaf(-2, dot, cn) screens each 32-column
//               chunk and only chunks that can still win form the exact
//               distances fmaf(-2, dot, pn + cn) (packed f32x2, 3-input-min
//               tree, index search on improvement).  After each row tile's
//               first (hinted) centroid tile the quadrant's three warps swap
//               their minima; the j = 0 warp merges the three slices and writes
//               the label.  One warp hands centroid-ring slots back to the
//               producer once their tile's MMAs have completed.
// Argmin kernels rebalance registers with setmaxnreg (warpgroup 0: 80,
// epilogue warpgroups: 144).
#include <cstring>

#include "common.cuh"
#include "kernels.cuh"
#include "mx_codec.cuh"

namespace mxk {
namespace {

constexpr int kBM = kPointTileRows;      // points per tile = TMEM lanes
constexpr int kBN = kCentroidTileRows;   // centroids per accumulator tile (MMA N)
constexpr int kChunk = 128;              // K bytes per chunk = one SWIZZLE_128B row
constexpr int kATileBytes = kBM * kChunk;   // 16 KB
constexpr int kBTileBytes = kBN * kChunk;   // 24 KB
constexpr int kSfAtom = 512;             // 128 rows x 4 scale bytes
constexpr int kBAtoms = (kBN + 127) / 128;  // scale atoms per centroid-tile chunk
constexpr int kMaxBStages = 12;          // centroid-chunk ring depth: as many as shared memory holds
constexpr int kMaxAStages = 4;           // point-tile stages (4 when no FP32 staging takes the room)
constexpr int kAccStages = 2;            // 2 x 192 accumulator columns
constexpr int kEpiPerQuad = 3;  // epilogue warps per TMEM lane quadrant
constexpr int kSliceCols = kBN / kEpiPerQuad;  // accumulator columns per epilogue warp
constexpr int kSubChunks = kSliceCols / 32;    // 32-column TMEM loads per warp and tile
constexpr int kEpiWarps = 4 * kEpiPerQuad;
constexpr int kEpiWarp0 = 4;             // warpgroup 0: producer, MMA issuer, two quantizer warps
constexpr int kThreads = (kEpiWarp0 + kEpiWarps) * 32;
// Registers: one CTA per SM owns the whole register file.  With three epilogue
// warpgroups the kernel launches at 128 per thread and rebalances with
// setmaxnreg: warpgroup 0 drops to kLowRegs and the epilogue warpgroups rise to
// kHighRegs (per SM sub-partition 80 + 3 * 144 = 512 = 4 * 128 registers per
// lane, exactly the launch budget).  (Six epilogue warps per quadrant at 72
// registers each, for more latency hiding, spilled heavily.)
constexpr bool kRegSplit = kEpiPerQuad == 3;
constexpr int kLaunchRegs = (65536 / kThreads) / 8 * 8;
constexpr int kLowRegs = 80;
constexpr int kHighRegs = 144;
static_assert(!kRegSplit || kLowRegs + 3 * kHighRegs == 4 * kLaunchRegs,
              "register split must equal the launch budget");
constexpr int kMaxSmemNorms = 8192;      // centroid norms staged in shared memory up to this k
constexpr int kMaxChunks = 8;            // K <= 1024
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kSfaCol = kAccStages * kBN;  // 384: 4 columns per K chunk (<= 32)
constexpr uint32_t kSfbCol = kSfaCol + 32;       // 416: centroid scales, 4 columns per atom
constexpr int kSfbChunkCols = 4 * kBAtoms;       // TMEM columns per (centroid tile, K chunk)
constexpr int kMaxResidentSfb = (512 - (int)kSfbCol) / kSfbChunkCols;  // 12 (tile, chunk) pairs
constexpr int kNumBars = 80;             // mbarrier slots (see the kernel's carve-up); TMEM slot after them
static_assert(kSliceCols % 32 == 0 && kBN % kEpiPerQuad == 0, "each epilogue warp drains whole 32-column chunks");
static_assert(kSfbCol + kSfbChunkCols <= kTmemCols, "TMEM budget");

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
    int epi_release;  // ring slots are freed by the epilogue per tile (ring holds >= 2 tiles),
                      // else by the MMA thread per chunk
    int sfb_resident; // every centroid scale atom sits in TMEM for the whole kernel (tiles_n *
                      // kchunks <= kMaxResidentSfb); else each ring slot carries its tile's atoms
    int sfb_atoms;    // scale atoms in the shared-memory centroid-scale region
    int fuse_x;       // the point tile is quantized in the kernel from FP32 rows (tmap_x, D = 128,
                      // MXFP8): gathered by pid, encoded exactly as quantize_rows, no separate pass
    int64_t xrows;    // rows of the FP32 point matrix (a gather at this row reads zeros)
    const float* pn;
    const float* cn;
    const int* pid;
    int* labels;
    float* gaps;
    const int* start_hint;  // optional: a label per point; each tile's sweep starts at its first row's tile
    // optional (argmin): per point tile, the centroid tiles that can hold one of
    // its rows' nearest centroids (bit t = tile t; the others are neither loaded,
    // multiplied nor scanned).  Every bit set when null.  Needs tiles_n <= 64.
    const uint64_t* tile_mask;
    unsigned long long* tiles_done;  // count of multiplied 128 x 192 tiles (all K chunks)
    unsigned long long* rows_done;   // count of processed point rows
    float* best_dist;  // optional (argmin): each point's distance to its nearest centroid, at
    int best_dist_stride;  // best_dist[point * best_dist_stride] (and MxArgmin::second_bound's at + 1)
    const float4* row_bound;  // optional (argmin): MxArgmin::row_bound
    int by_row;               // MxArgmin::by_row
    int* row_labels;          // MxArgmin::row_labels
    const float* bmax32;      // MxArgmin::beta_max32 (kSec kernels)
    int4* changes;            // optional (argmin, with row_bound): MxArgmin::changes
    int* change_count;
    unsigned* err;
};

// Position in a ring of n slots whose use count crosses a phase every n uses.
struct RingPos {
    int slot;
    uint32_t phase;
    int n;
    __device__ __forceinline__ void advance(int k) {
        slot += k;
        while (slot >= n) slot -= n, phase ^= 1u;
    }
};

struct SmemLayout {
    uint32_t a_off, b_off, x_off, sfa_off, sfb_off, merge_off, seed_off, cn_off, bar_off, total;
};

// cn_floats: centroid norms staged in shared memory (0 when read from global).
// sfb_atoms: centroid scale atoms held in shared memory -- all of them (resident
// mode, staged once) or kBAtoms per ring slot.
__host__ __device__ inline SmemLayout smem_layout(int kchunks, int a_stages, int cn_floats, int b_stages,
                                                  int sfb_atoms, int fuse_x) {
    SmemLayout s;
    s.a_off = 0;  // every operand tile starts on a 1024-byte boundary (SWIZZLE_128B atoms)
    s.b_off = s.a_off + a_stages * kchunks * kATileBytes;
    s.x_off = s.b_off + b_stages * kBTileBytes;   // FP32 staging of one point tile (fused quantize)
    s.sfa_off = s.x_off + (fuse_x ? kBM * kChunk * 4 : 0);
    s.sfb_off = s.sfa_off + a_stages * kchunks * kSfAtom;
    s.merge_off = s.sfb_off + sfb_atoms * kSfAtom;  // [2 buffers][kEpiPerQuad - 1 depositors][128 rows] x 16 B
    s.seed_off = s.merge_off + 2 * (kEpiPerQuad - 1) * kBM * 16;  // [2 buffers][kEpiPerQuad warps][128 rows] x 8 B
    s.cn_off = s.seed_off + 2 * kEpiPerQuad * kBM * 8;
    s.bar_off = s.cn_off + (uint32_t)((cn_floats * 4 + 15) / 16 * 16);
    s.total = s.bar_off + kNumBars * 8 + 128;  // barriers, then TMEM slot, abort flag, sweep starts, norm maxima
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

// Row-major scales [rows][k/32] -> tcgen05 scale atoms for tiles of tile_rows
// rows: ceil(tile_rows / 128) 512-byte atoms per (tile, 128-feature chunk),
// tile-major, slice row r's four block scales at (r % 32) * 16 + (r / 32) * 4 +
// block % 4; rows past `rows` (and slice rows past the tile) get 0 (2^-127).
__global__ void __launch_bounds__(256) scales_to_atoms_kernel(int64_t rows, int kchunks, int tile_rows,
                                                              const uint8_t* __restrict__ src,
                                                              uint8_t* __restrict__ atoms, int64_t n_words) {
    const int per_tile = (tile_rows + 127) >> 7;
    for (int64_t w = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; w < n_words; w += (int64_t)gridDim.x * blockDim.x) {
        // word w = atom a, 32-bit slot (lane l, row group i): slice rows r = l + 32 i
        const int64_t a = w >> 7;
        const int slot = (int)(w & 127);
        const int l = slot >> 2, i = slot & 3;
        const int64_t tk = a / per_tile;  // (tile, chunk) pair
        const int slice = (int)(a - tk * per_tile);
        const int64_t tile = tk / kchunks;
        const int kc = (int)(tk - tile * kchunks);
        const int rr = slice * 128 + l + 32 * i;
        const int64_t row = tile * tile_rows + rr;
        uint32_t v = 0;
        if (rr < tile_rows && row < rows) v = *reinterpret_cast<const uint32_t*>(src + row * (int64_t)kchunks * 4 + 4 * kc);
        reinterpret_cast<uint32_t*>(atoms)[w] = v;
    }
}

// Sweep start: every 128-row point tile sweeps the centroid tiles beginning with
// the one holding the hint label of its first row (the driver passes the
// previous iteration's labels, and rows are ordered by them, so that tile usually
// holds every row's nearest centroid and later chunks rarely improve a row).
// Any start gives the same result: ties are broken by index, not by sweep order.

// Centroid norms: staged in shared memory (read with ld.shared through the
// shared-window address) or read from global memory.
template <bool kShared>
struct NormSrc {
    const float* g;   // global norms
    uint32_t s;       // shared-window address of the staged norms
    __device__ __forceinline__ float4 load4(int c) const {
        if constexpr (kShared) return dev::lds_f4(s + 4u * (uint32_t)c);
        else return __ldg(reinterpret_cast<const float4*>(g + c));
    }
    __device__ __forceinline__ float load1(int c) const {
        if constexpr (kShared) return dev::lds_f1(s + 4u * (uint32_t)c);
        else return __ldg(g + c);
    }
};

// Label of a row minimum that holds no centroid yet (its distance may be a
// bound rather than a candidate's).
constexpr int kNoLabel = 0x7fffffff;

// Running (distance, index) minimum and two largest distances of one row;
// sec (kSec kernels): the smallest key seen, in the units of the screen's keys
// fmaf(-2, dot, cn) -- a screened chunk's k_min, an exact distance less pn --
// over every centroid other than the current minimum's.
struct RowMin {
    float first, largest, next;
    int best;
    float sec;
};

// Folds 32 consecutive columns c0..c0+31 (all < n) of one row into `m`:
// distances fmaf(-2, dot, pn + cn) two at a time (add/fma .f32x2, each lane
// rounded exactly like the scalar operations), a 3-input-min tree, and an index
// search only when the chunk minimum can change the running minimum (smaller,
// or equal, resolved by the lower index as insert_distance does).  NaN
// distances never compare, as in the reference.
// force: evaluate the chunk even when its minimum exceeds m.first, taking it if
// m holds no centroid yet (m.first is then only a bound).  kSec: the columns
// that are not (or no longer) the minimum lower m.sec.
template <bool kGaps, bool kSec, class Norms>
__device__ __forceinline__ void argmin_chunk32(const uint32_t (&v)[32], const Norms& cn, float2 pn2, int c0,
                                               RowMin& m, bool force = false, float pn = 0.0f) {
    float dist[32];
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
        const float4 cv = cn.load4(c0 + j);
        dev::dist2(v[j], v[j + 1], pn2, cv.x, cv.y, dist[j], dist[j + 1]);
        dev::dist2(v[j + 2], v[j + 3], pn2, cv.z, cv.w, dist[j + 2], dist[j + 3]);
    }
    if constexpr (kGaps) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            m.next = fmaxf(m.next, fminf(m.largest, dist[j]));
            m.largest = fmaxf(m.largest, dist[j]);
        }
    }
    float m3[11];
#pragma unroll
    for (int t = 0; t < 10; ++t) m3[t] = dev::min3f(dist[3 * t], dist[3 * t + 1], dist[3 * t + 2]);
    m3[10] = fminf(dist[30], dist[31]);
    const float ma = dev::min3f(m3[0], m3[1], m3[2]);
    const float mb = dev::min3f(m3[3], m3[4], m3[5]);
    const float mc = dev::min3f(m3[6], m3[7], m3[8]);
    const float cm = fminf(dev::min3f(ma, mb, mc), fminf(m3[9], m3[10]));
    if (cm <= m.first || (force && cm == cm)) {
        int idx = 31;
#pragma unroll
        for (int j = 30; j >= 0; --j) idx = dist[j] == cm ? j : idx;
        const int cand = c0 + idx;
        if (cm < m.first || (cm == m.first && cand < m.best) || m.best == kNoLabel) {
            if constexpr (kSec) {  // the chunk's other columns and the previous minimum
                const float inf = __int_as_float(0x7f800000);
                float s2 = inf;
#pragma unroll
                for (int j = 0; j < 32; j += 2)
                    s2 = dev::min3f(s2, j == idx ? inf : dist[j], j + 1 == idx ? inf : dist[j + 1]);
                if (m.best != kNoLabel) s2 = fminf(s2, m.first);
                m.sec = fminf(m.sec, s2 - pn);
            }
            m.first = cm;
            m.best = cand;
            return;
        }
    }
    if constexpr (kSec) m.sec = fminf(m.sec, cm - pn);  // no column of the chunk is the minimum
}

// argmin_chunk32 behind a cheap screen.  Keys k_j = fmaf(-2, dot_j, cn_j) need
// one FP32 operation per column instead of two; the exact distances
// d_j = fmaf(-2, dot_j, pn + cn_j) are formed only when the chunk could still
// reach the row's running minimum.  Rounding bound: each d_j and k_j carries at
// most a few units of 2^-24 of the magnitudes S = pn + max(cn) + |k_min| + |first|
// and of its own excess over k_min, so d_j > first for every j in the chunk once
// pn + k_min - 2^-20 * S > first.  Skipping then changes nothing: the result is
// bit-identical to argmin_chunk32 alone.  NaN or infinite inputs fail the test
// and take the exact path.  pc = pn + max(cn).  kSec: a screened-out chunk
// lowers m.sec to its k_min (each d_j >= pn + k_min - 2^-18 (pc + |k_min|) by
// the same rounding argument).
template <bool kSec, class Norms>
__device__ __forceinline__ void argmin_chunk32_screened(const uint32_t (&v)[32], const Norms& cn, float2 pn2,
                                                        float pn, float pc, int c0, RowMin& m, bool force) {
    // keys folded into two running 3-input minima as they are formed (few live registers)
    float ka = __int_as_float(0x7f800000), kb = ka;
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
        const float4 cv = cn.load4(c0 + j);
        float k0, k1, k2, k3;
        dev::key2(v[j], v[j + 1], cv.x, cv.y, k0, k1);
        dev::key2(v[j + 2], v[j + 3], cv.z, cv.w, k2, k3);
        ka = dev::min3f(ka, k0, k1);
        kb = dev::min3f(kb, k2, k3);
    }
    const float kmin = fminf(ka, kb);
    const float scale = pc + fabsf(kmin) + fabsf(m.first);
    if (!force && fmaf(-0x1p-20f, scale, pn + kmin) > m.first) {
        if constexpr (kSec) m.sec = fminf(m.sec, kmin);
        return;
    }
    argmin_chunk32<false, kSec>(v, cn, pn2, c0, m, force, pn);
}

// Columns c0.. of a 32-column chunk that runs past n: one column at a time
// (column `forced` is taken while m holds no centroid, as in argmin_chunk32).
template <bool kGaps, bool kSec, class Norms>
__device__ __forceinline__ void argmin_tail(const uint32_t (&v)[32], const Norms& cn, float pn, int c0, int64_t n,
                                            RowMin& m, int forced) {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        if (c0 + j < n) {
            const float dist = fmaf(-2.0f, __uint_as_float(v[j]), pn + cn.load1(c0 + j));
            if (dist < m.first || (dist == m.first && c0 + j < m.best) ||
                (c0 + j == forced && m.best == kNoLabel && dist == dist)) {
                if constexpr (kSec)
                    if (m.best != kNoLabel) m.sec = fminf(m.sec, m.first - pn);
                m.first = dist;
                m.best = c0 + j;
            } else if constexpr (kSec) {
                m.sec = fminf(m.sec, dist - pn);
            }
            if constexpr (kGaps) {
                m.next = fmaxf(m.next, fminf(m.largest, dist));
                m.largest = fmaxf(m.largest, dist);
            }
        }
    }
}

// One 32-column chunk of a row starting at column cc: screened fast path, the
// exact path when gaps are needed, one column at a time past n.  The chunk
// holding column `forced` (the row's previous label, or -1) is always
// evaluated exactly, so a row whose minimum starts at a bound finds a centroid.
// screen: take the key screen first (else every chunk takes the exact path,
// cheaper when most chunks would fail the screen anyway -- rows without a
// sweep hint or bound, whose minima still improve often).
template <bool kGaps, bool kSec, class Norms>
__device__ __forceinline__ void fold_chunk(const uint32_t (&v)[32], const Norms& cn, float2 pn2, float pn, float pc,
                                           int cc, int64_t n, RowMin& m, int forced, bool screen = true) {
    if (cc + 32 <= n) {
        if constexpr (kGaps)
            argmin_chunk32<true, false>(v, cn, pn2, cc, m);
        else if (screen)
            argmin_chunk32_screened<kSec>(v, cn, pn2, pn, pc, cc, m, (unsigned)(forced - cc) < 32u);
        else
            argmin_chunk32<false, kSec>(v, cn, pn2, cc, m, (unsigned)(forced - cc) < 32u, pn);
    } else if (cc < n) {
        argmin_tail<kGaps, kSec>(v, cn, pn, cc, n, m, forced);
    }
}

// Lexicographic (distance, index) minimum and two-largest merge of a partial
// result (d, b, l, nx) into m; a partial without a centroid never displaces one.
// kSec: the partial's key bound s and whichever candidate loses (if it is
// another centroid; its distance less pn) lower m.sec.
template <bool kGaps, bool kSec = false>
__device__ __forceinline__ void merge_rowmin(RowMin& m, float d, int b, float l, float nx, float s = 0.0f,
                                             float pn = 0.0f) {
    const bool take = b != kNoLabel && (d < m.first || (d == m.first && b < m.best) || m.best == kNoLabel);
    if constexpr (kSec) {
        if (take) {
            if (m.best != kNoLabel && m.best != b) m.sec = fminf(m.sec, m.first - pn);
        } else if (b != kNoLabel && b != m.best) {
            m.sec = fminf(m.sec, d - pn);
        }
        m.sec = fminf(m.sec, s);
    }
    if (take) m.first = d, m.best = b;
    if constexpr (kGaps) {
        m.next = fmaxf(fminf(m.largest, l), fmaxf(m.next, nx));
        m.largest = fmaxf(m.largest, l);
    }
}

template <bool kArgmin, bool kGaps, bool kSec = false>
__global__ void __launch_bounds__(kThreads, 1)
    mx_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                   const __grid_constant__ CUtensorMap tmap_x, const GemmParams p) {
    static_assert(!kSec || (kArgmin && !kGaps), "the second-nearest bound is an argmin-only, gap-free output");
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const SmemLayout L = smem_layout(p.kchunks, p.a_stages, p.cn_smem, p.b_stages, p.sfb_atoms, p.fuse_x);
    const int kBStages = p.b_stages;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bar_off);
    uint64_t* a_full = bars;                 // [kMaxAStages]
    uint64_t* a_empty = bars + kMaxAStages;  // [kMaxAStages]
    uint64_t* b_full = bars + 2 * kMaxAStages;  // [kMaxBStages]
    uint64_t* b_empty = b_full + kMaxBStages;
    uint64_t* acc_full = b_empty + kMaxBStages;  // [kAccStages]
    uint64_t* acc_empty = acc_full + kAccStages;
    uint64_t* drain = acc_empty + kAccStages;
    uint64_t* merge_full = drain + 1;        // [q * 2 + row-tile parity] two depositing warps -> merging warp
    uint64_t* merge_empty = merge_full + 8;  // [q * 2 + row-tile parity] merging warp has read the deposits
    uint64_t* seed_bar = merge_empty + 8;    // [q] the quadrant's three first-tile minima are published
    uint64_t* sfb_full = seed_bar + 4;       // resident centroid scales have landed in shared memory
    uint64_t* x_full = sfb_full + 1;         // [8] 16 FP32 rows of a quantizer warp gathered (fused quantize)
    uint64_t* x_empty = x_full + 8;          // [8] the quantizer warp has encoded those rows
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + kNumBars) + 1;
    // after the barriers (32 words): [0] TMEM slot, [1] abort flag, [2, 6) sweep
    // starts per A stage, [6, 6 + 16) per-warp centroid-norm maxima, [24, 32) the
    // point tile's centroid-tile mask per A stage (64-bit, published with sweep0)
    volatile int* sweep0 = reinterpret_cast<volatile int*>(bars + kNumBars) + 2;  // [kMaxAStages]
    float* warp_cmax = reinterpret_cast<float*>(bars + kNumBars) + 2 + kMaxAStages;  // [kThreads / 32]
    volatile unsigned long long* sweep_mask = reinterpret_cast<volatile unsigned long long*>(bars + kNumBars) + 12;
    static_assert(2 * kMaxAStages + 2 * kMaxBStages + 2 * kAccStages + 1 + 16 + 4 + 1 + 16 <= kNumBars,
                  "barrier slots");
    static_assert(2 + kMaxAStages + kThreads / 32 <= 24 && 24 + 2 * kMaxAStages <= 32, "words after the barriers");

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t mrows = p.m_dev ? (int64_t)*p.m_dev : p.m;
    const int64_t tiles_m = (mrows + kBM - 1) / kBM;
    const int tiles_n = (int)((p.n + kBN - 1) / kBN);

    if (threadIdx.x == 0 && blockIdx.x == 0 && p.rows_done) atomicAdd(p.rows_done, (unsigned long long)mrows);
    if (threadIdx.x == 0) {
        // fused quantize: the two quantizer warps arrive
        for (int i = 0; i < kMaxAStages; ++i)
            dev::mbar_init(&a_full[i], p.fuse_x ? 2 : 1), dev::mbar_init(&a_empty[i], 1);
        for (int i = 0; i < kBStages; ++i) dev::mbar_init(&b_full[i], 1), dev::mbar_init(&b_empty[i], 1);
        for (int i = 0; i < kAccStages; ++i)
            dev::mbar_init(&acc_full[i], 1), dev::mbar_init(&acc_empty[i], kEpiWarps);
        dev::mbar_init(drain, 1);
        for (int i = 0; i < 8; ++i) {
            dev::mbar_init(&merge_full[i], kEpiPerQuad - 1);
            dev::mbar_init(&merge_empty[i], 1);
        }
        for (int q = 0; q < 4; ++q) dev::mbar_init(&seed_bar[q], kEpiPerQuad);
        dev::mbar_init(sfb_full, 1);
        for (int i = 0; i < 8; ++i) dev::mbar_init(&x_full[i], 1), dev::mbar_init(&x_empty[i], 1);
        *abort_flag = 0;
        dev::fence_barrier_init();
    }
    if (warp == 1) dev::tmem_alloc(tmem_slot, kTmemCols);
    if (kArgmin) {
        // centroid norms -> shared memory (when they fit) and their maximum
        float* cn_s = reinterpret_cast<float*>(smem + L.cn_off);
        float cmax = 0.0f;
        for (int i = threadIdx.x; i < p.n; i += blockDim.x) {
            const float c = p.cn[i];
            if (p.cn_smem) cn_s[i] = c;
            cmax = c > cmax || c != c ? c : cmax;  // NaN propagates (and disables the screen)
        }
        for (int o = 16; o; o >>= 1) {
            const float other = __shfl_xor_sync(0xffffffffu, cmax, o);
            cmax = other > cmax || other != other ? other : cmax;
        }
        if (lane == 0) warp_cmax[warp] = cmax;
    }
    if (warp == 0 && lane == 0) {
        if (p.fuse_x) dev::prefetch_tensor_map(&tmap_x);
        else if (p.a_bits == 8) dev::prefetch_tensor_map(&tmap_a);
        dev::prefetch_tensor_map(&tmap_b);
    }
    dev::tc_fence_before();
    __syncthreads();
    dev::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp < kEpiWarp0) {
    if constexpr (kArgmin && kRegSplit) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kLowRegs));
    if (warp == 0) {
        // ------------------------------------------------------------ producer
        RingPos bring{0, 0u, kBStages};
        uint32_t issued = 0;
        int it = 0;
        bool ok = true;
        if (p.sfb_resident && lane == 0) {
            const uint32_t bytes = (uint32_t)(p.sfb_atoms * kSfAtom);
            dev::mbar_arrive_expect_tx(sfb_full, bytes);
            dev::bulk_load(smem + L.sfb_off, p.b_scales, bytes, sfb_full);
        }
        // Sweep starts come from two dependent global loads (the lead row's point
        // id, then its hint); they are software-pipelined two row tiles ahead.
        const int64_t step = gridDim.x;
        auto lead_id = [&](int64_t t) -> int64_t {
            if (!p.start_hint || t >= tiles_m || lane != 0) return -1;
            return p.pid ? (int64_t)p.pid[t * kBM] : t * kBM;
        };
        auto hint_of = [&](int64_t id) -> int { return id >= 0 ? p.start_hint[id] : -1; };
        auto mask_of = [&](int64_t t) -> uint64_t {  // (lane 0 only) centroid tiles of point tile t
            return p.tile_mask && t < tiles_m && lane == 0 ? p.tile_mask[t] : ~0ull;
        };
        uint32_t xf_issued = 0;  // (fused quantize) bit G: staging group G has been gathered
        uint32_t xf_par = 0;     // bit G: number of gathers into group G, mod 2
        if (p.fuse_x) {
            // Fused quantize: this warp also refills the quantizers' FP32 staging.
            // Two streams are served as their barriers allow: centroid tiles into
            // the B ring, and the next row tile's point rows into each 16-row
            // staging group a quantizer warp has released (x_empty), in the order
            // the two warps consume them (0, 4, 1, 5, ...).  The rows' point ids
            // are loaded one group ahead, the centroid-tile masks and sweep starts
            // one and two row tiles ahead, so neither stream waits on a global load.
            constexpr uint32_t kGroupBytes = 16u * kChunk * 4u;
            auto group_of = [](int k) { return (k & 1) * 4 + (k >> 1); };
            int64_t gt = blockIdx.x;  // row tile being gathered
            int gk = 0;               // position of the next group in the consumption order
            uint32_t xe_par = 0xffu;  // bit G: parity awaited on x_empty[G] (a fresh barrier passes 1)
            int32_t y[4] = {0, 0, 0, 0};
            auto load_ids = [&](int64_t t, int G) {
                if (lane < 4) {
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int64_t g = t * kBM + 16 * G + 4 * lane + u;
                        y[u] = g < mrows ? (p.pid ? p.pid[g] : (int32_t)g) : (int32_t)p.xrows;  // past the end: zeros
                    }
                }
            };
            bool g_more = gt < tiles_m;
            if (g_more) load_ids(gt, group_of(0));
            // centroid stream (lane 0): row tile bt, sweep position bi
            int64_t bt = blockIdx.x;
            int bi = 0;
            auto ct0_of = [&](int h) { return h >= 0 && (int64_t)h < p.n ? h / kBN : 0; };
            int ct0 = ct0_of(hint_of(lead_id(bt)));
            uint64_t bmask = mask_of(bt);
            int hint_nxt = hint_of(lead_id(bt + step));
            uint64_t mask_nxt = mask_of(bt + step);
            int64_t lead_nn = lead_id(bt + 2 * step);
            auto next_b = [&]() -> bool {  // (lane 0) advance to the next centroid tile to load
                while (bt < tiles_m) {
                    for (; bi < tiles_n; ++bi) {
                        const int ct = ct0 + bi < tiles_n ? ct0 + bi : ct0 + bi - tiles_n;
                        if ((bmask >> ct) & 1ull) return true;
                    }
                    bt += step;
                    bi = 0;
                    ct0 = ct0_of(hint_nxt);
                    bmask = mask_nxt;
                    hint_nxt = hint_of(lead_nn);
                    mask_nxt = mask_of(bt + step);
                    lead_nn = lead_id(bt + 2 * step);
                }
                return false;
            };
            bool b_more = __shfl_sync(0xffffffffu, lane == 0 ? (int)next_b() : 0, 0) != 0;
            long long idle_since = clock64();
            while (g_more || b_more) {
                bool progressed = false;
                if (g_more) {
                    const int G = group_of(gk);
                    const int ready = __shfl_sync(
                        0xffffffffu, lane == 0 ? (int)dev::mbar_test(&x_empty[G], (xe_par >> G) & 1u) : 0, 0);
                    if (ready) {
                        xe_par ^= 1u << G;
                        if (lane == 0) dev::mbar_arrive_expect_tx(&x_full[G], kGroupBytes);
                        __syncwarp();
                        if (lane < 4)  // staging rows 16 G + 4 lane .. + 3: inside the 64 KB buffer
                            dev::tma_gather4(smem + L.x_off + (uint32_t)(16 * G + 4 * lane) * kChunk * 4u, &tmap_x, 0,
                                             y[0], y[1], y[2], y[3], &x_full[G]);
                        xf_issued |= 1u << G;
                        xf_par ^= 1u << G;
                        if (++gk == 8) gk = 0, gt += step;
                        g_more = gt < tiles_m;
                        if (g_more) load_ids(gt, group_of(gk));
                        progressed = true;
                    }
                }
                if (b_more) {
                    const int ready = __shfl_sync(
                        0xffffffffu, lane == 0 ? (int)dev::mbar_test(&b_empty[bring.slot], bring.phase ^ 1u) : 0, 0);
                    if (ready) {
                        int more = 0;
                        if (lane == 0) {
                            const int ct = ct0 + bi < tiles_n ? ct0 + bi : ct0 + bi - tiles_n;
                            uint64_t* full = &b_full[bring.slot];
                            dev::mbar_arrive_expect_tx(
                                full, (uint32_t)(kBTileBytes + (p.sfb_resident ? 0 : kBAtoms * kSfAtom)));
                            dev::tma_load_2d(smem + L.b_off + bring.slot * kBTileBytes, &tmap_b, 0, ct * kBN, full);
                            if (!p.sfb_resident)
                                dev::bulk_load(smem + L.sfb_off + bring.slot * kBAtoms * kSfAtom,
                                               p.b_scales + (int64_t)ct * kBAtoms * kSfAtom, kBAtoms * kSfAtom, full);
                            ++issued;
                            bring.advance(1);
                            ++bi;
                            more = next_b();
                        }
                        b_more = __shfl_sync(0xffffffffu, more, 0) != 0;
                        progressed = true;
                    }
                }
                if (progressed) {
                    idle_since = clock64();
                } else {
                    // nothing to issue: back off briefly (this warp shares its
                    // scheduler with epilogue warps), give up on an abort or a
                    // wait past the limit
                    int quit = 0;
                    if (lane == 0) {
                        if (*abort_flag) {
                            quit = 1;
                        } else if (clock64() - idle_since > dev::kWaitLimitCycles) {
                            *abort_flag = 1;
                            if (p.err) atomicOr(p.err, 1u << MXK_ERR_TIMEOUT);
                            quit = 1;
                        }
                    }
                    if (__shfl_sync(0xffffffffu, quit, 0)) {
                        ok = false;
                        break;
                    }
                    __nanosleep(20);
                }
            }
        }
        int hint_cur = hint_of(lead_id(blockIdx.x));
        int64_t lead_nxt = lead_id(blockIdx.x + step);
        uint64_t mask_nxt = mask_of(blockIdx.x);
        for (int64_t tile = blockIdx.x; tile < tiles_m && ok && !p.fuse_x; tile += gridDim.x, ++it) {
            const int ct0 = hint_cur >= 0 && (int64_t)hint_cur < p.n ? hint_cur / kBN : 0;
            const uint64_t tmask = mask_nxt;
            hint_cur = hint_of(lead_nxt);
            lead_nxt = lead_id(tile + 2 * step);
            mask_nxt = mask_of(tile + step);
            const int as = it % p.a_stages;
            const uint32_t aph = (uint32_t)(it / p.a_stages) & 1u;
            if (!dev::mbar_wait(&a_empty[as], aph ^ 1u, abort_flag, p.err)) { ok = false; break; }
            uint8_t* a_smem = smem + L.a_off + (uint32_t)as * p.kchunks * kATileBytes;
            uint8_t* sfa = smem + L.sfa_off + (uint32_t)as * p.kchunks * kSfAtom;
            if (lane == 0) {
                const uint32_t bytes = (p.a_bits == 8 ? p.kchunks * kATileBytes : 0) + p.kchunks * kSfAtom;
                if (bytes)
                    asm volatile("mbarrier.expect_tx.shared::cta.b64 [%0], %1;" ::"r"(dev::smem_addr(&a_full[as])),
                                 "r"(bytes));
                if (p.a_bits == 8)
                    for (int kc = 0; kc < p.kchunks; ++kc)
                        dev::tma_load_2d(a_smem + kc * kATileBytes, &tmap_a, kc * kChunk, (int32_t)(tile * kBM),
                                         &a_full[as]);
                dev::bulk_load(sfa, p.a_scales + tile * p.kchunks * kSfAtom, (uint32_t)(p.kchunks * kSfAtom),
                               &a_full[as]);
            }
            if (p.a_bits != 8)
                for (int kc = 0; kc < p.kchunks; ++kc)
                    fill_a_subbyte(a_smem + kc * kATileBytes, p, tile * kBM, kc, mrows, lane);
            if (lane == 0) sweep0[as] = ct0, sweep_mask[as] = tmask;  // published by the a_full arrival
            dev::fence_proxy_async();
            __syncwarp();
            if (lane == 0) dev::mbar_arrive(&a_full[as]);
            // Centroid chunks: one thread walks the ring.  A slot is handed back by
            // the epilogue once the tile that read it has completed, or by the MMA
            // thread's per-chunk commit when the ring holds less than two tiles.
            if (lane == 0) {
                for (int i = 0; i < tiles_n && ok; ++i) {
                    const int ct = ct0 + i < tiles_n ? ct0 + i : ct0 + i - tiles_n;
                    if (!((tmask >> ct) & 1ull)) continue;
                    for (int kc = 0; kc < p.kchunks; ++kc) {
                        if (!dev::mbar_wait(&b_empty[bring.slot], bring.phase ^ 1u, abort_flag, p.err)) {
                            ok = false;
                            break;
                        }
                        uint64_t* full = &b_full[bring.slot];
                        dev::mbar_arrive_expect_tx(
                            full, (uint32_t)(kBTileBytes + (p.sfb_resident ? 0 : kBAtoms * kSfAtom)));
                        dev::tma_load_2d(smem + L.b_off + bring.slot * kBTileBytes, &tmap_b, kc * kChunk, ct * kBN,
                                         full);
                        if (!p.sfb_resident)
                            dev::bulk_load(smem + L.sfb_off + bring.slot * kBAtoms * kSfAtom,
                                           p.b_scales + ((int64_t)ct * p.kchunks + kc) * kBAtoms * kSfAtom,
                                           kBAtoms * kSfAtom, full);
                        ++issued;
                        bring.advance(1);
                    }
                }
            }
            ok = __shfl_sync(0xffffffffu, (int)ok, 0) != 0;
        }
        // Unwinding after an abort: wait (bounded) for the copies this warp
        // issued, so no TMA write lands in shared memory after the CTA exits.
        if (!ok && lane == 0) {
            volatile int no_abort = 0;
            for (uint32_t c = issued > (uint32_t)kBStages ? issued - kBStages : 0; c < issued; ++c)
                dev::mbar_wait(&b_full[c % kBStages], (c / kBStages) & 1u, &no_abort, nullptr);
            if (p.fuse_x) {
                for (int G = 0; G < 8; ++G)
                    if ((xf_issued >> G) & 1u)
                        dev::mbar_wait(&x_full[G], ((xf_par >> G) & 1u) ^ 1u, &no_abort, nullptr);
            } else {
                for (int j = it > p.a_stages ? it - p.a_stages : 0; j <= it; ++j)
                    dev::mbar_wait(&a_full[j % p.a_stages], (uint32_t)(j / p.a_stages) & 1u, &no_abort, nullptr);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        // One thread issues every MMA (tcgen05.mma streams issued by two threads
        // at once gave wrong products on B200).  Its own instruction latency --
        // about 80 cycles per MMA and 250 per commit, the same for any N -- is
        // what limits a tile, hence the wide 192-column tiles, one commit per
        // tile, ring positions advanced incrementally and completed barriers
        // detected with a non-suspending test first.
        if (lane == 0) {
            RingPos brd{0, 0u, kBStages};
            uint32_t tiles_issued = 0;
            int s = 0;           // accumulator stage of tile a = a % 2
            uint32_t sph = 0;    // (a / 2) & 1
            int it = 0;
            bool ok = true;
            const uint32_t idesc0 = dev::mx_idesc(dev::kFmtE4M3, dev::kFmtE4M3, kBM, kBN, 0);
            if (p.sfb_resident) {
                // every (centroid tile, K chunk)'s scale atoms -> TMEM once
                if (!dev::mbar_wait(sfb_full, 0, abort_flag, p.err)) ok = false;
                const uint32_t base = dev::smem_addr(smem + L.sfb_off);
                for (int t = 0; t < p.sfb_atoms && ok; ++t)
                    dev::tc_copy_32x128b_x4(tmem + kSfbCol + 4 * t,
                                            dev::smem_desc(base + t * kSfAtom, 16, 128, dev::kLayoutNone));
            }
            const bool fast = p.kchunks == 1 && p.sfb_resident && p.epi_release;
            if (fast) {
                // D = 128 hot loop: one K chunk per tile, resident centroid scales,
                // ring slots freed by the epilogue -- per tile only the two
                // barrier tests, four MMAs and one commit remain.
                const uint64_t bdesc_base = dev::smem_desc(dev::smem_addr(smem + L.b_off), 16, 1024,
                                                           dev::kLayoutSwizzle128);
                const uint32_t sfa = tmem + kSfaCol;
                int slot = 0;
                uint32_t bph = 0;
                for (int64_t tile = blockIdx.x; tile < tiles_m && ok; tile += gridDim.x, ++it) {
                    const int as = it % p.a_stages;
                    const uint32_t aph = (uint32_t)(it / p.a_stages) & 1u;
                    if (!dev::mbar_wait_lean(&a_full[as], aph, abort_flag, p.err)) { ok = false; break; }
                    dev::tc_fence_after();
                    const uint32_t a_off = L.a_off + (uint32_t)as * kATileBytes;
                    dev::tc_copy_32x128b_x4(sfa, dev::smem_desc(dev::smem_addr(smem + L.sfa_off + (uint32_t)as * kSfAtom),
                                                                16, 128, dev::kLayoutNone));
                    const uint64_t adesc = dev::smem_desc(dev::smem_addr(smem + a_off), 16, 1024, dev::kLayoutSwizzle128);
                    int ct = sweep0[as];
                    const uint64_t tmask = sweep_mask[as];
                    uint32_t sfb = tmem + kSfbCol + (uint32_t)(ct * kSfbChunkCols);
                    for (int i = 0; i < tiles_n; ++i) {
                        if (!((tmask >> ct) & 1ull)) {  // pruned centroid tile
                            if (++ct == tiles_n) ct = 0, sfb = tmem + kSfbCol;
                            else sfb += kSfbChunkCols;
                            continue;
                        }
                        if (!dev::mbar_wait_lean(&acc_empty[s], sph ^ 1u, abort_flag, p.err)) { ok = false; break; }
                        dev::tc_fence_after();
                        if (!dev::mbar_wait_lean(&b_full[slot], bph, abort_flag, p.err)) { ok = false; break; }
                        const uint64_t bdesc = bdesc_base + (uint64_t)(slot * (kBTileBytes >> 4));
                        const uint32_t d = tmem + (s ? (uint32_t)kBN : 0u);
#pragma unroll
                        for (int kb = 0; kb < 4; ++kb)
                            dev::tc_mma_mx(d, adesc + 2u * kb, bdesc + 2u * kb, idesc0 | dev::mx_idesc_sf((uint32_t)kb),
                                           sfa | ((uint32_t)kb << 30), sfb | ((uint32_t)kb << 30), kb != 0);
                        dev::tc_commit(&acc_full[s]);
                        ++tiles_issued;
                        s ^= 1;
                        sph ^= (uint32_t)(s == 0);
                        if (++slot == kBStages) slot = 0, bph ^= 1u;
                        if (++ct == tiles_n) ct = 0, sfb = tmem + kSfbCol;
                        else sfb += kSfbChunkCols;
                    }
                    if (ok) dev::tc_commit(&a_empty[as]);
                }
            }
            for (int64_t tile = blockIdx.x; tile < tiles_m && ok && !fast; tile += gridDim.x, ++it) {
                const int as = it % p.a_stages;
                const uint32_t aph = (uint32_t)(it / p.a_stages) & 1u;
                if (!dev::mbar_wait_lean(&a_full[as], aph, abort_flag, p.err)) { ok = false; break; }
                dev::tc_fence_after();
                const uint32_t a_base = dev::smem_addr(smem + L.a_off + (uint32_t)as * p.kchunks * kATileBytes);
                const uint32_t sfa_base = dev::smem_addr(smem + L.sfa_off + (uint32_t)as * p.kchunks * kSfAtom);
                for (int kc = 0; kc < p.kchunks; ++kc)
                    dev::tc_copy_32x128b_x4(tmem + kSfaCol + 4 * kc,
                                            dev::smem_desc(sfa_base + kc * kSfAtom, 16, 128, dev::kLayoutNone));
                const uint64_t adesc0 = dev::smem_desc(a_base, 16, 1024, dev::kLayoutSwizzle128);
                int ct = sweep0[as];
                const uint64_t tmask = sweep_mask[as];
                for (int i = 0; i < tiles_n && ok; ++i, ct = ct + 1 == tiles_n ? 0 : ct + 1) {
                    if (!((tmask >> ct) & 1ull)) continue;  // pruned centroid tile
                    if (!dev::mbar_wait_lean(&acc_empty[s], sph ^ 1u, abort_flag, p.err)) { ok = false; break; }
                    dev::tc_fence_after();
                    const uint32_t d_tmem = tmem + (uint32_t)s * kBN;
                    for (int kc = 0; kc < p.kchunks; ++kc) {
                        if (!dev::mbar_wait_lean(&b_full[brd.slot], brd.phase, abort_flag, p.err)) { ok = false; break; }
                        uint32_t sfb_col = tmem + kSfbCol + (uint32_t)((ct * p.kchunks + kc) * kSfbChunkCols);
                        if (!p.sfb_resident) {
                            sfb_col = tmem + kSfbCol;
                            const uint32_t sfb = dev::smem_addr(smem + L.sfb_off + brd.slot * kBAtoms * kSfAtom);
#pragma unroll
                            for (int t = 0; t < kBAtoms; ++t)
                                dev::tc_copy_32x128b_x4(sfb_col + 4 * t,
                                                        dev::smem_desc(sfb + t * kSfAtom, 16, 128, dev::kLayoutNone));
                        }
                        // +32 bytes along K = +2 in a descriptor's address field
                        const uint64_t adesc = adesc0 + (uint64_t)(kc * (kATileBytes >> 4));
                        const uint64_t bdesc = dev::smem_desc(dev::smem_addr(smem + L.b_off + brd.slot * kBTileBytes),
                                                              16, 1024, dev::kLayoutSwizzle128);
#pragma unroll
                        for (int kb = 0; kb < 4; ++kb)
                            dev::tc_mma_mx(d_tmem, adesc + 2u * kb, bdesc + 2u * kb, idesc0 | dev::mx_idesc_sf((uint32_t)kb),
                                           (tmem + kSfaCol + 4 * kc) | ((uint32_t)kb << 30),
                                           sfb_col | ((uint32_t)kb << 30), (kc | kb) != 0);
                        if (!p.epi_release) dev::tc_commit(&b_empty[brd.slot]);
                        brd.advance(1);
                    }
                    if (!ok) break;
                    dev::tc_commit(&acc_full[s]);
                    ++tiles_issued;
                    if (++s == kAccStages) s = 0, sph ^= 1u;
                }
                if (ok) dev::tc_commit(&a_empty[as]);
            }
            // Make sure every issued MMA/copy has finished before TMEM is freed.
            if (p.tiles_done && ok) atomicAdd(p.tiles_done, (unsigned long long)tiles_issued);
            dev::tc_commit(drain);
            volatile int no_abort = 0;
            dev::mbar_wait(drain, 0, &no_abort, p.err);
        }
        __syncwarp();
    } else if (p.fuse_x) {
        // ------------------------------------------------------------ quantizers
        // Warps 2 and 3 encode the gathered FP32 rows (rows 64 (w-2) .. +63) into
        // the MXFP8 point tile and its scale atom, with the arithmetic of
        // quantize_rows: per 32-feature block the UE8M0 scale of amax / 448 (1 for
        // an all-zero block; computed from amax's bits, see ue8m0_mxfp8_scale),
        // values times its exact reciprocal, E4M3 round-to-nearest-even saturating.
        // One lane owns one (row, block) pair per pass of 8 rows: lane L takes
        // row 8 g + (L & 7) and block L >> 3, so the block maximum needs no
        // shuffle.  The staging rows are 512 B apart; lane L reads its eight
        // 16-byte chunks starting at chunk (L & 7), so the 8 lanes of each
        // shared-memory phase hit 8 different bank groups.
        // The warp's 64 staging rows form 4 groups of 16 with two barriers each:
        // the producer warp gathers a group's rows (x_full) and refills it with
        // the next row tile's as soon as this warp has encoded it (x_empty), so
        // the copies overlap the encoding.
        constexpr int kRowsPerWarp = kBM / 2;  // 64
        constexpr int kGroupRows = 16;
        constexpr int kGroups = kRowsPerWarp / kGroupRows;  // 4
        static_assert(2 * kRowsPerWarp == kBM && kChunk == 128 && kGroups * kGroupRows == kRowsPerWarp,
                      "quantizer row split");
        const int r0 = (warp - 2) * kRowsPerWarp;
        uint64_t* xf = x_full + (warp - 2) * kGroups;
        uint64_t* xe = x_empty + (warp - 2) * kGroups;
        uint32_t xphase = 0;  // bit G: parity of group G's next completion
        // sweep starts and centroid-tile masks (warp 2 publishes them), pipelined
        // like the producer's
        const int64_t step = gridDim.x;
        const bool lead_lane = lane == 0 && warp == 2;
        auto lead_id = [&](int64_t t) -> int64_t {
            if (!p.start_hint || t >= tiles_m || !lead_lane) return -1;
            return p.pid ? (int64_t)p.pid[t * kBM] : t * kBM;
        };
        auto hint_of = [&](int64_t id) -> int { return id >= 0 ? p.start_hint[id] : -1; };
        auto mask_of = [&](int64_t t) -> uint64_t {
            return p.tile_mask && t < tiles_m && lead_lane ? p.tile_mask[t] : ~0ull;
        };
        int hint_cur = hint_of(lead_id(blockIdx.x));
        int64_t lead_nxt = lead_id(blockIdx.x + step);
        uint64_t mask_cur = mask_of(blockIdx.x);
        bool ok = true;
        int it = 0;
        const int blk = lane >> 3;      // 32-feature block of this lane
        const uint32_t rot = lane & 7;  // first chunk read (row % 8 of this lane's rows)
        const uint32_t xbase = dev::smem_addr(smem + L.x_off) + (uint32_t)(r0 + (lane & 7)) * (kChunk * 4) +
                               (uint32_t)blk * 128u;
        for (int64_t tile = blockIdx.x; tile < tiles_m && ok; tile += gridDim.x, ++it) {
            const int ct0 = hint_cur >= 0 && (int64_t)hint_cur < p.n ? hint_cur / kBN : 0;
            const uint64_t tmask = mask_cur;
            hint_cur = hint_of(lead_nxt);
            lead_nxt = lead_id(tile + 2 * step);
            mask_cur = mask_of(tile + step);
            const int as = it % p.a_stages;
            const uint32_t aph = (uint32_t)(it / p.a_stages) & 1u;
            if (!dev::mbar_wait(&a_empty[as], aph ^ 1u, abort_flag, p.err)) { ok = false; break; }
            const uint32_t a_tile = dev::smem_addr(smem + L.a_off + (uint32_t)as * kATileBytes);
            const uint32_t sfa = dev::smem_addr(smem + L.sfa_off + (uint32_t)as * kSfAtom);
            for (int grp = 0; grp < kGroups && ok; ++grp) {
                if (!dev::mbar_wait(&xf[grp], (xphase >> grp) & 1u, abort_flag, p.err)) { ok = false; break; }
                xphase ^= 1u << grp;
#pragma unroll 1
                for (int pass = 0; pass < kGroupRows / 8; ++pass) {
                    const int rbase = r0 + grp * kGroupRows + pass * 8;  // multiple of 8
                    const int r = rbase + (lane & 7);
                    const uint32_t src = xbase + (uint32_t)(grp * kGroupRows + pass * 8) * (kChunk * 4);
                    float4 x[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) x[i] = dev::lds_f4(src + 16u * ((rot + i) & 7u));
                    // fmaxf drops NaN in any order; starting from 0 the maximum is never NaN or -0
                    float m[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        m[i] = fmaxf(fmaxf(fabsf(x[i].x), fabsf(x[i].y)), fmaxf(fabsf(x[i].z), fabsf(x[i].w)));
                    const float amax = fmaxf(fmaxf(fmaxf(fmaxf(0.0f, m[0]), fmaxf(m[1], m[2])),
                                                   fmaxf(m[3], m[4])),
                                             fmaxf(fmaxf(m[5], m[6]), m[7]));
                    bool rare;
                    uint32_t sc = dev::ue8m0_mxfp8_scale_common(amax, rare);
                    if (__any_sync(0xffffffffu, rare)) {  // tiny or infinite maxima: warp-uniform detour
                        if (rare) sc = dev::ue8m0_mxfp8_scale(amax);
                    }
                    const float rcp = dev::ue8m0_reciprocal(sc);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const uint32_t c = (rot + i) & 7u;  // chunk held in x[i]: features 32 blk + 4 c ..
                        dev::mul2(x[i].x, x[i].y, rcp);
                        dev::mul2(x[i].z, x[i].w, rcp);
                        const uint32_t lo = dev::e4m3x2_encode(x[i].x, x[i].y);
                        const uint32_t hi = dev::e4m3x2_encode(x[i].z, x[i].w);
                        dev::sts_u32(a_tile + sw128_offset(r, 32 * blk + 4 * (int)c), (lo & 0xffffu) | (hi << 16));
                    }
                    dev::sts_u8(sfa + ((r & 31) << 4) + ((r >> 5) << 2) + blk, sc);
                }
                // the group's staging rows are consumed: the producer refills them
                __syncwarp();
                if (lane == 0) dev::mbar_arrive(&xe[grp]);
            }
            if (!ok) break;
            dev::fence_proxy_async();  // generic shared-memory writes -> visible to the tensor core
            __syncwarp();
            if (lead_lane) {  // published to the MMA thread by the a_full arrival
                sweep0[as] = ct0;
                sweep_mask[as] = tmask;
            }
            if (lane == 0) dev::mbar_arrive(&a_full[as]);
        }
    }
    } else {
        // ------------------------------------------------------------ epilogue
        if constexpr (kArgmin && kRegSplit) asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kHighRegs));
        // Warp (q, j): TMEM lane quadrant q = warp % 4 (the only lanes it may
        // read), columns [64 j, 64 j + 64) of every accumulator tile.  All three
        // warps of a quadrant drain each tile together, so a stage is held only
        // for two 32-column loads.
        const int q = warp & 3;
        const int j = (warp - kEpiWarp0) >> 2;
        const int r = q * 32 + lane;     // row within the point tile
        float4* merge = reinterpret_cast<float4*>(smem + L.merge_off);
        float2* seed = reinterpret_cast<float2*>(smem + L.seed_off);
        const uint32_t cn_saddr = dev::smem_addr(smem + L.cn_off);
        const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(j * kSliceCols);
        // After each row tile's first (hinted) centroid tile the quadrant's three
        // warps swap their running minima, so each then starts from the likely
        // winner and rarely needs an index search.  With row bounds each row's
        // minimum starts at its bound instead, which needs no exchange.
        const bool seeding = kArgmin && tiles_n >= 2 && !p.row_bound;
        // (no sweep hint and no row bounds: most chunks improve some row of the warp)
        const bool screen = p.start_hint || p.row_bound;
        // One warp hands the tile's centroid-ring slots back to the producer:
        // acc_full means every MMA that read them has completed.
        const bool releaser = p.epi_release && q == 0 && j == 0 && lane == 0;
        float cmax = 0.0f;
        for (int w = 0; w < kThreads / 32; ++w) {
            const float c = warp_cmax[w];
            cmax = c > cmax || c != c ? c : cmax;
        }
        // kSec: the largest beta of all centroids (the key bound's conversion)
        float bmax_all = -__int_as_float(0x7f800000);
        if constexpr (kSec) {
            for (int c = lane; c < (int)((p.n + 31) >> 5); c += 32) bmax_all = fmaxf(bmax_all, __ldg(p.bmax32 + c));
            for (int o = 16; o; o >>= 1) bmax_all = fmaxf(bmax_all, __shfl_xor_sync(0xffffffffu, bmax_all, o));
        }
        RingPos rel{0, 0u, kBStages};
        uint32_t seed_ph = 0;  // phase of this quadrant's seed exchanges
        int s = 0;           // accumulator stage of the next tile
        uint32_t sph = 0;
        bool ok = true;
        int it = 0;
        // Per-row-tile inputs (the row's point id and norm, the sweep start)
        // come from dependent global loads; they are software-pipelined: ids
        // two row tiles ahead, norms and hints one ahead, so no warp stalls on
        // them while its accumulator stage waits to be drained.
        const int64_t step = gridDim.x;
        auto row_id = [&](int64_t t) -> int64_t {  // point id of this lane's row of tile t (-1: none)
            const int64_t g = t * kBM + r;
            if (!kArgmin || t >= tiles_m || g >= mrows) return -1;
            return p.pid ? (int64_t)p.pid[g] : g;
        };
        auto lead_id = [&](int64_t t) -> int64_t {  // point id of tile t's first row (-1: no hint)
            if (!p.start_hint || t >= tiles_m) return -1;
            return p.pid ? (int64_t)p.pid[t * kBM] : t * kBM;
        };
        auto norm_of = [&](int64_t id) -> float { return id >= 0 ? p.pn[id] : 0.0f; };
        auto hint_of = [&](int64_t id) -> int { return id >= 0 ? p.start_hint[id] : -1; };
        auto mask_of = [&](int64_t t) -> uint64_t {  // centroid tiles of point tile t
            return p.tile_mask && t < tiles_m ? p.tile_mask[t] : ~0ull;
        };
        auto bound_of = [&](int64_t t) -> float4 {  // (bound, previous label, excluded tiles' bound) of tile t's row
            const int64_t g = t * kBM + r;
            const float inf = __int_as_float(0x7f800000);
            return kArgmin && p.row_bound && t < tiles_m && g < mrows ? p.row_bound[g]
                                                                      : make_float4(inf, __int_as_float(-1), inf, 0.0f);
        };
        int64_t id_cur = row_id(blockIdx.x), lead_cur = lead_id(blockIdx.x);
        float pn_cur = norm_of(id_cur);
        int hint_cur = hint_of(lead_cur);
        uint64_t mask_cur = mask_of(blockIdx.x);
        float4 rb_cur = bound_of(blockIdx.x);
        int64_t id_nxt = row_id(blockIdx.x + step), lead_nxt = lead_id(blockIdx.x + step);
        for (int64_t tile = blockIdx.x; tile < tiles_m && ok; tile += gridDim.x, ++it) {
            const int buf = it & 1;
            const int64_t grow = tile * kBM + r;
            const bool valid = grow < mrows;
            const int64_t point = kArgmin && valid ? id_cur : grow;
            const float pn = pn_cur;
            const int ct0 = hint_cur >= 0 && (int64_t)hint_cur < p.n ? hint_cur / kBN : 0;
            // issue the next row tiles' loads now; they are consumed an iteration later
            const float pn_nxt = norm_of(id_nxt);
            const int hint_nxt = hint_of(lead_nxt);
            const uint64_t tmask = mask_cur;
            const uint64_t mask_nxt = mask_of(tile + step);
            const float4 rb = rb_cur;
            const float4 rb_nxt = bound_of(tile + step);
            const int forced = __float_as_int(rb.y);
            const int64_t id_nn = row_id(tile + 2 * step), lead_nn = lead_id(tile + 2 * step);
            const float2 pn2 = make_float2(pn, pn);
            const float pc = pn + cmax;
            RowMin m{rb.x, -1e38f, -1e38f, kNoLabel, __int_as_float(0x7f800000)};
            for (int i = 0; i < tiles_n; ++i) {
                const int ct = ct0 + i < tiles_n ? ct0 + i : ct0 + i - tiles_n;
                if (!((tmask >> ct) & 1ull)) continue;  // pruned centroid tile (the first, ct0, never is)
                const int slice0 = ct * kBN + j * kSliceCols;
                if (!dev::mbar_wait(&acc_full[s], sph, abort_flag, p.err)) { ok = false; break; }
                dev::tc_fence_after();
                if (releaser) {
                    for (int kc = 0; kc < p.kchunks; ++kc) {
                        dev::mbar_arrive(&b_empty[rel.slot]);
                        rel.advance(1);
                    }
                }
                uint32_t v[kSubChunks][32];
#pragma unroll
                for (int sub = 0; sub < kSubChunks; ++sub)
                    dev::tmem_ld_32x32b_x32(lane_base + (uint32_t)s * kBN + 32u * sub, v[sub]);
                dev::tmem_wait_ld();
                dev::tc_fence_before();
                __syncwarp();
                if (lane == 0) dev::mbar_arrive(&acc_empty[s]);
                if (++s == kAccStages) s = 0, sph ^= 1u;
#pragma unroll
                for (int sub = 0; sub < kSubChunks; ++sub) {
                    const int cc = slice0 + sub * 32;
                    if constexpr (!kArgmin) {
                        if (valid) {
                            float* orow = p.out + grow * p.n;
                            if (cc + 32 <= p.n && p.out_vec) {
#pragma unroll
                                for (int c = 0; c < 32; c += 4)
                                    *reinterpret_cast<float4*>(orow + cc + c) = make_float4(
                                        __uint_as_float(v[sub][c]), __uint_as_float(v[sub][c + 1]),
                                        __uint_as_float(v[sub][c + 2]), __uint_as_float(v[sub][c + 3]));
                            } else {
#pragma unroll
                                for (int c = 0; c < 32; ++c)
                                    if (cc + c < p.n) orow[cc + c] = __uint_as_float(v[sub][c]);
                            }
                        }
                    } else if (p.cn_smem) {
                        fold_chunk<kGaps, kSec>(v[sub], NormSrc<true>{p.cn, cn_saddr}, pn2, pn, pc, cc, p.n, m,
                                                forced, screen);
                    } else {
                        fold_chunk<kGaps, kSec>(v[sub], NormSrc<false>{p.cn, 0u}, pn2, pn, pc, cc, p.n, m, forced,
                                                screen);
                    }
                }
                if (seeding && i == 0 && (tmask & (tmask - 1ull)) != 0) {  // (more tiles follow in this row tile)
                    // The exchange is skipped for row tiles with a single centroid tile,
                    // so its barrier phase and buffer follow their own count (the same
                    // in the quadrant's three warps, which see the same masks).
                    float2* mine = seed + (size_t)(seed_ph * kEpiPerQuad) * kBM;
                    mine[j * kBM + r] = make_float2(m.first, __int_as_float(m.best));
                    __syncwarp();
                    if (lane == 0) dev::mbar_arrive(&seed_bar[q]);
                    if (!dev::mbar_wait(&seed_bar[q], seed_ph, abort_flag, p.err)) { ok = false; break; }
                    seed_ph ^= 1u;
#pragma unroll
                    for (int o = 0; o < kEpiPerQuad; ++o) {
                        if (o == j) continue;
                        const float2 sd = mine[o * kBM + r];
                        // (the partial's bound comes with the final merge)
                        merge_rowmin<false, kSec>(m, sd.x, __float_as_int(sd.y), 0.0f, 0.0f,
                                                  __int_as_float(0x7f800000), pn);
                    }
                }
            }
            if (!ok) break;
            if constexpr (kArgmin) {
                // Combine the three column slices of each row.  The hand-off uses
                // mbarriers with bounded waits (never bar.sync).
                const int hb = q * 2 + buf;
                const uint32_t hph = (uint32_t)(it >> 1) & 1u;
                float4* slots = merge + (size_t)buf * (kEpiPerQuad - 1) * kBM;
                if (j != 0) {
                    if (!dev::mbar_wait(&merge_empty[hb], hph ^ 1u, abort_flag, p.err)) { ok = false; break; }
                    slots[(j - 1) * kBM + r] =
                        make_float4(m.first, __int_as_float(m.best), kSec ? m.sec : m.largest, m.next);
                    __syncwarp();
                    if (lane == 0) dev::mbar_arrive(&merge_full[hb]);
                } else {
                    if (!dev::mbar_wait(&merge_full[hb], hph, abort_flag, p.err)) { ok = false; break; }
                    float4 o[kEpiPerQuad - 1];
#pragma unroll
                    for (int w = 0; w < kEpiPerQuad - 1; ++w) o[w] = slots[w * kBM + r];
                    __syncwarp();
                    if (lane == 0) dev::mbar_arrive(&merge_empty[hb]);
                    if (valid) {
#pragma unroll
                        for (int w = 0; w < kEpiPerQuad - 1; ++w)
                            merge_rowmin<kGaps, kSec>(m, o[w].x, __float_as_int(o[w].y), o[w].z, o[w].w, o[w].z,
                                                      pn);
                        p.labels[point] = m.best;
                        // the row's position in the visiting order (by_row outputs)
                        const int64_t at = !p.by_row ? point : p.row_bound ? (int64_t)__float_as_int(rb.w) : grow;
                        if (p.row_labels) p.row_labels[at] = m.best;
                        if constexpr (kSec) {
                            // keys -> a bound on d - beta_c (less the largest beta), with the
                            // excluded tiles' bound from the row record
                            const float sec = fminf(rb.z, fmaf(-0x1p-18f, pc + fabsf(m.sec), pn + m.sec) - bmax_all);
                            *reinterpret_cast<float2*>(p.best_dist + at * p.best_dist_stride) =
                                make_float2(m.first, sec);
                        }
                        else if (p.best_dist)
                            p.best_dist[at * p.best_dist_stride] = m.first;
                        if constexpr (kGaps) p.gaps[point] = m.largest - m.next;
                    }
                    if (p.changes) {  // label changes, one counter update per warp
                        const bool moved = valid && forced >= 0 && m.best != forced;
                        const unsigned bal = __ballot_sync(0xffffffffu, moved);
                        if (bal) {
                            const int leader = __ffs(bal) - 1;
                            int base = 0;
                            if (lane == leader) base = atomicAdd(p.change_count, __popc(bal));
                            base = __shfl_sync(0xffffffffu, base, leader);
                            if (moved)
                                p.changes[base + __popc(bal & ((1u << lane) - 1u))] =
                                    make_int4((int)point, forced, m.best, 0);
                        }
                    }
                }
            }
            id_cur = id_nxt, lead_cur = lead_nxt, pn_cur = pn_nxt, hint_cur = hint_nxt, mask_cur = mask_nxt;
            rb_cur = rb_nxt;
            id_nxt = id_nn, lead_nxt = lead_nn;
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
                   cudaStream_t stream, bool scale_atoms, const float* points_f32, int64_t points_rows) {
    if (bits != 4 && bits != 6 && bits != 8) return fail(MXK_ERR_INVALID, "Precision must be 4, 6, or 8");
    if (m <= 0 || n <= 0) return MXK_OK;
    MXK_REQUIRE(k > 0 && k % kChunk == 0, "gemm_mx: k must be a positive multiple of 128");
    if (k / kChunk > kMaxChunks) return fail(MXK_ERR_UNSUPPORTED, "gemm_mx: k > 1024 is not supported");
    const bool fuse_x = points_f32 != nullptr;
    if (fuse_x) {
        MXK_REQUIRE(bits == 8 && k == kChunk && argmin, "fused quantize: MXFP8, d = 128 and the argmin epilogue only");
        MXK_REQUIRE(aligned(points_f32, 16) && points_rows > 0 && points_rows < (1ll << 31),
                    "fused quantize: points must be 16-byte aligned with 1..2^31-1 rows");
        MXK_REQUIRE(argmin->pid || m <= points_rows, "fused quantize: more rows than points");
    } else {
        MXK_REQUIRE(a && a_scales, "gemm_mx: null operand");
        MXK_REQUIRE(aligned(a, 16), "gemm_mx: operands must be 16-byte aligned");
        MXK_REQUIRE(aligned(a_scales, scale_atoms ? 16 : 4), "gemm_mx: scales must be 4-byte aligned (16 for the atom layout)");
    }
    MXK_REQUIRE(b && b_scales, "gemm_mx: null operand");
    MXK_REQUIRE(aligned(b, 16), "gemm_mx: operands must be 16-byte aligned");
    MXK_REQUIRE(aligned(b_scales, scale_atoms ? 16 : 4), "gemm_mx: scales must be 4-byte aligned (16 for the atom layout)");
    MXK_REQUIRE(n < (1ll << 31) && m < (1ll << 31), "gemm_mx: m and n must be below 2^31 (TMA coordinates)");
    if (argmin) {
        MXK_REQUIRE(argmin->point_norms && argmin->centroid_norms && argmin->labels, "assign: null pointer");
        MXK_REQUIRE(aligned(argmin->centroid_norms, 16), "assign: centroid norms must be 16-byte aligned");
    } else {
        MXK_REQUIRE(out != nullptr, "gemm_mx: null output");
    }

    CUtensorMap tmap_a, tmap_b, tmap_x;
    std::memset(&tmap_a, 0, sizeof(tmap_a));
    std::memset(&tmap_x, 0, sizeof(tmap_x));
    if (bits == 8 && !fuse_x)
        MXK_CHECK(encode_tensor_map_2d(&tmap_a, a, (uint64_t)k, (uint64_t)m, (uint64_t)k, kChunk, kBM,
                                       CU_TENSOR_MAP_DATA_TYPE_UINT8, CU_TENSOR_MAP_SWIZZLE_128B));
    if (fuse_x)  // one-row box for tile::gather4; rows past points_rows read as zeros
        MXK_CHECK(encode_tensor_map_2d(&tmap_x, points_f32, (uint64_t)k, (uint64_t)points_rows, (uint64_t)k * 4,
                                       (uint32_t)k, 1, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, CU_TENSOR_MAP_SWIZZLE_NONE));
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
    p.fuse_x = fuse_x;
    p.xrows = points_rows;
    if (argmin) {
        p.pn = argmin->point_norms;
        p.cn = argmin->centroid_norms;
        p.pid = argmin->pid;
        p.labels = argmin->labels;
        p.gaps = argmin->gaps;
        p.start_hint = argmin->start_hint;
        p.tile_mask = argmin->tile_mask;
        p.best_dist = argmin->best_dist;
        p.best_dist_stride = argmin->best_dist_stride;
        p.row_bound = argmin->row_bound;
        p.by_row = argmin->by_row;
        p.row_labels = argmin->row_labels;
        MXK_REQUIRE(!p.row_labels || p.by_row, "gemm_mx: row labels are indexed by row");
        p.bmax32 = argmin->beta_max32;
        MXK_REQUIRE(!argmin->second_bound ||
                        (p.best_dist && p.bmax32 && !p.gaps && p.best_dist_stride >= 2 &&
                         p.best_dist_stride % 2 == 0 && aligned(p.best_dist, 8)),
                    "gemm_mx: the second-nearest bound needs best_dist (even stride, 8-byte aligned), beta_max32 "
                    "and no gaps");
        p.changes = argmin->changes;
        p.change_count = argmin->change_count;
        MXK_REQUIRE(!p.changes || (p.row_bound && p.change_count), "gemm_mx: label changes need row bounds and a count");
        MXK_REQUIRE(!(p.row_bound && p.gaps), "gemm_mx: row bounds and gaps are exclusive");
        MXK_REQUIRE(!p.tile_mask || (n + kBN - 1) / kBN <= 64, "gemm_mx: a tile mask covers at most 64 centroid tiles");
    }
    p.err = device_error_word();
    p.tiles_done = device_tile_counter();
    p.rows_done = device_row_counter();
    if (!p.err) return fail(MXK_ERR_CUDA, "gemm_mx: cannot allocate the device error word");

    int max_smem = 0, dev = 0;
    MXK_CUDA(cudaGetDevice(&dev));
    MXK_CUDA(cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    // Shared-memory plan: two point-tile stages when they fit, the centroid norms
    // when they fit, then as deep a centroid-chunk ring as the rest allows
    // (deeper rings keep more TMA bytes in flight per SM).
    const int64_t tiles_n = (n + kBN - 1) / kBN;
    p.sfb_resident = tiles_n * p.kchunks <= kMaxResidentSfb;
    auto sfb_atoms = [&](int bs) { return p.sfb_resident ? (int)(tiles_n * p.kchunks * kBAtoms) : bs * kBAtoms; };
    auto fits = [&](int as, int cn, int bs) {
        return (int)smem_layout(p.kchunks, as, cn, bs, sfb_atoms(bs), p.fuse_x).total + 1024 <= max_smem;
    };
    p.cn_smem = (argmin && n <= kMaxSmemNorms) ? (int)n : 0;
    // (with the fused quantizer's 64 KB staging, two point stages leave room for
    // three ring slots; a single point stage would serialize encoding and MMA)
    // Point-tile stages: up to four when they fit beside four ring slots (the
    // gathered-A path, whose tiles are short when centroid tiles are pruned),
    // else two beside three (with the fused quantizer's 64 KB FP32 staging a
    // single stage would serialize encoding and MMA), else one.
    p.a_stages = 1;
    for (int as = kMaxAStages; as >= 2; --as)
        if (!p.fuse_x && fits(as, p.cn_smem, 4)) { p.a_stages = as; break; }
    if (p.a_stages == 1 && fits(2, p.cn_smem, 3)) p.a_stages = 2;
    if (!fits(p.a_stages, p.cn_smem, 3)) p.cn_smem = 0;
    if (!fits(p.a_stages, p.cn_smem, 2)) return fail(MXK_ERR_UNSUPPORTED, "gemm_mx: shared memory budget exceeded");
    p.b_stages = 2;
    while (p.b_stages < kMaxBStages && fits(p.a_stages, p.cn_smem, p.b_stages + 1)) ++p.b_stages;
    // A slot freed only when its whole tile completes needs room for the next
    // tile's chunks too; otherwise each chunk is freed by its own commit.
    p.epi_release = p.b_stages >= 2 * p.kchunks;
    p.sfb_atoms = sfb_atoms(p.b_stages);
    // At least 116 KB so that no second CTA shares the SM (each CTA holds all
    // 512 TMEM columns while it runs).
    const uint32_t smem_bytes =
        std::max<uint32_t>(smem_layout(p.kchunks, p.a_stages, p.cn_smem, p.b_stages, p.sfb_atoms, p.fuse_x).total + 1024,
                           116u * 1024u);
    if ((int)smem_bytes > max_smem) return fail(MXK_ERR_UNSUPPORTED, "gemm_mx: shared memory budget exceeded");

    const int64_t tiles_m = (m + kBM - 1) / kBM;
    const int grid = (int)std::min<int64_t>(tiles_m, sm_count());

    // Row-major scales (the API layout) are converted once per call into the
    // atom layout the kernel bulk-copies; the temporaries are stream-ordered.
    uint8_t* tmp_atoms = nullptr;
    if (!scale_atoms) {
        // (the fused quantizer writes the point scales itself; only B needs them)
        MXK_REQUIRE(!rows_dev || fuse_x, "gemm_mx: device-side row counts need atom-layout scales");
        const int64_t a_bytes = fuse_x ? 0 : scale_atom_bytes(m, k, kBM);
        const int64_t b_bytes = scale_atom_bytes(n, k, kBN);
        MXK_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&tmp_atoms), (size_t)(a_bytes + b_bytes), stream));
        const int sms = sm_count();
        {
            LaunchScope scope("scales_to_atoms", stream);
            if (a_bytes)
                scales_to_atoms_kernel<<<sms * 4, 256, 0, stream>>>(m, p.kchunks, kBM, a_scales, tmp_atoms,
                                                                    a_bytes / 4);
            scales_to_atoms_kernel<<<sms * 4, 256, 0, stream>>>(n, p.kchunks, kBN, b_scales, tmp_atoms + a_bytes,
                                                                b_bytes / 4);
        }
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) {
            cudaFreeAsync(tmp_atoms, stream);
            return fail_cuda("scales_to_atoms_kernel", e);
        }
        if (a_bytes) p.a_scales = tmp_atoms;
        p.b_scales = tmp_atoms + a_bytes;
    }

    auto launch = [&](auto kernel, const char* name) -> int {
        MXK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bytes));
        if (argmin) {
            // the setmaxnreg split assumes exactly kLaunchRegs registers at launch
            cudaFuncAttributes attr{};
            MXK_CUDA(cudaFuncGetAttributes(&attr, kernel));
            if (attr.numRegs != kLaunchRegs)
                return fail(MXK_ERR_UNSUPPORTED, "gemm_mx: argmin kernel built with " + std::to_string(attr.numRegs) +
                                                     " registers, the register split needs " +
                                                     std::to_string(kLaunchRegs));
        }
        LaunchScope scope(name, stream);
        kernel<<<grid, kThreads, smem_bytes, stream>>>(tmap_a, tmap_b, tmap_x, p);
        MXK_CUDA(cudaGetLastError());
        return MXK_OK;
    };
    int st;
    if (!argmin)
        st = launch(mx_gemm_kernel<false, false>, "mx_gemm_dense");
    else if (argmin->gaps)
        st = launch(mx_gemm_kernel<true, true>, "mx_gemm_argmin_gap");
    else if (argmin->second_bound)
        st = launch(mx_gemm_kernel<true, false, true>, "mx_gemm_argmin");
    else
        st = launch(mx_gemm_kernel<true, false>, "mx_gemm_argmin");
    if (tmp_atoms) cudaFreeAsync(tmp_atoms, stream);
    return st;
}

}  // namespace mxk

extern "C" {

int mxk_gemm_mx(int bits, int64_t m, int64_t n, int k, const void* a, const uint8_t* a_scales, const uint8_t* b,
                const uint8_t* b_scales, float* out, void* stream) {
    MXK_CHECK(mxk::launch_gemm_mx(bits, m, n, k, a, a_scales, b, b_scales, out, nullptr, nullptr,
                                  mxk::as_stream(stream)));
    return mxk::check_device_error(mxk::as_stream(stream));
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
    MXK_CHECK(mxk::launch_gemm_mx(bits, rows, k, d, a, a_scales, b, b_scales, nullptr, &am, nullptr,
                                  mxk::as_stream(stream)));
    return mxk::check_device_error(mxk::as_stream(stream));
}

int mxk_assign_f32_fused(int64_t rows, int k, int d, const float* points, int64_t n_points, const uint8_t* b,
                         const uint8_t* b_scales, const float* point_norms, const float* centroid_norms,
                         const int* pid, int* labels, float* gaps, const int* start_hint, void* stream) {
    mxk::MxArgmin am;
    am.point_norms = point_norms;
    am.centroid_norms = centroid_norms;
    am.pid = pid;
    am.labels = labels;
    am.gaps = gaps;
    am.start_hint = start_hint;
    MXK_REQUIRE(points != nullptr, "assign_f32_fused: null points");
    MXK_CHECK(mxk::launch_gemm_mx(8, rows, k, d, nullptr, nullptr, b, b_scales, nullptr, &am, nullptr,
                                  mxk::as_stream(stream), false, points, n_points));
    return mxk::check_device_error(mxk::as_stream(stream));
}

}  // extern "C"
