// Internal launchers shared by the C-ABI entry points and the Lloyd driver.
// All return an mxk_status; pointers are device pointers; launches go to
// `stream` and do not synchronize.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mxk {

// ---- quantize.cu ------------------------------------------------------------
// rows_dev (optional): device-resident row count that overrides `rows`, which
// then only sizes the grid (an upper bound).  atom_rows > 0: write the scales in
// the tcgen05 atom layout for tiles of atom_rows rows (scale_atom_bytes(rows, d,
// atom_rows) bytes, d % 128 == 0) instead of row-major [rows][d/32].
//
// Atom layout: rows form tiles of tile_rows (a point tile is kPointTileRows, a
// centroid tile kCentroidTileRows); each (tile, 128-feature chunk) owns
// ceil(tile_rows / 128) consecutive 512-byte atoms, one per 128-row slice of the
// tile, holding slice row r's four block scales at (r % 32) * 16 + (r / 32) * 4 +
// block % 4 -- the image tcgen05.cp .32x128b.warpx4 copies into TMEM.
constexpr int kPointTileRows = 128;
constexpr int kCentroidTileRows = 192;
// name: the launch's name in the library's kernel timing (mxk_profile_read).
int launch_quantize(int bits, int64_t rows, int d, const float* points, const int* pid, void* values,
                    uint8_t* scales, float* max_errors, const int* rows_dev, cudaStream_t stream,
                    int atom_rows = 0, const char* name = "quantize_mx");
inline int64_t scale_atom_bytes(int64_t rows, int d, int tile_rows = kPointTileRows) {
    return (rows + tile_rows - 1) / tile_rows * (d / 128) * ((tile_rows + 127) / 128) * 512;
}
int launch_l2_norm(int64_t rows, int d, const float* x, float* norms, cudaStream_t stream);
// Rows of an MXFP8 matrix (d bytes per row, d / 32 row-major scale bytes)
// gathered in the order pid (null: identity) into contiguous rows, scales in the
// kPointTileRows atom layout.  stop: the Lloyd loop's stop word (optional).
int launch_gather_mxfp8_rows(int64_t rows, int d, const uint8_t* src, const uint8_t* src_scales, const int* pid,
                             uint8_t* dst, uint8_t* dst_scales, const int* stop, cudaStream_t stream);
int launch_point_bounds(int64_t n, int d, const float* points, const float* norms, float* upper,
                        cudaStream_t stream);
// lc/ec either as host values (lc_dev == nullptr) or read from device memory.
// policy 0: select_precision (the reference's rule, always 8); 1: the candidate
// precision_candidate returns (mxk_set_precision_policy).
int launch_assign_precisions(int64_t n, int d, const float* upper, const float* gaps, float lc, float ec,
                             const float* lc_ec_dev, int* precision, int* group_counts, cudaStream_t stream,
                             int policy = 0);
// stats[0] = sqrt(max errors), stats[1] = sqrt(max norms)  (src/kmeans.cu:38-41)
int launch_centroid_stats(int k, const float* errors, const float* norms, float* stats, cudaStream_t stream);
// Stable per-precision compaction of point ids (src/kmeans.cu:45-52).
// ids: 3*n ints (groups 4, 6, 8 at offsets 0, n, 2n); group_counts: 3 ints.
// scratch: compaction_scratch_ints(n) ints.  order (optional, n ints): the
// sequence to compact (element i is point order[i]); null = 0..n-1.
int64_t compaction_scratch_ints(int64_t n);
// stop (optional, device word): when it is non-zero at run time the launches
// do nothing except report empty groups (the Lloyd loop's converged state).
int launch_group_compaction(int64_t n, const int* precision, const int* order, int* ids, int* group_counts,
                            int* scratch, cudaStream_t stream, const int* stop = nullptr);

// ---- order.cu -----------------------------------------------------------------
// order = point indices 0..n-1 sorted by labels[] (counting sort over k keys;
// order within a key is unspecified).  scratch: label_sort_scratch_ints(k) ints.
int64_t label_sort_scratch_ints(int k);
// Per-row state kept in the visiting order (the pruning pass's records and
// the rows' labels), moved along when the order is rebuilt: state[g] is the
// record (not moved while null) and label[g] the current label of the point at
// position g; tmp_* are n-entry scratch.  With it the sort reorders the
// current visiting order (the order buffer must hold a permutation, e.g.
// launch_identity_order's) by label[] instead of the points 0..n-1 by
// labels[]; k <= 16384.
struct RowState {
    float4* state = nullptr;
    int* label = nullptr;
    float4* tmp_state = nullptr;
    int* tmp_label = nullptr;
    int* tmp_order = nullptr;
};
// order = 0, 1, ..., n - 1 (the identity order).
int launch_identity_order(int64_t n, int* order, cudaStream_t stream);
// stop (optional, device word): non-zero at run time = do nothing.
// row_state (optional): moved into the new order.
int launch_label_sort(int64_t n, int k, const int* labels, int* order, int* scratch, cudaStream_t stream,
                      const int* stop = nullptr, const RowState* row_state = nullptr);
// Rebuild gate for the label sort: ctl = (label changes since the last
// rebuild, skip word), zero at the start of a run.  Adds *changes (this
// iteration's label changes) and sets the skip word -- the stop word to pass to
// launch_label_sort -- unless at least `threshold` labels have changed since
// the last rebuild (then clears it and restarts the count); also set while
// *stop is.
int launch_sort_gate(const int* stop, const int* changes, int* ctl, int threshold, cudaStream_t stream);

// ---- gemm_mx.cu ---------------------------------------------------------------
struct MxArgmin {
    const float* point_norms = nullptr;     // indexed by pid[row] (or row)
    const float* centroid_norms = nullptr;  // k
    const int* pid = nullptr;
    int* labels = nullptr;
    float* gaps = nullptr;  // optional two-largest gap (init -1e38)
    // optional label per point (may be `labels` itself, read before it is
    // overwritten): each 128-row tile sweeps the centroids starting at the tile
    // of its first row's hint; results do not depend on it
    const int* start_hint = nullptr;
    // optional: per 128-row point tile, a mask of the 192-centroid tiles that may
    // hold a row's nearest centroid (bit t = centroid tile t; the tile of the
    // first row's start_hint must be set); the others are skipped.  n <= 64 tiles.
    const uint64_t* tile_mask = nullptr;
    // optional: each point's distance to its nearest centroid, at
    // best_dist[point * best_dist_stride]
    float* best_dist = nullptr;
    int best_dist_stride = 1;
    // with best_dist (stride >= 2, 8-byte aligned rows) and beta_max32: also a
    // lower bound on d(x, c) - beta_c for every centroid c other than the
    // point's nearest, at best_dist[point * best_dist_stride + 1] (from the
    // screened chunk minima and the exact chunks, each less the largest beta of
    // its 32 centroids, and, with row_bound, the bound of the tiles the row's
    // own mask excludes); beta_c = |c|^2 - |c^|^2 of the MXFP8 round trip c^
    bool second_bound = false;
    const float* beta_max32 = nullptr;  // [ceil(n / 32)] the largest beta of each 32 consecutive centroids
    // optional, per GEMM row (the order of pid): (an upper bound on the row's
    // distance to its nearest centroid or inf, the row's previous label as int
    // bits or -1, a lower bound on d(x, c) - beta_c for every centroid c of the
    // tiles its own mask excludes or +inf, the row's position in the visiting
    // order as int bits).  The epilogue starts each row's minimum at the bound
    // and always evaluates the chunk holding the previous label exactly; the
    // result is unchanged.
    const float4* row_bound = nullptr;
    // best_dist (and its second bound) and row_labels (optional: the label
    // again) are indexed by the row's position in the visiting order -- the GEMM
    // row, or row_bound's fourth field -- instead of by point
    bool by_row = false;
    int* row_labels = nullptr;
    // optional (with row_bound): every row whose label differs from its
    // previous one (row_bound's) is recorded as (point, previous, new, 0) at
    // changes[atomicAdd(change_count, 1)]
    int4* changes = nullptr;
    int* change_count = nullptr;
};
// Dense: out[m x n] = A . B^T.  Argmin: labels of the m rows against n centroids.
// rows_dev (optional) = device-resident m (m is then an upper bound).
// scale_atoms: the point scales are in the atom layout for kPointTileRows and the
// centroid scales for kCentroidTileRows (see launch_quantize), which the kernel
// fetches with bulk copies; otherwise both are row-major and converted per call.
// points_f32 (argmin, bits 8, k 128 only): quantize the point tile in the kernel
// from these FP32 rows (points_rows of them, gathered through argmin->pid), with
// the bytes quantize_rows would write; a / a_scales are then unused.
int launch_gemm_mx(int bits, int64_t m, int64_t n, int k, const void* a, const uint8_t* a_scales,
                   const uint8_t* b, const uint8_t* b_scales, float* out, const MxArgmin* argmin,
                   const int* rows_dev, cudaStream_t stream, bool scale_atoms = false,
                   const float* points_f32 = nullptr, int64_t points_rows = 0);

// ---- prune.cu ----------------------------------------------------------------
// Exact pruning of centroid tiles (see prune.cu for the bounds).  Supported for
// at most 64 centroid tiles and d % 128 == 0, d <= 1024.
bool prune_supported(int64_t k, int d);
// Centroid preparation of an MX iteration with pruning, one pass per centroid
// row: cn (|c|^2, compute_l2_norm's values), the MXFP8 codes qcent (k x d) and
// scales cscales (atom layout for kCentroidTileRows-row tiles, as
// launch_quantize writes them), chat (k x d dequantized centroids), cst (k x
// (|c|^2 - |c^|^2, |c^|^2, |c|^2, 0)) and delta (k upper bounds of |c^ -
// c^_prev|, +inf without prev).  stop: the Lloyd loop's stop word (optional).
int launch_centroid_prep(int k, int d, const float* centroids, const float* prev, float* cn, float* chat,
                         float4* cst, float* delta, uint8_t* qcent, uint8_t* cscales, const int* stop,
                         cudaStream_t stream);
// dmin (k x tiles lower bounds of quantized centroid-to-tile distances, from
// an FP32 Gram product reduced in registers), the tile stats tst (2 x tiles:
// per tile t, tst[t] = (min beta, max |c^|^2, max |c|^2, non-finite flag) and
// tst[tiles + t] = (max beta, max delta, 0, 0)) and bmax32 (ceil(k / 32): the
// largest beta of each 32 consecutive centroids) from chat, cst and delta.
int launch_centroid_pairs(int k, int d, const float* chat, const float4* cst, const float* delta, float* dmin,
                          float4* tst, float* bmax32, const int* stop, cudaStream_t stream);
// Between full computations: dmin lowered in place by the centroids' movement
// bounds (delta, from launch_centroid_prep), and tst and bmax32 as above.
int launch_centroid_pairs_drift(int k, int d, const float* delta, const float4* cst, float* dmin, float4* tst,
                                float* bmax32, const int* stop, cudaStream_t stream);
// Row compaction of the pruned fused iteration (launch_tile_mask's `work`):
// device buffers for the rows that stay in the GEMM, in visiting order.
struct WorkRows {
    int* pid = nullptr;            // [rows] their point ids
    float4* rb = nullptr;          // [rows] their MxArgmin::row_bound records
    unsigned long long* cmask = nullptr;  // [row tiles] centroid-tile masks of the compacted 128-row tiles
    uint4* need_bits = nullptr;    // [row tiles] scratch: which rows of each tile stay
    int* counts = nullptr;         // [row tiles] scratch
    int* offsets = nullptr;        // [row tiles] scratch
    int* seg_total = nullptr;      // [row tiles / 1024 + 1] scratch
    int* rows = nullptr;           // [1] how many rows stay (0 once the loop has stopped)
};
// Per 128-row point tile (rows in pid order), the mask of centroid tiles that
// may hold a row's nearest centroid, from the rows' previous labels and pinfo
// records (both per row, in pid order: RowState's label and state) and the
// current (cst) and previous (cst_old) centroid stats; row_bound
// (optional, one per row) receives MxArgmin::row_bound's records.  tst_old
// (optional): the tile stats of the previous iteration's centroids, when that
// iteration's GEMM wrote its points' second-nearest bounds into pinfo (the
// row test then also uses them).  With work: a row whose bounds prove that
// every other centroid is strictly farther than its previous label's keeps
// that label and leaves the GEMM (its pinfo distance becomes its upper bound,
// its second-nearest bound the lower one); the other rows are compacted into
// work (ids, records, masks of the compacted tiles, count), for a GEMM launched
// on work->pid with rows_dev = work->rows.
// fresh: pinfo's distances already bound the distance to the rows' current
// centroids (launch_row_distance_bound), so no centroid move is added.
int launch_tile_mask(int64_t rows, int k, int d, const int* pid, const int* prev_label, float4* pinfo,
                     const float4* cst, const float4* cst_old, const float4* tst, const float4* tst_old,
                     const float* delta, const float* dmin, uint64_t* mask, float4* row_bound, const int* stop,
                     cudaStream_t stream, WorkRows* work = nullptr, bool fresh = false);
// Per row (in pid order, labels and pinfo per row as launch_tile_mask reads
// them): the whole pinfo record -- an upper bound on the row's distance to its
// label's current centroid, 0, alpha_x, |x^| -- from the point's row (MXFP8
// round trip) and chat[label]: one pass over the points, for the first pruned
// iteration, whose centroids moved far.
int launch_row_distance_bound(int64_t rows, int k, int d, const int* pid, const int* label, float4* pinfo,
                              const float* chat, const float4* cst, const float* points, const int* stop,
                              cudaStream_t stream);

// ---- fp32.cu -----------------------------------------------------------------
int launch_gemm_fp32(int64_t m, int64_t n, int k, const float* a, const float* b, float* out,
                     cudaStream_t stream);

// ---- assign.cu ---------------------------------------------------------------
int launch_assign_clusters(int64_t rows, int k, const float* point_norms, const float* centroid_norms,
                           const float* dots, const int* pid, int* labels, float* gaps, cudaStream_t stream);

// ---- update.cu ---------------------------------------------------------------
// sums (k x d) and counts (k) must be zeroed by the caller.  order (optional):
// visit the points in this sequence (label-sorted orders make long label runs).
// stop (optional, device word): non-zero at run time = do nothing.  The sums
// are FP32 (the reference-facing update, as the reference's) or FP64 (the Lloyd
// driver, whose running sums also take label-change deltas).
int launch_accumulate(int64_t n, int d, int k, const float* points, const int* labels, const int* order,
                      float* sums, int* counts, cudaStream_t stream, const int* stop = nullptr);
// switched: a launch launch_update_gate may turn into a no-op; its profile
// records carry a "_switched" suffix.
int launch_accumulate(int64_t n, int d, int k, const float* points, const int* labels, const int* order,
                      double* sums, int* counts, cudaStream_t stream, const int* stop = nullptr,
                      bool switched = false);
// centroids = counts ? sums / counts : old.  If shift_scratch is not null
// (shift_scratch_floats() floats, zeroed once before the first use by a Lloyd
// loop), shift_scratch[shift_total_index()] receives sum((old - new)^2),
// reduced in a fixed order (bit-reproducible).  sums and centroids may alias.
int64_t shift_scratch_floats();
int64_t shift_total_index();
//
// loop (optional, device words, Lloyd driver): loop[0] = stopped, loop[1] =
// completed iterations, loop[2] = stopped on a non-finite shift, loop[3] = the
// row count later launches read (set to 0 when the loop stops).  While
// loop[0] is zero the launch updates the centroids, counts the iteration and
// sets loop[0] when the shift is <= tolerance or not finite (the reference's
// stopping rule, kmeans.cu:62-67); once it is set the launch does nothing, so a
// driver may enqueue iterations before it has read whether the previous one
// converged.  Requires shift_scratch.  With loop, the driver's options:
// old_centroids may be centroids itself (updated in place); prev_out receives
// the old centroids; zero_sums leaves sums and counts zero for the next
// accumulation; host_state (host-mapped pinned memory) receives the four state
// words once the launch is done, also after the loop has stopped.  acc_sums
// (k x d FP64) and acc_counts (k): running sums and counts kept across
// iterations, to which this iteration's sums / counts are added (full: which
// they replace); the centroids come from the running values.  zero_word
// (optional) is zeroed once the launch has read everything.
// full_dev (optional): a device word read at run time in place of `full`.
int launch_finalize(int d, int k, float* sums, int* counts, const float* old_centroids, float* centroids,
                    float* shift_scratch, cudaStream_t stream, int* loop = nullptr, float tolerance = 0.0f,
                    float* prev_out = nullptr, bool zero_sums = false, int* host_state = nullptr,
                    double* acc_sums = nullptr, int* acc_counts = nullptr, bool full = true,
                    int* zero_word = nullptr, const int* full_dev = nullptr);
int launch_finalize(int d, int k, double* sums, int* counts, const float* old_centroids, float* centroids,
                    float* shift_scratch, cudaStream_t stream, int* loop = nullptr, float tolerance = 0.0f,
                    float* prev_out = nullptr, bool zero_sums = false, int* host_state = nullptr,
                    double* acc_sums = nullptr, int* acc_counts = nullptr, bool full = true,
                    int* zero_word = nullptr, const int* full_dev = nullptr);
// Chooses between the incremental update and a fresh accumulation on the
// device from this iteration's change count: words = (stop word for
// launch_accumulate_changes, stop word for launch_accumulate, `full` word for
// launch_finalize); fresh once *changes > threshold.  stop: the loop's stop
// word (both skipped once it is set).
int launch_update_gate(const int* stop, const int* changes, int threshold, int* words, cudaStream_t stream);
// The label changes recorded by the GEMM (rec[i] = (point, old label, new
// label, 0), *count of them): each moves its point's row and count from the old
// cluster's to the new one's in sums / counts (this iteration's additions).
int launch_accumulate_changes(int d, int k, const float* points, const int4* rec, const int* count, double* sums,
                              int* counts, cudaStream_t stream, const int* stop = nullptr);
// sum((previous - current)^2) into shift_scratch[shift_scratch_floats() - 1].
int launch_shift(int64_t elements, const float* previous, const float* current, float* shift_scratch,
                 cudaStream_t stream);

}  // namespace mxk
