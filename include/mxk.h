/*
 * mxk.h -- C ABI of the B200 (sm_100a) MX-KMeans library, libmxkmeans.so.
 *
 * Every entry point returns an mxk_status; on failure mxk_last_error() returns a
 * thread-local message.  Pointers named points/centroids/labels/... are DEVICE
 * pointers owned by the caller unless the name says host_.  `stream` is a
 * cudaStream_t passed as void* (NULL = the legacy default stream).  Sizes are
 * 64-bit where the reference used int, so N*D and N*K may exceed 2^31.
 *
 * Each entry point names the reference interface it replaces
 * (ParCIS/MX-KMeans, include/kmeans.cuh and src/ ... file:line).  The C++
 * drop-in header include/kmeans.cuh wraps these with the reference's exact
 * signatures and exception behaviour.
 */
#ifndef MXK_H
#define MXK_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    MXK_OK = 0,
    MXK_ERR_INVALID = 1,     /* bad argument (reference: std::invalid_argument) */
    MXK_ERR_CUDA = 2,        /* CUDA runtime/driver error (reference: CUDA_CHECK) */
    MXK_ERR_UNSUPPORTED = 3, /* shape or device outside what the kernels support */
    MXK_ERR_NONFINITE = 4,   /* non-finite centroid shift (src/kmeans.cu:64) */
    MXK_ERR_TIMEOUT = 5,     /* a bounded device wait gave up */
    MXK_ERR_COMM = 6         /* NCCL error or unavailable */
} mxk_status;

/* Options of a Lloyd run.  Same fields and defaults as the reference's
 * KMeansOptions (include/kmeans.cuh:11-16): 300, 0, 1e-4, 0. */
typedef struct {
    int max_iterations;
    int fp32_iterations;
    float tolerance;
    int verbose;
} mxk_options;

const char* mxk_last_error(void);
int mxk_version(void);
/* Number of kernels this library launched since load (all devices). */
uint64_t mxk_launch_count(void);
/* No reference counterpart (the reference allocates and frees its workspace in
 * every kmeans_mixed call, src/kmeans.cu:17-27).  kmeans_mixed takes its
 * workspace from a per-device pool that keeps the memory mapped between calls;
 * this returns the current device's pooled memory to the driver (synchronizes
 * the device). */
int mxk_release_workspace(void);
/* Measurement aid, no reference counterpart: the number of 128 x 192 tiles the
 * current device's MX GEMM launches have multiplied since the last reset
 * (synchronizes the device); pruned tiles are not counted. */
int mxk_gemm_tiles_multiplied(unsigned long long* count, int reset);
/* Measurement aid, no reference counterpart: the number of point rows the
 * current device's MX GEMM launches have processed since the last reset
 * (synchronizes the device); rows whose labels the Lloyd loop's bounds proved
 * beforehand are not counted. */
int mxk_gemm_rows_processed(unsigned long long* count, int reset);

/* ---- ops (include/kmeans.cuh:23-47) ------------------------------------ */

/* compute_l2_norm, include/kmeans.cuh:23 / src/kernels/assignment.cu:7-16,60-63 */
int mxk_compute_l2_norm(int64_t rows, int d, const float* points, float* norms, void* stream);

/* quantize_rows, include/kmeans.cuh:42-43 / src/kernels/quantize.cu:13-72,111-123.
 * bits in {4,6,8}; d % 32 == 0.  values: packed rows (rows*d*bits/8 bytes);
 * scales: rows*(d/32) UE8M0 bytes, row-major; max_errors (optional, caller
 * zeroed) receives the max squared reconstruction error per row.  pid (optional)
 * maps output row r to source row pid[r]. */
int mxk_quantize_rows(int bits, int64_t rows, int d, const float* points, const int* pid,
                      void* values, uint8_t* scales, float* max_errors, void* stream);

/* precompute_point_bounds, include/kmeans.cuh:35-36 / src/kernels/quantize.cu:74-98,125-128.
 * upper: ceil(n/32)*96 floats. */
int mxk_precompute_point_bounds(int64_t n, int d, const float* points, const float* norms,
                                float* upper, void* stream);

/* assign_precisions, include/kmeans.cuh:37-38 / src/kernels/quantize.cu:100-108,130-134 */
int mxk_assign_precisions(int64_t n, int d, const float* upper, const float* gaps, float lc,
                          float ec, int* precision, void* stream);

/* Self-check, no reference counterpart: runs every float32 bit pattern through
 * the division-free MXFP8 scale rule of mxk_assign_f32_fused's in-kernel
 * quantizer and through ue8m0(amax / 448), the rule of quantize_rows
 * (src/kernels/quantize.cu:33-43).  result: 2 device words, [0] = number of
 * disagreements, [1] = smallest disagreeing pattern (all ones when none). */
int mxk_check_mxfp8_scale_codec(unsigned long long* result, void* stream);

/* Self-check, no reference counterpart: failure detection of the kernels'
 * bounded waits.  One CTA waits on an mbarrier that nothing arrives on: warp 0
 * through the bounded wait every pipelined kernel of this library uses, with
 * limit_cycles (> 0, at most the kernels' own limit of 2^33 cycles), warp 1
 * with the kernels' own limit, leaving when warp 0's timeout raises the CTA's
 * abort flag.  outcome: 2 device ints, 1 = that warp's wait completed, 0 = it
 * gave up.  Returns what a public call reports after such a wait,
 * MXK_ERR_TIMEOUT, with the device error word cleared for the next call. */
int mxk_check_wait_timeout(long long limit_cycles, int* outcome, void* stream);

/* gemm_mx, include/kmeans.cuh:46-47 / src/kernels/gemm.cu:348-363.
 * out[m x n] (row-major FP32) = A[m x k] (packed MX{bits}) . B[n x k]^T (MXFP8),
 * scales row-major per 32 features.  tcgen05 block-scaled MMA; k % 128 == 0. */
int mxk_gemm_mx(int bits, int64_t m, int64_t n, int k, const void* a, const uint8_t* a_scales,
                const uint8_t* b, const uint8_t* b_scales, float* out, void* stream);

/* gemm_fp32, include/kmeans.cuh:45 / src/kernels/gemm.cu:365-380.
 * out[m x n] = A[m x k] . B[n x k]^T in FP32 (no TF32). */
int mxk_gemm_fp32(int64_t m, int64_t n, int k, const float* a, const float* b, float* out,
                  void* stream);

/* assign_clusters, include/kmeans.cuh:31-33 / src/kernels/assignment.cu:19-57,65-71.
 * labels[pid[r]] = argmin_c fmaf(-2, dots[r][c], pn[pid[r]] + cn[c]) (lowest index on
 * ties); gaps[pid[r]] = largest - second largest distance (init -1e38 with pid,
 * -1 without). */
int mxk_assign_clusters(int64_t rows, int k, const float* point_norms, const float* centroid_norms,
                        const float* dots, const int* pid, int* labels, float* gaps, void* stream);

/* update_centroids, include/kmeans.cuh:24-25 / src/kernels/update.cu:7-31,41-52.
 * centroids = per-cluster mean of points; empty clusters keep old_centroids. */
int mxk_update_centroids(int64_t n, int d, int k, const float* points, const int* labels,
                         const float* old_centroids, float* centroids, int* counts, void* stream);

/* centroid_shift, include/kmeans.cuh:26-27 / src/kernels/update.cu:32-38,54-61.
 * Writes sum((prev-cur)^2) to device_sum and (synchronously) to *host_result. */
int mxk_centroid_shift(int64_t elements, const float* previous, const float* current,
                       float* device_sum, float* host_result, void* stream);

/* No counterpart in the reference.  The same convergence shift as
 * mxk_centroid_shift for callers that cannot allocate device memory (a plugin
 * inside a framework whose pool owns the device, a loop with a fixed memory
 * budget): its scratch is a fixed device array inside the library (64 KB per
 * GPU, held until exit), so the call allocates nothing.  elements <= 33,554,432,
 * larger inputs return MXK_ERR_INVALID.  The first call on a device looks up the
 * array's device address (make it before any stream capture); calls that overlap
 * on the GPU share the array and race.  device_sum may be NULL. */
int mxk_centroid_shift_noalloc(int64_t elements, const float* previous, const float* current,
                               float* device_sum, float* host_result, void* stream);

/* ---- fused hot op (replaces gemm_mx + assign_clusters, src/kmeans.cu:54-56) ---- */

/* Nearest centroid of `rows` quantized points against k MXFP8 centroids with no
 * N x K product buffer: tcgen05 MMA into TMEM, distance fmaf(-2,dot,pn+cn) and
 * lowest-index argmin in the epilogue.  Writes labels[pid[r]] and, when gaps is
 * not NULL, the two-largest gap (init -1e38) like assign_clusters.
 * start_hint (optional, one label per point, may alias labels): every 128-row
 * tile sweeps the centroids starting at the 192-centroid tile of its first
 * row's hint -- previous labels make the sweep find the minimum early; the
 * result does not depend on the hint. */
int mxk_assign_mx_fused(int bits, int64_t rows, int k, int d, const void* a, const uint8_t* a_scales,
                        const uint8_t* b, const uint8_t* b_scales, const float* point_norms,
                        const float* centroid_norms, const int* pid, int* labels, float* gaps,
                        const int* start_hint, void* stream);

/* mxk_assign_mx_fused with the point quantization inside the kernel (no
 * counterpart in the reference, whose Lloyd step runs quantize_rows and then the
 * GEMM): `rows` FP32 points (points[pid[r]], or points[r] without pid; n_points
 * rows of d floats) are MXFP8-encoded in shared memory with the bytes
 * quantize_rows would produce, so the result equals quantize_rows(8, ...) followed
 * by mxk_assign_mx_fused.  d must be 128. */
int mxk_assign_f32_fused(int64_t rows, int k, int d, const float* points, int64_t n_points, const uint8_t* b,
                         const uint8_t* b_scales, const float* point_norms, const float* centroid_norms,
                         const int* pid, int* labels, float* gaps, const int* start_hint, void* stream);

/* ---- centroid initialisation on the GPU ----------------------------------- */

/* init_centroids_farthest, include/host_utils.hpp:121-141, on device data:
 * centroids (k x d) receive the same rows the reference's host function picks
 * (float squared distances feature by feature, the first maximum; first center
 * row 0).  points: n x d device rows, 16-byte aligned, d % 4 == 0, 1 <= k <= n.
 * Synchronous on `stream`. */
int mxk_init_farthest(int64_t n, int d, int k, const float* points, float* centroids, void* stream);

/* init_centroids, include/host_utils.hpp:80-119 (D^2-sampling K-Means++ with
 * std::mt19937(seed)), on device data: the same rows as the reference's host
 * function for the same seed (same random draws, double distances, and the
 * choice its sequential running sum makes).  Same requirements as
 * mxk_init_farthest; n < 2^31.  Synchronous on `stream`. */
int mxk_init_kmeanspp(int64_t n, int d, int k, const float* points, float* centroids, uint32_t seed,
                      void* stream);

/* ---- Lloyd driver --------------------------------------------------------- */

/* kmeans_mixed, include/kmeans.cuh:20-21 / src/kmeans.cu:12-68.  Points n x d
 * (d padded, % 128 == 0), centroids k x d in/out, labels n out.  *iterations
 * receives the completed iteration count.  Synchronous on `stream`. */
int mxk_kmeans_mixed(int64_t n, int d, int k, const float* points, float* centroids, int* labels,
                     const mxk_options* options, int* iterations, void* stream);

/* Opt-in variant, no reference counterpart: the same Lloyd loop with the points'
 * MXFP8 encoding computed once per call and kept (n * d + n * d / 32 bytes
 * more device memory) instead of re-quantizing every iteration as the
 * reference does (src/kmeans.cu:45-57).  Under the forced-MXFP8 policy the
 * bytes are the same every iteration, so labels and centroids are those of
 * mxk_kmeans_mixed. */
int mxk_kmeans_mixed_cached(int64_t n, int d, int k, const float* points, float* centroids, int* labels,
                            const mxk_options* options, int* iterations, void* stream);

/* Test hook, no counterpart in the reference.  Precision policy of the Lloyd
 * calls that start after it, process-wide.  0 (default): the reference's
 * select_precision (include/precision.hpp:20-26), which always returns MXFP8.
 * 1: the candidate that function computes and discards (precision_candidate,
 * include/precision.hpp:10-17), so points with a large two-largest distance
 * gap go to the MXFP4 / MXFP6 groups and the loop runs the reference's
 * per-precision sequence (src/kmeans.cu:42-57: policy, stable compaction, one
 * quantize + GEMM + assignment per group).  Other values: MXK_ERR_INVALID. */
int mxk_set_precision_policy(int policy);

/* Diagnostics, no counterpart in the reference (whose only per-iteration output
 * is the verbose group-size line, src/kmeans.cu:58-60).  Arms a trace of the
 * NEXT Lloyd call (mxk_kmeans_mixed, _cached or _sharded) made on the current
 * device.  For each iteration i < max_iterations that call copies, into the
 * caller's device buffers (any may be NULL; they must stay valid until the call
 * returns): centroids + i*k*d <- the centroids iteration i assigns against;
 * labels + i*n <- the labels it assigns (the shard's rows in a sharded call);
 * group_sizes + 3*i <- the rows of its MXFP4, MXFP6 and MXFP8 groups (zeros in
 * an FP32 iteration).  Entries of iterations enqueued after the stopping rule
 * fired hold the stopped state (the final centroids and labels, empty groups). */
typedef struct {
    float* centroids;
    int* labels;
    int* group_sizes;
    int max_iterations;
} mxk_trace;
int mxk_trace_next_call(const mxk_trace* trace);

/* ---- multi-GPU (no counterpart in the reference, which is single-GPU) ------ */

/* Row-sharded Lloyd: each rank holds n_local rows; centroids are replicated; per
 * iteration the K x D sums and K counts are NCCL-allreduced.  comm comes from
 * mxk_comm_init (one rank per GPU, any process layout). */
int mxk_comm_unique_id(unsigned char id[128]);
int mxk_comm_init(void** comm, int nranks, int rank, const unsigned char id[128]);
int mxk_comm_destroy(void* comm);
/* Test hook, no reference counterpart: the sharded Lloyd loop of `rank`
 * (mxk_kmeans_mixed_sharded, and the ranks of mxk_kmeans_mixed_multi) returns
 * MXK_ERR_CUDA when it reaches `iteration`, on the host, after the work it has
 * enqueued has finished: a rank that leaves between steps.  rank < 0 disarms.
 * Process-wide. */
int mxk_inject_rank_failure(int rank, int iteration);
int mxk_kmeans_mixed_sharded(void* comm, int64_t n_local, int d, int k, const float* points,
                             float* centroids, int* labels, const mxk_options* options,
                             int* iterations, void* stream);
/* kmeans_mixed over num_gpus GPUs of this node (devices 0..num_gpus-1) from
 * HOST buffers: points n x d (d as kmeans_mixed), centroids k x d in/out,
 * labels n out.  Rows are split into contiguous shards (n / num_gpus each, the
 * first n % num_gpus one more), one host thread per GPU, centroids replicated,
 * sums and counts all-reduced each iteration (mxk_kmeans_mixed_sharded); with
 * num_gpus == 1 it is mxk_kmeans_mixed on device 0.  Blocking; restores the
 * caller's current device. */
int mxk_kmeans_mixed_multi(int64_t n, int d, int k, const float* points, float* centroids, int* labels,
                           const mxk_options* options, int num_gpus, int* iterations);

/* ---- host-side helpers of the CLI (include/host_utils.hpp:40-141) -------- */

/* K-Means++ (std::mt19937(seed) D^2 sampling) and farthest-first centroid
 * initialisation on HOST arrays; same selections as the reference for a seed. */
int mxk_host_init_kmeanspp(const float* points, int64_t n, int d, int k, uint32_t seed, float* out);
int mxk_host_init_farthest(const float* points, int64_t n, int d, int k, float* out);
/* read_points, include/host_utils.hpp:40-67: dense CSV with header, d features
 * (+ optional ignored label column), zero padded to padded_d; rejects
 * non-finite values and row-count mismatches with the reference's messages.
 * Parsed on all host threads; the values are bit-identical to std::stof's. */
int mxk_host_read_points(const char* path, int64_t n, int d, int padded_d, float* out);
/* The same with an explicit thread count (<= 0: all hardware threads) and
 * chunk size in bytes (<= 0: automatic); results do not depend on either. */
int mxk_host_read_points_ex(const char* path, int64_t n, int d, int padded_d, int threads,
                            int64_t chunk_bytes, float* out);
/* Binary fast path (no reference counterpart; the reference reads CSV only):
 * n x d little-endian float32 values, row-major, no header, exactly n*d*4
 * bytes; zero padded to padded_d; non-finite values rejected as in the CSV. */
int mxk_host_read_points_f32(const char* path, int64_t n, int d, int padded_d, float* out);
/* write_labels, include/host_utils.hpp:69-76: "clusters" then one label per
 * line, the same bytes as the reference (formatted on all host threads). */
int mxk_host_write_labels(const char* path, const int* labels, int64_t n);

/* ---- kernel timing (CUDA events around each launch on its stream) ---------- */
int mxk_profile_enable(int on);
/* Copies up to max entries of {name, launches, total_ms} for the current device. */
typedef struct {
    char name[48];
    uint64_t launches;
    double total_ms;
} mxk_kernel_stat;
int mxk_profile_read(mxk_kernel_stat* out, int max, int* count);

#ifdef __cplusplus
}
#endif
#endif
