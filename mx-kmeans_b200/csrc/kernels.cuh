// Internal launchers shared by the C-ABI entry points and the Lloyd driver.
// All return an mxk_status; pointers are device pointers; launches go to
// `stream` and do not synchronize.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mxk {

// ---- quantize.cu ------------------------------------------------------------
// rows_dev (optional): device-resident row count that overrides `rows`, which
// then only sizes the grid (an upper bound).
int launch_quantize(int bits, int64_t rows, int d, const float* points, const int* pid, void* values,
                    uint8_t* scales, float* max_errors, const int* rows_dev, cudaStream_t stream);
int launch_l2_norm(int64_t rows, int d, const float* x, float* norms, cudaStream_t stream);
int launch_point_bounds(int64_t n, int d, const float* points, const float* norms, float* upper,
                        cudaStream_t stream);
// lc/ec either as host values (lc_dev == nullptr) or read from device memory.
int launch_assign_precisions(int64_t n, int d, const float* upper, const float* gaps, float lc, float ec,
                             const float* lc_ec_dev, int* precision, int* group_counts, cudaStream_t stream);
// stats[0] = sqrt(max errors), stats[1] = sqrt(max norms)  (src/kmeans.cu:38-41)
int launch_centroid_stats(int k, const float* errors, const float* norms, float* stats, cudaStream_t stream);
// Stable per-precision compaction of point ids (src/kmeans.cu:45-52).
// ids: 3*n ints (groups 4, 6, 8 at offsets 0, n, 2n); group_counts: 3 ints.
// scratch: compaction_scratch_ints(n) ints.
int64_t compaction_scratch_ints(int64_t n);
int launch_group_compaction(int64_t n, const int* precision, int* ids, int* group_counts, int* scratch,
                            cudaStream_t stream);

// ---- gemm_mx.cu ---------------------------------------------------------------
struct MxArgmin {
    const float* point_norms = nullptr;     // indexed by pid[row] (or row)
    const float* centroid_norms = nullptr;  // k
    const int* pid = nullptr;
    int* labels = nullptr;
    float* gaps = nullptr;  // optional two-largest gap (init -1e38)
};
// Dense: out[m x n] = A . B^T.  Argmin: labels of the m rows against n centroids.
// rows_dev (optional) = device-resident m (m is then an upper bound).
int launch_gemm_mx(int bits, int64_t m, int64_t n, int k, const void* a, const uint8_t* a_scales,
                   const uint8_t* b, const uint8_t* b_scales, float* out, const MxArgmin* argmin,
                   const int* rows_dev, cudaStream_t stream);

// ---- fp32.cu -----------------------------------------------------------------
int launch_gemm_fp32(int64_t m, int64_t n, int k, const float* a, const float* b, float* out,
                     cudaStream_t stream);

// ---- assign.cu ---------------------------------------------------------------
int launch_assign_clusters(int64_t rows, int k, const float* point_norms, const float* centroid_norms,
                           const float* dots, const int* pid, int* labels, float* gaps, cudaStream_t stream);

// ---- update.cu ---------------------------------------------------------------
// sums (k x d) and counts (k) must be zeroed by the caller.
int launch_accumulate(int64_t n, int d, int k, const float* points, const int* labels, float* sums,
                      int* counts, cudaStream_t stream);
// centroids = counts ? sums / counts : old.  If shift_scratch is not null
// (shift_scratch_floats() floats), its last element receives sum((old - new)^2),
// reduced in a fixed order (bit-reproducible).  sums and centroids may alias.
int64_t shift_scratch_floats();
int launch_finalize(int d, int k, const float* sums, const int* counts, const float* old_centroids,
                    float* centroids, float* shift_scratch, cudaStream_t stream);
// sum((previous - current)^2) into shift_scratch[shift_scratch_floats() - 1].
int launch_shift(int64_t elements, const float* previous, const float* current, float* shift_scratch,
                 cudaStream_t stream);

}  // namespace mxk
