/*
 * CPU oracle for the MX-KMeans Lloyd iteration.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker that the parity tests,
 * `__graft_entry__.smoke()` and the CPU-baseline leg of `bench.py` compare the
 * CUDA product against.  Nothing in the product (`mx-kmeans_b200/`, `include/`)
 * links, loads or calls it.
 *
 * It restates, in plain C, the arithmetic of ParCIS/MX-KMeans for one Lloyd
 * iteration of `kmeans_mixed` (src/kmeans.cu:12-68): MX quantization
 * (src/kernels/quantize.cu), the precision policy (include/precision.hpp),
 * nearest-centroid assignment (src/kernels/assignment.cu), the centroid update
 * and convergence shift (src/kernels/update.cu) and the reconstructed-value GEMM
 * check of tests/cuda_checks.cu:23-33,75-86.  Each function cites the reference
 * lines it follows.
 *
 * The MX element and scale conversions of the reference come from CUTLASS
 * (cutlass/float8.h, cutlass/exmy_base.h; pinned 4.3.5 @ 6b3e607, present here
 * as 4.5.0) and CUDA cuda_fp6.h.  They are restated from their published rule
 * (IEEE round-to-nearest-even with saturation to the largest finite value; the
 * UE8M0 scale rounds toward +inf) and pinned against the installed CUTLASS host
 * conversions by oracle/cutlass_pin.cpp.
 */
#ifndef MXK_ORACLE_H
#define MXK_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element formats */
enum { ORC_E4M3 = 0, ORC_E2M3 = 1, ORC_E2M1 = 2, ORC_E3M2 = 3, ORC_UE8M0 = 4 };

uint8_t orc_encode(int format, float x);
float orc_decode_elem(int format, uint8_t bits);
void orc_encode_batch(int format, int64_t n, const float* in, uint8_t* out);
void orc_decode_batch(int format, int64_t n, const uint8_t* in, float* out);

/* include/precision.hpp:10-48 */
int orc_precision_candidate(float p4, float p6, float lc, int dimensions, float gap);
int orc_select_precision(float p4, float p6, float lc, float ec, int dimensions, float gap);

/* src/kernels/assignment.cu:7-16 */
void orc_l2_norm(int64_t rows, int d, const float* x, float* norms);

/* src/kernels/quantize.cu:13-72,111-123 */
int orc_quantize_rows(int bits, int64_t rows, int d, const float* points, const int* pid,
                      uint8_t* values, uint8_t* scales, float* max_errors);
/* src/kernels/quantize.cu:74-98 */
void orc_point_bounds(int64_t n, int d, const float* points, const float* norms, float* upper);
/* src/kernels/quantize.cu:100-108 */
void orc_assign_precisions(int64_t n, int d, const float* upper, const float* gaps, float lc,
                           float ec, int* precision);

/* tests/cuda_checks.cu:23-33 */
float orc_decode_packed(const uint8_t* bytes, const uint8_t* scales, int bits, int64_t row, int d,
                        int feature);
void orc_dequantize_rows(int bits, int64_t rows, int d, const uint8_t* bytes, const uint8_t* scales,
                         float* out);
/* tests/cuda_checks.cu:75-86: double products of reconstructed values */
void orc_gemm_mx(int bits, int64_t m, int64_t n, int k, const uint8_t* a, const uint8_t* a_scales,
                 const uint8_t* b, const uint8_t* b_scales, double* out, double* magnitude);
/* plain FP32-input product accumulated in double (src/kernels/gemm.cu:365-380 semantics) */
void orc_gemm_f32(int64_t m, int64_t n, int k, const float* a, const float* b, double* out);

/* src/kernels/assignment.cu:19-57 */
void orc_assign_clusters(int64_t rows, int k, const float* point_norms, const float* centroid_norms,
                         const float* dots, const int* pid, int* labels, float* gaps);
/* true nearest / second nearest (not exported by the reference; used for label tolerance) */
void orc_top2(int64_t rows, int k, const float* point_norms, const float* centroid_norms,
              const float* dots, int* nearest, float* first, float* second);

/* src/kernels/update.cu:7-31,41-52 (sums in point order, float) */
void orc_update_centroids(int64_t n, int d, int k, const float* points, const int* labels,
                          const float* old_centroids, float* centroids, int* counts);
/* src/kernels/update.cu:32-38,54-61 */
float orc_centroid_shift(int64_t elements, const float* previous, const float* current);
/* sum over points of |x - c_label|^2 in double */
double orc_inertia(int64_t n, int d, const float* points, const float* centroids, const int* labels);

/* src/kmeans.cu:12-68.  Returns iterations (>0) or a negative error code:
 * -1 non-finite shift, -2 bad argument. threads<=0 uses all host cores. */
int orc_kmeans_mixed(int64_t n, int d, int k, const float* points, float* centroids, int* labels,
                     int max_iterations, int fp32_iterations, float tolerance, int threads);
/* orc_kmeans_mixed with a precision policy (0: select_precision, the
 * reference; 1: precision_candidate's choice, the library's test hook) and,
 * when group_sizes is not NULL, the rows of the MXFP4/6/8 groups of every MX
 * iteration at group_sizes[3 * it + g] (entries of FP32 iterations untouched). */
int orc_kmeans_mixed_ex(int64_t n, int d, int k, const float* points, float* centroids, int* labels,
                        int max_iterations, int fp32_iterations, float tolerance, int threads, int policy,
                        int* group_sizes);

/* One MX Lloyd step from given centroids (quantize, product, assign, update, shift):
 * the unit the step-parity tests and the CPU baseline use. */
float orc_lloyd_step(int64_t n, int d, int k, const float* points, const float* point_norms,
                     float* centroids, int* labels, float* dots_out, int threads);

/* FP32 Lloyd (dots in FP32 from unquantized values), the reported CPU baseline. */
int orc_lloyd_fp32(int64_t n, int d, int k, const float* points, float* centroids, int* labels,
                   int max_iterations, float tolerance, int threads);

int orc_hardware_threads(void);

#ifdef __cplusplus
}
#endif
#endif
