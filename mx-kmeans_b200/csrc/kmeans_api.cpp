// C++ drop-in API (include/kmeans.cuh) over the C ABI (include/mxk.h).
// Reference declarations: ParCIS/MX-KMeans include/kmeans.cuh:20-47.
#include <stdexcept>
#include <string>

#include "kmeans.cuh"
#include "kmeans_multi.cuh"
#include "mxk.h"

namespace {
void throw_on(int status) {
    if (status == MXK_OK) return;
    const std::string message = mxk_last_error();
    if (status == MXK_ERR_INVALID) throw std::invalid_argument(message);
    throw std::runtime_error(message);
}
}  // namespace

int kmeans_mixed(int n, int d, int k, const float* points, float* centroids, int* labels,
                 const KMeansOptions& options) {
    mxk_options o{options.max_iterations, options.fp32_iterations, options.tolerance, options.verbose ? 1 : 0};
    int iterations = 0;
    throw_on(mxk_kmeans_mixed(n, d, k, points, centroids, labels, &o, &iterations, nullptr));
    return iterations;
}

int kmeans_mixed_multi(int64_t n, int d, int k, const float* host_points, float* host_centroids, int* host_labels,
                       const KMeansOptions& options, int num_gpus) {
    mxk_options o{options.max_iterations, options.fp32_iterations, options.tolerance, options.verbose ? 1 : 0};
    int iterations = 0;
    throw_on(mxk_kmeans_mixed_multi(n, d, k, host_points, host_centroids, host_labels, &o, num_gpus, &iterations));
    return iterations;
}

void compute_l2_norm(int rows, int d, const float* points, float* norms) {
    throw_on(mxk_compute_l2_norm(rows, d, points, norms, nullptr));
}

void update_centroids(int n, int d, int k, const float* points, const int* labels, const float* old_centroids,
                      float* centroids, int* counts) {
    throw_on(mxk_update_centroids(n, d, k, points, labels, old_centroids, centroids, counts, nullptr));
}

float centroid_shift(int elements, const float* previous, const float* current, float* device_sum) {
    float result = 0.0f;
    throw_on(mxk_centroid_shift(elements, previous, current, device_sum, &result, nullptr));
    return result;
}

void assign_clusters(int rows, int k, const float* point_norms, const float* centroid_norms, const float* dots,
                     const int* pid, int* labels, float* gaps) {
    throw_on(mxk_assign_clusters(rows, k, point_norms, centroid_norms, dots, pid, labels, gaps, nullptr));
}

void precompute_point_bounds(int n, int d, const float* points, const float* norms, float* upper) {
    throw_on(mxk_precompute_point_bounds(n, d, points, norms, upper, nullptr));
}

void assign_precisions(int n, int d, const float* upper, const float* gaps, float lc, float ec, int* precision) {
    throw_on(mxk_assign_precisions(n, d, upper, gaps, lc, ec, precision, nullptr));
}

void quantize_rows(int bits, int rows, int d, const float* points, const int* pid, void* values, Scale* scales,
                   float* max_errors) {
    throw_on(mxk_quantize_rows(bits, rows, d, points, pid, values, reinterpret_cast<uint8_t*>(scales), max_errors,
                               nullptr));
}

void gemm_fp32(int m, int n, int k, const float* a, const float* b, float* out) {
    throw_on(mxk_gemm_fp32(m, n, k, a, b, out, nullptr));
}

void gemm_mx(int bits, int m, int n, int k, const void* a, const Scale* a_scales, const MXFP8* b, const Scale* b_scales,
             float* out) {
    throw_on(mxk_gemm_mx(bits, m, n, k, a, reinterpret_cast<const uint8_t*>(a_scales),
                         reinterpret_cast<const uint8_t*>(b), reinterpret_cast<const uint8_t*>(b_scales), out, nullptr));
    // The reference's gemm_mx synchronizes the device before returning (src/kernels/gemm.cu:134).
    CUDA_CHECK(cudaDeviceSynchronize());
}
