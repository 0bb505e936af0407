// Multi-GPU entry of the C++ drop-in API.  The reference's include/kmeans.cuh
// (ParCIS/MX-KMeans, single-GPU) stays unchanged; this header adds the
// row-sharded Lloyd over several GPUs of one node, same options and
// exceptions as kmeans_mixed.
#pragma once

#include <cstdint>

#include "kmeans.cuh"

// Points (n x d), centroids (k x d, in/out) and labels (n, out) are HOST
// arrays; d follows kmeans_mixed's rules.  The rows are sharded over devices
// 0..num_gpus-1 (contiguous, n / num_gpus each, the first n % num_gpus one
// more); the centroids are replicated and the per-cluster sums and counts are
// all-reduced over NCCL every iteration, so every GPU finalizes the same
// centroids.  Returns the number of completed Lloyd iterations.
int kmeans_mixed_multi(int64_t n, int d, int k, const float* host_points, float* host_centroids, int* host_labels,
                       const KMeansOptions& options, int num_gpus);
