// Nearest-centroid assignment over a dense product matrix (the reference's
// assign_clusters op, src/kernels/assignment.cu:19-57,65-71).  The Lloyd driver
// does not use it -- its assignment is fused into the tcgen05 GEMM epilogue --
// but the op is part of the drop-in API and of the FP32-iteration path.
#include "common.cuh"
#include "kernels.cuh"
#include "precision.hpp"

namespace mxk {
namespace {

constexpr unsigned kFull = 0xffffffffu;

// One warp per row: each lane scans columns lane, lane+32, ..., then the lanes
// merge (distance, index) with the lowest index on ties and the two largest
// distances.  Same statistics and initial values as the reference.
__global__ void __launch_bounds__(256) nearest_kernel(int64_t rows, int k, const float* __restrict__ pn,
                                                      const float* __restrict__ cn, const float* __restrict__ dots,
                                                      const int* __restrict__ pid, int* __restrict__ labels,
                                                      float* __restrict__ gaps) {
    const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const int64_t point = pid ? (int64_t)pid[row] : row;
    float first = __int_as_float(0x7f800000), second = first;
    float largest = pid ? -1e38f : -1.0f;
    float next_largest = largest;
    int best = 0x7fffffff;
    const float pnv = pn[point];
    const float* drow = dots + row * k;
    for (int c = lane; c < k; c += 32) {
        const float dist = fmaf(-2.0f, drow[c], pnv + cn[c]);
        insert_distance(dist, c, first, second, best);
        insert_largest_distance(dist, largest, next_largest);
    }
    for (int o = 16; o; o >>= 1) {
        const float of = __shfl_xor_sync(kFull, first, o);
        const int ob = __shfl_xor_sync(kFull, best, o);
        const float ol = __shfl_xor_sync(kFull, largest, o);
        const float on = __shfl_xor_sync(kFull, next_largest, o);
        if (of < first || (of == first && ob < best)) {
            first = of;
            best = ob;
        }
        next_largest = fmaxf(fminf(largest, ol), fmaxf(next_largest, on));
        largest = fmaxf(largest, ol);
    }
    if (lane == 0) {
        labels[point] = best;
        if (gaps) gaps[point] = largest - next_largest;
    }
}

}  // namespace

int launch_assign_clusters(int64_t rows, int k, const float* point_norms, const float* centroid_norms,
                           const float* dots, const int* pid, int* labels, float* gaps, cudaStream_t stream) {
    if (rows <= 0) return MXK_OK;
    MXK_REQUIRE(k > 0 && point_norms && centroid_norms && dots && labels, "assign_clusters: bad arguments");
    const int64_t blocks = (rows * 32 + 255) / 256;
    MXK_REQUIRE(blocks < (1ll << 31), "assign_clusters: too many rows");
    LaunchScope scope("assign_dense", stream);
    nearest_kernel<<<(unsigned)blocks, 256, 0, stream>>>(rows, k, point_norms, centroid_norms, dots, pid, labels, gaps);
    MXK_CUDA(cudaGetLastError());
    return MXK_OK;
}

}  // namespace mxk

extern "C" int mxk_assign_clusters(int64_t rows, int k, const float* point_norms, const float* centroid_norms,
                                   const float* dots, const int* pid, int* labels, float* gaps, void* stream) {
    return mxk::launch_assign_clusters(rows, k, point_norms, centroid_norms, dots, pid, labels, gaps,
                                       mxk::as_stream(stream));
}
