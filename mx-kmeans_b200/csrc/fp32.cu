// FP32 product for the `--fp32-iters` warm-up iterations (the reference's
// gemm_fp32, src/kernels/gemm.cu:365-380: cuBLAS SGEMM with pedantic math, i.e.
// plain FP32 FMAs and no TF32).  out[m x n] = A[m x k] . B[n x k]^T, every
// output accumulated by FMA in increasing k.
#include "common.cuh"
#include "kernels.cuh"

namespace mxk {
namespace {

constexpr int kTile = 128, kSlice = 8, kThreadsF = 256;

__global__ void __launch_bounds__(kThreadsF) sgemm_nt_kernel(int64_t m, int64_t n, int k, const float* __restrict__ a,
                                                             const float* __restrict__ b, float* __restrict__ out) {
    __shared__ float As[2][kSlice][kTile + 4];
    __shared__ float Bs[2][kSlice][kTile + 4];
    const int tid = threadIdx.x;
    const int64_t row0 = (int64_t)blockIdx.y * kTile, col0 = (int64_t)blockIdx.x * kTile;
    const int tr = tid / 16, tc = tid % 16;  // 16 x 16 threads, 8 x 8 outputs each
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;

    // each thread loads 4 consecutive k of one row of A and of B per slice
    const int lrow = tid / 2, lk = (tid % 2) * 4;
    const bool vec = (k % 4 == 0) && ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) % 16 == 0);
    auto load = [&](const float* src, int64_t rbase, int64_t rows, int k0, float (&v)[4]) {
        const int64_t r = rbase + lrow;
        if (r < rows && vec && k0 + lk + 3 < k) {
            const float4 t = *reinterpret_cast<const float4*>(src + r * k + k0 + lk);
            v[0] = t.x, v[1] = t.y, v[2] = t.z, v[3] = t.w;
        } else {
#pragma unroll
            for (int q = 0; q < 4; ++q) v[q] = (r < rows && k0 + lk + q < k) ? src[r * k + k0 + lk + q] : 0.0f;
        }
    };
    float ra[4], rb[4];
    load(a, row0, m, 0, ra);
    load(b, col0, n, 0, rb);
#pragma unroll
    for (int q = 0; q < 4; ++q) As[0][lk + q][lrow] = ra[q], Bs[0][lk + q][lrow] = rb[q];
    __syncthreads();
    int buf = 0;
    for (int k0 = 0; k0 < k; k0 += kSlice) {
        const bool more = k0 + kSlice < k;
        if (more) {
            load(a, row0, m, k0 + kSlice, ra);
            load(b, col0, n, k0 + kSlice, rb);
        }
#pragma unroll
        for (int kk = 0; kk < kSlice; ++kk) {
            float av[8], bv[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) av[i] = As[buf][kk][tr * 8 + i];
#pragma unroll
            for (int j = 0; j < 8; ++j) bv[j] = Bs[buf][kk][tc * 8 + j];
            if (k0 + kk < k) {
#pragma unroll
                for (int i = 0; i < 8; ++i)
#pragma unroll
                    for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
            }
        }
        if (more) {
#pragma unroll
            for (int q = 0; q < 4; ++q) As[buf ^ 1][lk + q][lrow] = ra[q], Bs[buf ^ 1][lk + q][lrow] = rb[q];
        }
        __syncthreads();
        buf ^= 1;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int64_t r = row0 + tr * 8 + i;
        if (r >= m) continue;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int64_t c = col0 + tc * 8 + j;
            if (c < n) out[r * n + c] = acc[i][j];
        }
    }
}

}  // namespace

int launch_gemm_fp32(int64_t m, int64_t n, int k, const float* a, const float* b, float* out, cudaStream_t stream) {
    if (m <= 0 || n <= 0) return MXK_OK;
    MXK_REQUIRE(k > 0 && a && b && out, "gemm_fp32: bad arguments");
    const int64_t gy = (m + kTile - 1) / kTile, gx = (n + kTile - 1) / kTile;
    MXK_REQUIRE(gy < 65536 && gx < (1ll << 31), "gemm_fp32: shape too large for one launch");
    LaunchScope scope("sgemm_nt", stream);
    sgemm_nt_kernel<<<dim3((unsigned)gx, (unsigned)gy), kThreadsF, 0, stream>>>(m, n, k, a, b, out);
    MXK_CUDA(cudaGetLastError());
    return MXK_OK;
}

}  // namespace mxk

extern "C" int mxk_gemm_fp32(int64_t m, int64_t n, int k, const float* a, const float* b, float* out, void* stream) {
    return mxk::launch_gemm_fp32(m, n, k, a, b, out, mxk::as_stream(stream));
}
