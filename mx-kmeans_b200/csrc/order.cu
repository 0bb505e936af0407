// Label-sorted point order for the Lloyd driver.
//
// Each iteration after the first, the driver visits the points grouped by the
// label they received in the previous iteration (a counting sort of the point
// indices over the k labels).  Results are unchanged -- every point's
// assignment is independent of where it sits in the sequence -- but 32
// consecutive rows of a GEMM tile then mostly share a nearest centroid, which
// keeps the argmin epilogue's rare index-search branch warp-uniform, and the
// update sees long runs of equal labels, so its per-run flushes replace one
// atomic reduction per point.
#include "common.cuh"
#include "kernels.cuh"

#include <algorithm>

namespace mxk {
namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kSmemBins = 16384;  // keys counted in shared memory up to this k

__device__ __forceinline__ int clamp_key(int v, int k) { return (unsigned)v < (unsigned)k ? v : k - 1; }

__global__ void __launch_bounds__(512) label_histogram_kernel(int64_t n, int k, const int* __restrict__ labels,
                                                              int* __restrict__ hist, const int* __restrict__ stop) {
    if (stop && *stop) return;  // the Lloyd loop has already converged
    extern __shared__ int local[];
    const bool use_smem = k <= kSmemBins;
    if (use_smem) {
        for (int i = threadIdx.x; i < k; i += blockDim.x) local[i] = 0;
        __syncthreads();
    }
    for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < n; p += (int64_t)gridDim.x * blockDim.x) {
        const int key = clamp_key(labels[p], k);
        const unsigned peers = __match_any_sync(__activemask(), key);
        if ((threadIdx.x & 31) == __ffs(peers) - 1) {
            if (use_smem)
                atomicAdd(&local[key], __popc(peers));
            else
                atomicAdd(&hist[key], __popc(peers));
        }
    }
    if (use_smem) {
        __syncthreads();
        for (int i = threadIdx.x; i < k; i += blockDim.x)
            if (local[i]) atomicAdd(&hist[i], local[i]);
    }
}

// Exclusive scan of the k counts (one block of 1024 threads).
__global__ void __launch_bounds__(1024) label_scan_kernel(int k, int* __restrict__ hist,
                                                          const int* __restrict__ stop) {
    if (stop && *stop) return;
    __shared__ int warp_tot[32];
    __shared__ int carry;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (int base = 0; base < k; base += blockDim.x) {
        const int i = base + threadIdx.x;
        const int v = i < k ? hist[i] : 0;
        int incl = v;
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(kFull, incl, o);
            if (lane >= o) incl += t;
        }
        if (lane == 31) warp_tot[warp] = incl;
        __syncthreads();
        if (warp == 0) {
            int w = lane < (int)(blockDim.x >> 5) ? warp_tot[lane] : 0;
            int wi = w;
            for (int o = 1; o < 32; o <<= 1) {
                const int t = __shfl_up_sync(kFull, wi, o);
                if (lane >= o) wi += t;
            }
            warp_tot[lane] = wi - w;  // exclusive warp offsets
        }
        __syncthreads();
        if (i < k) hist[i] = carry + warp_tot[warp] + incl - v;
        __syncthreads();
        if (threadIdx.x == blockDim.x - 1) carry += warp_tot[warp] + incl;
        __syncthreads();
    }
}

// Block-aggregated scatter: each CTA owns a contiguous slice of the points,
// counts its keys in shared memory, reserves one range per present key with a
// single global atomic, and places its points through shared-memory cursors.
__global__ void __launch_bounds__(512) label_scatter_block_kernel(int64_t n, int k, const int* __restrict__ labels,
                                                                  int* __restrict__ offsets, int* __restrict__ order,
                                                                  int64_t per_block, const int* __restrict__ stop) {
    if (stop && *stop) return;
    extern __shared__ int cursor[];
    const int64_t begin = (int64_t)blockIdx.x * per_block;
    const int64_t end = begin + per_block < n ? begin + per_block : n;
    for (int i = threadIdx.x; i < k; i += blockDim.x) cursor[i] = 0;
    __syncthreads();
    const int lane = threadIdx.x & 31;
    for (int64_t b = begin; b < end; b += blockDim.x) {
        const int64_t p = b + threadIdx.x;
        const int key = p < end ? clamp_key(labels[p], k) : -1;
        const unsigned peers = __match_any_sync(kFull, key);
        if (key >= 0 && lane == __ffs(peers) - 1) atomicAdd(&cursor[key], __popc(peers));
    }
    __syncthreads();
    for (int i = threadIdx.x; i < k; i += blockDim.x) {
        const int c = cursor[i];
        cursor[i] = c ? atomicAdd(&offsets[i], c) : 0;
    }
    __syncthreads();
    for (int64_t b = begin; b < end; b += blockDim.x) {
        const int64_t p = b + threadIdx.x;
        const int key = p < end ? clamp_key(labels[p], k) : -1;
        const unsigned peers = __match_any_sync(kFull, key);
        const int leader = __ffs(peers) - 1;
        int pos = 0;
        if (key >= 0 && lane == leader) pos = atomicAdd(&cursor[key], __popc(peers));
        pos = __shfl_sync(kFull, pos, leader);
        if (key >= 0) order[pos + __popc(peers & ((1u << lane) - 1u))] = (int)p;
    }
}

// The same scatter over the current visiting order when per-row state follows
// it (RowState): CTA slices of positions g, key = rs.label[g]; the point id
// order[g], its record and label go to the new position in rs.tmp_*, which
// row_state_copy_kernel copies back.  Points keep their relative order within
// a CTA's slice, so records move in short runs.
__global__ void __launch_bounds__(512) label_scatter_rows_kernel(int64_t n, int k, const int* __restrict__ order,
                                                                 int* __restrict__ offsets, int64_t per_block,
                                                                 RowState rs, const int* __restrict__ stop) {
    if (stop && *stop) return;
    extern __shared__ int cursor[];
    const int64_t begin = (int64_t)blockIdx.x * per_block;
    const int64_t end = begin + per_block < n ? begin + per_block : n;
    for (int i = threadIdx.x; i < k; i += blockDim.x) cursor[i] = 0;
    __syncthreads();
    const int lane = threadIdx.x & 31;
    for (int64_t b = begin; b < end; b += blockDim.x) {
        const int64_t g = b + threadIdx.x;
        const int key = g < end ? clamp_key(rs.label[g], k) : -1;
        const unsigned peers = __match_any_sync(kFull, key);
        if (key >= 0 && lane == __ffs(peers) - 1) atomicAdd(&cursor[key], __popc(peers));
    }
    __syncthreads();
    for (int i = threadIdx.x; i < k; i += blockDim.x) {
        const int c = cursor[i];
        cursor[i] = c ? atomicAdd(&offsets[i], c) : 0;
    }
    __syncthreads();
    for (int64_t b = begin; b < end; b += blockDim.x) {
        const int64_t g = b + threadIdx.x;
        const int label = g < end ? rs.label[g] : -1;
        const int key = g < end ? clamp_key(label, k) : -1;
        const unsigned peers = __match_any_sync(kFull, key);
        const int leader = __ffs(peers) - 1;
        int pos = 0;
        if (key >= 0 && lane == leader) pos = atomicAdd(&cursor[key], __popc(peers));
        pos = __shfl_sync(kFull, pos, leader);
        if (key >= 0) {
            const int dst = pos + __popc(peers & ((1u << lane) - 1u));
            rs.tmp_order[dst] = order[g];
            if (rs.state) rs.tmp_state[dst] = rs.state[g];
            rs.tmp_label[dst] = label;
        }
    }
}

// order[offset[key]++] = p, one atomic per group of equal keys within a warp
// (used when k is too large for the shared-memory cursors).
__global__ void __launch_bounds__(512) label_scatter_kernel(int64_t n, int k, const int* __restrict__ labels,
                                                            int* __restrict__ offsets, int* __restrict__ order,
                                                            const int* __restrict__ stop) {
    if (stop && *stop) return;
    for (int64_t base = (int64_t)blockIdx.x * blockDim.x; base < n; base += (int64_t)gridDim.x * blockDim.x) {
        const int64_t p = base + threadIdx.x;
        const bool valid = p < n;
        const int key = valid ? clamp_key(labels[p], k) : -1;
        const unsigned peers = __match_any_sync(kFull, key);
        const int lane = threadIdx.x & 31;
        const int leader = __ffs(peers) - 1;
        int pos = 0;
        if (valid && lane == leader) pos = atomicAdd(&offsets[key], __popc(peers));
        pos = __shfl_sync(kFull, pos, leader);
        if (valid) order[pos + __popc(peers & ((1u << lane) - 1u))] = (int)p;
    }
}

// The new order, records and labels copied back from RowState's scratch.
__global__ void __launch_bounds__(256) row_state_copy_kernel(int64_t n, RowState rs, int* __restrict__ order,
                                                             const int* __restrict__ stop) {
    if (stop && *stop) return;
    for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < n; g += (int64_t)gridDim.x * blockDim.x) {
        order[g] = rs.tmp_order[g];
        if (rs.state) rs.state[g] = rs.tmp_state[g];
        rs.label[g] = rs.tmp_label[g];
    }
}

__global__ void __launch_bounds__(256) iota_kernel(int64_t n, int* __restrict__ v) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        v[i] = (int)i;
}

// ctl = (label changes since the visiting order was last rebuilt, skip word).
// The skip word is set (the label sort that follows does nothing) while the
// loop has stopped or fewer than `threshold` labels have changed since the last
// rebuild, counting this iteration's *changes; otherwise it is cleared and the
// count starts over.
__global__ void sort_gate_kernel(const int* __restrict__ stop, const int* __restrict__ changes, int* __restrict__ ctl,
                                 int threshold) {
    if (threadIdx.x != 0) return;
    if (stop && *stop) {
        ctl[1] = 1;
        return;
    }
    const int since = ctl[0] + *changes;
    const bool sort = since >= threshold;
    ctl[0] = sort ? 0 : since;
    ctl[1] = sort ? 0 : 1;
}

}  // namespace

int launch_sort_gate(const int* stop, const int* changes, int* ctl, int threshold, cudaStream_t stream) {
    MXK_REQUIRE(changes && ctl, "sort_gate: bad arguments");
    LaunchScope scope("sort_gate", stream);
    sort_gate_kernel<<<1, 32, 0, stream>>>(stop, changes, ctl, threshold);
    MXK_CUDA(cudaGetLastError());
    return MXK_OK;
}

int64_t label_sort_scratch_ints(int k) { return k; }

int launch_identity_order(int64_t n, int* order, cudaStream_t stream) {
    if (n <= 0) return MXK_OK;
    LaunchScope scope("identity_order", stream);
    iota_kernel<<<sm_count() * 4, 256, 0, stream>>>(n, order);
    MXK_CUDA(cudaGetLastError());
    return MXK_OK;
}

int launch_label_sort(int64_t n, int k, const int* labels, int* order, int* scratch, cudaStream_t stream,
                      const int* stop, const RowState* row_state) {
    if (n <= 0) return MXK_OK;
    MXK_REQUIRE(k > 0 && labels && order && scratch, "label_sort: bad arguments");
    const RowState rs = row_state ? *row_state : RowState{};
    MXK_REQUIRE(!row_state || (rs.label && rs.tmp_state && rs.tmp_label && rs.tmp_order && k <= kSmemBins),
                "label_sort: incomplete row state, or k above the shared-memory cursors");
    MXK_CUDA(cudaMemsetAsync(scratch, 0, sizeof(int) * (size_t)k, stream));
    const int sms = sm_count();
    const size_t smem = k <= kSmemBins ? sizeof(int) * (size_t)k : 0;
    if (smem > 48 * 1024)
        MXK_CUDA(cudaFuncSetAttribute(label_histogram_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    {
        LaunchScope scope("label_histogram", stream);
        label_histogram_kernel<<<sms * 2, 512, smem, stream>>>(n, k, labels, scratch, stop);
        MXK_CUDA(cudaGetLastError());
    }
    {
        LaunchScope scope("label_scan", stream);
        label_scan_kernel<<<1, 1024, 0, stream>>>(k, scratch, stop);
        MXK_CUDA(cudaGetLastError());
    }
    if (row_state) {
        const int64_t blocks = std::min<int64_t>((int64_t)sms * 2, (n + 4095) / 4096);
        const int64_t per_block = (n + blocks - 1) / blocks;
        if (smem > 48 * 1024)
            MXK_CUDA(cudaFuncSetAttribute(label_scatter_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)smem));
        {
            LaunchScope scope("label_scatter", stream);
            label_scatter_rows_kernel<<<(unsigned)blocks, 512, smem, stream>>>(n, k, order, scratch, per_block, rs,
                                                                               stop);
            MXK_CUDA(cudaGetLastError());
        }
        LaunchScope scope("row_state_copy", stream);
        row_state_copy_kernel<<<sms * 8, 256, 0, stream>>>(n, rs, order, stop);
        MXK_CUDA(cudaGetLastError());
    } else if (k <= kSmemBins) {
        const int64_t blocks = std::min<int64_t>((int64_t)sms * 2, (n + 4095) / 4096);
        const int64_t per_block = (n + blocks - 1) / blocks;
        if (smem > 48 * 1024)
            MXK_CUDA(cudaFuncSetAttribute(label_scatter_block_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)smem));
        LaunchScope scope("label_scatter", stream);
        label_scatter_block_kernel<<<(unsigned)blocks, 512, smem, stream>>>(n, k, labels, scratch, order, per_block,
                                                                                stop);
        MXK_CUDA(cudaGetLastError());
    } else {
        LaunchScope scope("label_scatter", stream);
        label_scatter_kernel<<<sms * 4, 512, 0, stream>>>(n, k, labels, scratch, order, stop);
        MXK_CUDA(cudaGetLastError());
    }
    return MXK_OK;
}

}  // namespace mxk
