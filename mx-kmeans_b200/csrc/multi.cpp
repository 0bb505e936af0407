// kmeans_mixed over several GPUs of this node from host buffers: the
// "kmeans_mixed_multi" entry of the multi-GPU path (the reference,
// ParCIS/MX-KMeans src/kmeans.cu:12-68, runs on one GPU only).
//
// Rows are split into contiguous shards (n / G rows each, the first n % G
// shards one more), shard g lives on device g, centroids are replicated, and
// every Lloyd iteration all-reduces the K x D sums and K counts over NCCL
// (mxk_kmeans_mixed_sharded).  One host thread drives each GPU.  Allocations
// and the centroids' upload run first on every GPU; the communicator is
// created only once all of them have succeeded, so a failed allocation cannot
// leave the other ranks waiting in NCCL initialisation.  Each shard's points
// are then copied in row chunks by the Lloyd call itself, which starts the
// first iteration on the chunks that have landed.  A rank that fails raises a flag
// shared by the ranks; the others' host waits poll it, abort their
// communicators (which ends the collectives that wait for the failed rank) and
// return an error, so the call reports the failure instead of hanging.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <string>
#include <thread>
#include <vector>

#include "mxk.h"

namespace mxk {
int fail(int status, const std::string& message);
void comm_attach_group_flag(void* comm, std::atomic<int>* flag);
void comm_abort(void* comm);
cudaMemPool_t workspace_pool();
int kmeans_mixed_from_host(void* comm, int64_t n, int d, int k, const float* host_points, float* dev_points,
                           float* centroids, int* labels, const mxk_options* options, int* iterations,
                           cudaStream_t stream);
}

namespace {

struct Shard {
    int device = 0;
    int64_t row0 = 0, rows = 0;
    cudaStream_t stream = nullptr;
    float* points = nullptr;
    float* centroids = nullptr;
    int* labels = nullptr;
    void* comm = nullptr;
    int iterations = 0;
    int status = MXK_OK;
    std::string error;

    bool record(int st) {
        if (st == MXK_OK) return true;
        status = st;
        error = mxk_last_error();
        return false;
    }
    bool record_cuda(cudaError_t e, const char* what) {
        if (e == cudaSuccess) return true;
        status = MXK_ERR_CUDA;
        error = std::string(what) + ": " + cudaGetErrorString(e);
        return false;
    }
    void release() {
        if (cudaSetDevice(device) != cudaSuccess) return;
        if (comm && status != MXK_OK) mxk::comm_abort(comm);  // a failed rank's communicator is not destroyed in order
        if (comm) mxk_comm_destroy(comm);
        // (stream-ordered frees into the library's pool, which keeps the blocks
        // mapped for the next call)
        if (points) cudaFreeAsync(points, stream);
        if (centroids) cudaFreeAsync(centroids, stream);
        if (labels) cudaFreeAsync(labels, stream);
        if (stream) {
            cudaStreamSynchronize(stream);
            cudaStreamDestroy(stream);
        }
        comm = nullptr;
        points = centroids = nullptr;
        labels = nullptr;
        stream = nullptr;
    }
};

template <class F>
void on_every_gpu(std::vector<Shard>& shards, F&& body) {
    std::vector<std::thread> threads;
    threads.reserve(shards.size());
    for (auto& s : shards) threads.emplace_back([&body, &s] { body(s); });
    for (auto& t : threads) t.join();
}

}  // namespace

extern "C" int mxk_kmeans_mixed_multi(int64_t n, int d, int k, const float* points, float* centroids, int* labels,
                                      const mxk_options* options, int num_gpus, int* iterations) {
    if (!points || !centroids || !labels || !options || !iterations)
        return mxk::fail(MXK_ERR_INVALID, "kmeans_mixed_multi: null pointer");
    if (n <= 0 || d <= 0 || k <= 0 || num_gpus < 1)
        return mxk::fail(MXK_ERR_INVALID, "kmeans_mixed_multi: require n > 0, d > 0, k > 0 and num_gpus >= 1");
    int visible = 0;
    if (cudaGetDeviceCount(&visible) != cudaSuccess) {
        cudaGetLastError();
        return mxk::fail(MXK_ERR_CUDA, "kmeans_mixed_multi: no CUDA device");
    }
    if (num_gpus > visible) return mxk::fail(MXK_ERR_INVALID, "kmeans_mixed_multi: num_gpus exceeds the visible GPUs");
    int caller_device = 0;
    cudaGetDevice(&caller_device);

    const int G = num_gpus;
    const size_t centroid_bytes = sizeof(float) * size_t(k) * size_t(d);
    std::vector<Shard> shards(static_cast<size_t>(G));
    for (int g = 0; g < G; ++g) {
        Shard& s = shards[size_t(g)];
        s.device = g;
        s.row0 = n / G * g + std::min<int64_t>(g, n % G);
        s.rows = n / G + (g < n % G ? 1 : 0);
    }

    // Phase 1: allocate (from the library's stream-ordered pool on each device,
    // whose blocks stay mapped between calls) and upload the initial centroids.
    on_every_gpu(shards, [&](Shard& s) {
        const size_t rows = size_t(std::max<int64_t>(s.rows, 1));
        if (!s.record_cuda(cudaSetDevice(s.device), "cudaSetDevice") ||
            !s.record_cuda(cudaStreamCreateWithFlags(&s.stream, cudaStreamNonBlocking), "cudaStreamCreate"))
            return;
        cudaMemPool_t pool = mxk::workspace_pool();
        if (!pool) {
            s.record_cuda(cudaErrorMemoryAllocation, "workspace pool");
            return;
        }
        if (!s.record_cuda(cudaMallocFromPoolAsync(reinterpret_cast<void**>(&s.points),
                                                   sizeof(float) * rows * size_t(d), pool, s.stream),
                           "cudaMallocFromPoolAsync") ||
            !s.record_cuda(cudaMallocFromPoolAsync(reinterpret_cast<void**>(&s.centroids), centroid_bytes, pool,
                                                   s.stream),
                           "cudaMallocFromPoolAsync") ||
            !s.record_cuda(cudaMallocFromPoolAsync(reinterpret_cast<void**>(&s.labels), sizeof(int) * rows, pool,
                                                   s.stream),
                           "cudaMallocFromPoolAsync"))
            return;
        // (the shard's points are copied by the Lloyd call itself, overlapping its
        // first iteration)
        if (!s.record_cuda(cudaMemcpyAsync(s.centroids, centroids, centroid_bytes, cudaMemcpyHostToDevice, s.stream),
                           "cudaMemcpyAsync"))
            return;
        s.record_cuda(cudaStreamSynchronize(s.stream), "cudaStreamSynchronize");
    });
    bool uploaded = true;
    for (auto& s : shards) uploaded = uploaded && s.status == MXK_OK;

    // Phase 2 (only when every upload succeeded): communicator, Lloyd, labels.
    unsigned char uid[128] = {};
    if (uploaded && G > 1 && mxk_comm_unique_id(uid) != MXK_OK) {
        shards[0].record(MXK_ERR_COMM);
        uploaded = false;
    }
    std::atomic<int> group_failed{0};
    std::atomic<int> first_failed{-1};  // the rank whose own failure the others then report
    if (uploaded) {
        on_every_gpu(shards, [&](Shard& s) {
            if (!s.record_cuda(cudaSetDevice(s.device), "cudaSetDevice")) return;
            if (G > 1) {
                if (!s.record(mxk_comm_init(&s.comm, G, s.device, uid))) return;
                mxk::comm_attach_group_flag(s.comm, &group_failed);
                if (!s.record(mxk::kmeans_mixed_from_host(s.comm, s.rows, d, k, points + size_t(s.row0) * size_t(d),
                                                          s.points, s.centroids, s.labels, options, &s.iterations,
                                                          s.stream))) {
                    int none = -1;
                    if (!group_failed.load()) first_failed.compare_exchange_strong(none, s.device);
                    group_failed.store(1);  // the other ranks stop waiting for this one
                    return;
                }
            } else if (!s.record(mxk::kmeans_mixed_from_host(nullptr, s.rows, d, k, points, s.points, s.centroids,
                                                             s.labels, options, &s.iterations, s.stream))) {
                return;
            }
            if (!s.record_cuda(cudaMemcpyAsync(labels + s.row0, s.labels, sizeof(int) * size_t(s.rows),
                                               cudaMemcpyDeviceToHost, s.stream),
                               "cudaMemcpyAsync"))
                return;
            s.record_cuda(cudaStreamSynchronize(s.stream), "cudaStreamSynchronize");
        });
    }
    // Every rank finalizes the centroids identically; rank 0's copy is returned.
    Shard& first = shards[0];
    if (uploaded && first.status == MXK_OK)
        if (first.record_cuda(cudaSetDevice(first.device), "cudaSetDevice"))
            first.record_cuda(cudaMemcpy(centroids, first.centroids, centroid_bytes, cudaMemcpyDeviceToHost),
                              "cudaMemcpy");
    for (auto& s : shards) s.release();
    cudaSetDevice(caller_device);
    // the rank that failed first is the cause; the others report their aborted waits
    const int cause = first_failed.load();
    if (cause >= 0 && shards[size_t(cause)].status != MXK_OK)
        return mxk::fail(shards[size_t(cause)].status,
                         "kmeans_mixed_multi: GPU " + std::to_string(cause) + ": " + shards[size_t(cause)].error);
    for (auto& s : shards)
        if (s.status != MXK_OK) return mxk::fail(s.status, "kmeans_mixed_multi: GPU " + std::to_string(s.device) + ": " + s.error);
    *iterations = first.iterations;
    return MXK_OK;
}
