// CUDA error checking and an owning device buffer for C++ callers of the
// drop-in API (same names and behaviour as ParCIS/MX-KMeans
// include/cuda_utils.cuh:1-30: CUDA_CHECK throws std::runtime_error; a
// DeviceBuffer frees its allocation on scope exit and clear() zeroes it).
#pragma once

#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

inline void check_cuda(cudaError_t status, const char* operation) {
    if (status != cudaSuccess) throw std::runtime_error(std::string(operation) + ": " + cudaGetErrorString(status));
}
#define CUDA_CHECK(call) check_cuda((call), #call)

template <typename T>
class DeviceBuffer {
public:
    explicit DeviceBuffer(size_t count) : count_(count) {
        if (count) CUDA_CHECK(cudaMalloc(reinterpret_cast<void**>(&data_), count * sizeof(T)));
    }
    ~DeviceBuffer() {
        if (data_) cudaFree(data_);
    }
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
    T* get() const { return data_; }
    size_t size() const { return count_; }
    void clear() {
        if (count_) CUDA_CHECK(cudaMemset(data_, 0, count_ * sizeof(T)));
    }

private:
    T* data_ = nullptr;
    size_t count_;
};
