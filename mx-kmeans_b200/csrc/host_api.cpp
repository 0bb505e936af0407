// C entry points for the host-side pieces of the CLI (CSV reader and centroid
// initialisation), so embedding programs and tests can use them without the
// executable.  Mirrors ParCIS/MX-KMeans include/host_utils.hpp:40-141; the CSV
// reader runs on all host threads (point_reader.hpp).
#include <cstring>
#include <exception>
#include <string>
#include <vector>

#include "host_io.hpp"
#include "mxk.h"

namespace mxk {
int fail(int status, const std::string& message);
}

extern "C" {

int mxk_host_init_kmeanspp(const float* points, int64_t n, int d, int k, uint32_t seed, float* out) {
    if (!points || !out || n <= 0 || d <= 0 || k <= 0) return mxk::fail(MXK_ERR_INVALID, "init: bad arguments");
    try {
        const std::vector<float> p(points, points + size_t(n) * d);
        const auto c = mxk_cli::init_kmeanspp(p, n, d, k, seed);
        std::memcpy(out, c.data(), c.size() * sizeof(float));
        return MXK_OK;
    } catch (const std::exception& e) {
        return mxk::fail(MXK_ERR_INVALID, e.what());
    }
}

int mxk_host_init_farthest(const float* points, int64_t n, int d, int k, float* out) {
    if (!points || !out || n <= 0 || d <= 0 || k <= 0) return mxk::fail(MXK_ERR_INVALID, "init: bad arguments");
    try {
        const std::vector<float> p(points, points + size_t(n) * d);
        const auto c = mxk_cli::init_farthest(p, n, d, k);
        std::memcpy(out, c.data(), c.size() * sizeof(float));
        return MXK_OK;
    } catch (const std::exception& e) {
        return mxk::fail(MXK_ERR_INVALID, e.what());
    }
}

int mxk_host_read_points(const char* path, int64_t n, int d, int padded_d, float* out) {
    return mxk_host_read_points_ex(path, n, d, padded_d, 0, 0, out);
}

int mxk_host_read_points_ex(const char* path, int64_t n, int d, int padded_d, int threads, int64_t chunk_bytes,
                            float* out) {
    if (!path || !out || n <= 0 || d <= 0 || padded_d < d) return mxk::fail(MXK_ERR_INVALID, "read_points: bad arguments");
    try {
        mxk_cli::read_points_into(path, n, d, padded_d, out, threads, chunk_bytes);
        return MXK_OK;
    } catch (const std::exception& e) {
        return mxk::fail(MXK_ERR_INVALID, e.what());
    }
}

int mxk_host_read_points_f32(const char* path, int64_t n, int d, int padded_d, float* out) {
    if (!path || !out || n <= 0 || d <= 0 || padded_d < d)
        return mxk::fail(MXK_ERR_INVALID, "read_points_f32: bad arguments");
    try {
        mxk_cli::read_points_f32_into(path, n, d, padded_d, out);
        return MXK_OK;
    } catch (const std::exception& e) {
        return mxk::fail(MXK_ERR_INVALID, e.what());
    }
}

int mxk_host_write_labels(const char* path, const int* labels, int64_t n) {
    if (!path || (!labels && n > 0)) return mxk::fail(MXK_ERR_INVALID, "write_labels: bad arguments");
    try {
        mxk_cli::write_labels(path, labels, n);
        return MXK_OK;
    } catch (const std::exception& e) {
        return mxk::fail(MXK_ERR_INVALID, e.what());
    }
}

}  // extern "C"
