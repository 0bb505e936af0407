// Exposes the reference's own host-side code, compiled from its sources where
// they lie, to the tests.  TEST INFRASTRUCTURE ONLY (built into oracle/_ref/).
//
// include/host_utils.hpp (K-Means++ and farthest-first initialisation, CSV
// reader) and include/precision.hpp (precision rule and distance trackers) of
// ParCIS/MX-KMeans are plain C++; this translation unit includes them from the
// reference checkout (-I <reference>/include) and wraps them in C entry points.
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>
#include "host_utils.hpp"
#include "precision.hpp"

extern "C" int ref_precision_candidate(float p4, float p6, float lc, int d, float gap) {
    return precision_candidate(p4, p6, lc, d, gap);
}
extern "C" int ref_select_precision(float p4, float p6, float lc, float ec, int d, float gap) {
    return select_precision(p4, p6, lc, ec, d, gap);
}
extern "C" void ref_init_kmeanspp(const float* points, int n, int d, int k, uint32_t seed, float* out) {
    std::vector<float> p(points, points + size_t(n) * d);
    const auto c = init_centroids(p, n, d, k, seed);
    std::memcpy(out, c.data(), c.size() * sizeof(float));
}
extern "C" void ref_init_farthest(const float* points, int n, int d, int k, float* out) {
    std::vector<float> p(points, points + size_t(n) * d);
    const auto c = init_centroids_farthest(p, n, d, k);
    std::memcpy(out, c.data(), c.size() * sizeof(float));
}
// Returns 0 and fills out (n*padded_d floats) or 1 when the reader rejects the file.
extern "C" int ref_read_points(const char* path, int n, int d, int padded_d, float* out) {
    try {
        const auto v = read_points(path, n, d, padded_d);
        std::memcpy(out, v.data(), v.size() * sizeof(float));
        return 0;
    } catch (const std::exception&) {
        return 1;
    }
}
// The same, also copying the reader's exception text into msg (cap bytes).
extern "C" int ref_read_points_msg(const char* path, int n, int d, int padded_d, float* out, char* msg, int cap) {
    try {
        const auto v = read_points(path, n, d, padded_d);
        std::memcpy(out, v.data(), v.size() * sizeof(float));
        if (cap > 0) msg[0] = '\0';
        return 0;
    } catch (const std::exception& e) {
        if (cap > 0) {
            std::strncpy(msg, e.what(), size_t(cap) - 1);
            msg[cap - 1] = '\0';
        }
        return 1;
    }
}
// write_labels (host_utils.hpp:69-76); returns 1 when it throws.
extern "C" int ref_write_labels(const char* path, const int* labels, int64_t n) {
    try {
        write_labels(path, std::vector<int>(labels, labels + n));
        return 0;
    } catch (const std::exception&) {
        return 1;
    }
}
