// Host-side input/output and centroid initialisation of the mxkmeans CLI.
//
// Interface-compatible with ParCIS/MX-KMeans include/host_utils.hpp:1-141:
//   * CSV input (read on all host threads, same accept/reject rules and
//     messages): point_reader.hpp;
//   * labels: "clusters" header, one label per line (formatted on all host
//     threads, same bytes).
//   * K-Means++ (D^2 sampling with std::mt19937(seed), the first index from
//     uniform_int_distribution<int>(0, n-1), each next index by a
//     uniform_real_distribution<double>(0, total) draw against the running sum of
//     double squared distances) and farthest-first (from row 0, float distances,
//     first maximum).  The draw sequence and the distance arithmetic are kept as
//     in the reference so a seed selects the same centroids; the per-point
//     distances run on all host threads, the running sum, the draws and the
//     scans stay sequential.
#pragma once

#include <algorithm>
#include <charconv>
#include <cmath>
#include <cstdint>
#include <fstream>
#include <limits>
#include <random>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "point_reader.hpp"

namespace mxk_cli {

inline float parse_float(const std::string& text) {
    size_t used = 0;
    const float v = std::stof(text, &used);
    if (!std::isfinite(v) || text.find_first_not_of(" \t\r", used) != std::string::npos)
        throw std::invalid_argument("Invalid finite number: " + text);
    return v;
}

inline int parse_int(const std::string& text) {
    size_t used = 0;
    const int v = std::stoi(text, &used);
    if (used != text.size()) throw std::invalid_argument("Invalid integer: " + text);
    return v;
}

// The reference's label file (host_utils.hpp:69-76): "clusters", then one
// decimal label per line.  The text is formatted on all host threads in blocks
// (std::to_chars, the same digits as operator<<) and written in order, so the
// bytes are those of the reference's ofstream loop.
inline void write_labels(const std::string& path, const int* labels, int64_t n, int threads = 0) {
    std::ofstream out(path);
    if (!out) throw std::runtime_error("Cannot open output: " + path);
    out << "clusters\n";
    constexpr int64_t kBlock = int64_t(1) << 20;
    const int64_t blocks = (n + kBlock - 1) / kBlock;
    threads = detail::reader_threads(threads);
    // format a window of blocks in parallel, then write it, to bound memory
    const int64_t window = std::max<int64_t>(1, threads) * 2;
    std::vector<std::string> text(size_t(std::min(blocks, window)));
    for (int64_t b0 = 0; b0 < blocks && out; b0 += window) {
        const int64_t nb = std::min(window, blocks - b0);
        detail::parallel_for(int(nb), threads, [&](int i) {
            const int64_t r0 = (b0 + i) * kBlock, r1 = std::min(n, r0 + kBlock);
            std::string& t = text[size_t(i)];
            t.resize(size_t(r1 - r0) * 12);
            char* p = t.data();
            for (int64_t r = r0; r < r1; ++r) {
                p = std::to_chars(p, p + 11, labels[r]).ptr;
                *p++ = '\n';
            }
            t.resize(size_t(p - t.data()));
        });
        for (int64_t i = 0; i < nb && out; ++i) out.write(text[size_t(i)].data(), std::streamsize(text[size_t(i)].size()));
    }
    out.close();
    if (!out) throw std::runtime_error("Failed to write output: " + path);
}

inline void write_labels(const std::string& path, const std::vector<int>& labels) {
    write_labels(path, labels.data(), int64_t(labels.size()));
}

// Squared distance of row p to a center, accumulated in double.
inline double sq_dist_double(const float* row, const float* center, int d) {
    double s = 0.0;
    for (int j = 0; j < d; ++j) {
        const double diff = double(row[j]) - center[j];
        s += diff * diff;
    }
    return s;
}

// body(p0, p1) over contiguous point ranges on all host threads when the pass
// is large enough to pay for them.  Each point's value is computed by one
// thread with the sequential arithmetic, so results do not depend on the split.
template <class F>
void for_point_blocks(int64_t n, int d, F&& body) {
    const int threads = detail::reader_threads(0);
    if (threads <= 1 || n * int64_t(d) < (int64_t(1) << 20)) {
        body(int64_t(0), n);
        return;
    }
    const int blocks = threads * 4;
    const int64_t per = (n + blocks - 1) / blocks;
    detail::parallel_for(blocks, threads, [&](int b) {
        const int64_t p0 = std::min(n, int64_t(b) * per), p1 = std::min(n, p0 + per);
        if (p0 < p1) body(p0, p1);
    });
}

inline std::vector<float> init_kmeanspp(const std::vector<float>& points, int64_t n, int d, int k, uint32_t seed) {
    std::mt19937 rng(seed);
    std::vector<float> centers(size_t(k) * d);
    std::vector<double> dist(size_t(n), std::numeric_limits<double>::infinity());
    std::vector<char> chosen(size_t(n), 0);
    int64_t pick = std::uniform_int_distribution<int>(0, int(n - 1))(rng);
    for (int c = 0; c < k; ++c) {
        const float* src = points.data() + size_t(pick) * d;
        std::copy(src, src + d, centers.begin() + size_t(c) * d);
        chosen[pick] = 1;
        const float* center = centers.data() + size_t(c) * d;
        for_point_blocks(n, d, [&](int64_t p0, int64_t p1) {
            for (int64_t p = p0; p < p1; ++p) {
                const double v = sq_dist_double(points.data() + size_t(p) * d, center, d);
                dist[p] = chosen[p] ? 0.0 : std::min(dist[p], v);
            }
        });
        double total = 0.0;  // in point order, as the reference accumulates it
        for (int64_t p = 0; p < n; ++p) total += dist[p];
        if (c + 1 == k) break;
        pick = -1;
        if (total > 0.0) {
            const double target = std::uniform_real_distribution<double>(0.0, total)(rng);
            double run = 0.0;
            for (int64_t p = 0; p < n; ++p) {
                run += dist[p];
                if (!chosen[p] && dist[p] > 0.0 && run > target) {
                    pick = p;
                    break;
                }
            }
        }
        if (pick < 0) {  // all remaining rows duplicate a center, or rounding at the end of the sum
            for (int64_t p = 0; p < n; ++p)
                if (!chosen[p]) {
                    pick = p;
                    break;
                }
        }
    }
    return centers;
}

inline std::vector<float> init_farthest(const std::vector<float>& points, int64_t n, int d, int k) {
    std::vector<float> centers(size_t(k) * d);
    std::vector<float> dist(size_t(n), std::numeric_limits<float>::max());
    int64_t pick = 0;
    for (int c = 0; c < k; ++c) {
        const float* src = points.data() + size_t(pick) * d;
        std::copy(src, src + d, centers.begin() + size_t(c) * d);
        for_point_blocks(n, d, [&](int64_t p0, int64_t p1) {
            for (int64_t p = p0; p < p1; ++p) {
                const float* row = points.data() + size_t(p) * d;
                float s = 0.0f;
                for (int j = 0; j < d; ++j) {
                    const float diff = row[j] - src[j];
                    s += diff * diff;
                }
                dist[p] = std::min(dist[p], s);
            }
        });
        dist[pick] = -1.0f;
        pick = std::max_element(dist.begin(), dist.end()) - dist.begin();
    }
    return centers;
}

}  // namespace mxk_cli
