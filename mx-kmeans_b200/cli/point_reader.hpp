// Parallel point input of the mxkmeans CLI: the dense CSV of
// ParCIS/MX-KMeans include/host_utils.hpp:40-67 read on all host threads, and a
// raw float32 fast path for benchmark-sized inputs.
//
// CSV contract (the reference's read_points, kept exactly):
//   * the header is the first line ('\n'-terminated, as std::getline); its
//     cell count (commas + 1; 0 for an empty line) must be d or d + 1;
//   * data lines made only of ' ', '\t', '\r' are skipped and not counted;
//   * every other line must have the header's cell count; its first d cells
//     must parse completely as finite floats under std::stof's rules (leading
//     white space, decimal, hexadecimal, inf/nan spellings; out-of-range values
//     such as denormal results rejected), followed only by ' ', '\t', '\r';
//     a trailing label column is ignored;
//   * errors are reported for the first failing line in file order, with the
//     reference's messages and 1-based data row / column numbers, so a file is
//     rejected with the same text whatever the thread count.
//
// How: the file is mapped (or read, when it is not a regular file), the data
// lines are split into chunks at line boundaries, a first parallel pass counts
// each chunk's non-blank lines, a prefix sum gives each chunk its first row,
// and a second parallel pass parses the chunks straight into their rows of the
// padded output (pads zeroed by the same thread).  Each feature is first
// tried on an exact fast path: a plain decimal with at most 19 significant
// digits and a power of ten within 1e+-22 is formed as one correctly rounded
// double operation (mantissa and power both exact in double), then rounded to
// float; that equals strtof's correctly rounded float unless the double lands
// exactly on a midpoint between two floats, and the fast path also declines
// results outside the float normal range (where strtof reports ERANGE) and
// non-'.' locales.  Everything it declines goes to std::strtof on a
// NUL-terminated copy of the cell with the reference's checks.
//
// Binary (.f32): n x d little-endian IEEE float32 values, row-major, no
// header; the size must be exactly n * d * 4 bytes and every value finite.
#pragma once

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <cfloat>
#include <clocale>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

namespace mxk_cli {

namespace detail {

// The whole input as one byte range: mapped for regular files, read otherwise.
class InputBytes {
public:
    explicit InputBytes(const std::string& path) {
        fd_ = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
        if (fd_ < 0) throw std::runtime_error("Cannot open input: " + path);
        struct stat st {};
        if (::fstat(fd_, &st) == 0 && S_ISREG(st.st_mode)) {
            size_ = size_t(st.st_size);
            if (size_ == 0) return;
            void* p = ::mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
            if (p != MAP_FAILED) {
                map_ = p;
                data_ = static_cast<const char*>(p);
                return;
            }
        }
        // Not mappable (pipe, device, ...): read it to the end.
        size_ = 0;
        char block[1 << 16];
        while (true) {
            const ssize_t got = ::read(fd_, block, sizeof(block));
            if (got == 0) break;
            if (got < 0) {
                if (errno == EINTR) continue;
                read_error_ = true;
                break;
            }
            copy_.insert(copy_.end(), block, block + got);
        }
        size_ = copy_.size();
        data_ = copy_.data();
    }
    ~InputBytes() {
        if (map_) ::munmap(map_, size_);
        if (fd_ >= 0) ::close(fd_);
    }
    InputBytes(const InputBytes&) = delete;
    InputBytes& operator=(const InputBytes&) = delete;

    const char* data() const { return data_; }
    size_t size() const { return size_; }
    bool read_error() const { return read_error_; }

private:
    int fd_ = -1;
    void* map_ = nullptr;
    const char* data_ = nullptr;
    size_t size_ = 0;
    std::vector<char> copy_;
    bool read_error_ = false;
};

inline bool blank_range(const char* a, const char* b) {
    for (; a < b; ++a)
        if (*a != ' ' && *a != '\t' && *a != '\r') return false;
    return true;
}

inline bool trailing_ok(const char* a, const char* b) { return blank_range(a, b); }

// std::stof(cell) followed by the reference's finiteness and trailing-text
// checks (host_utils.hpp:23-29), on the cell [a, b).
inline bool parse_cell_exact(const char* a, const char* b, float* out) {
    char small[64];
    std::string large;
    const size_t len = size_t(b - a);
    const char* text;
    if (len < sizeof(small)) {
        std::memcpy(small, a, len);
        small[len] = '\0';
        text = small;
    } else {
        large.assign(a, len);
        text = large.c_str();
    }
    char* end = nullptr;
    const int saved = errno;
    errno = 0;
    const float v = std::strtof(text, &end);
    const bool range = errno == ERANGE;
    errno = saved;
    if (end == text || range) return false;  // std::stof: invalid_argument / out_of_range
    if (!std::isfinite(v)) return false;
    // find_first_not_of(" \t\r", used) over the whole cell (a NUL inside the
    // cell stops strtof and is then trailing text)
    if (!trailing_ok(a + (end - text), b)) return false;
    *out = v;
    return true;
}

// Exact fast path for plain decimals; false means "decline", not "invalid".
inline bool parse_cell_fast(const char* a, const char* b, float* out) {
    static const double kPow10[23] = {1e0,  1e1,  1e2,  1e3,  1e4,  1e5,  1e6,  1e7,  1e8,  1e9,  1e10, 1e11,
                                      1e12, 1e13, 1e14, 1e15, 1e16, 1e17, 1e18, 1e19, 1e20, 1e21, 1e22};
    const char* p = a;
    while (p < b && (*p == ' ' || *p == '\t')) ++p;
    bool neg = false;
    if (p < b && (*p == '+' || *p == '-')) neg = *p++ == '-';
    uint64_t m = 0;
    int sig = 0, exp10 = 0, digits = 0;
    for (; p < b && unsigned(*p - '0') < 10u; ++p, ++digits) {
        if (m == 0 && *p == '0') continue;
        if (++sig > 19) return false;
        m = m * 10 + unsigned(*p - '0');
    }
    if (p < b && *p == '.') {
        for (++p; p < b && unsigned(*p - '0') < 10u; ++p, ++digits) {
            --exp10;
            if (m == 0 && *p == '0') continue;
            if (++sig > 19) return false;
            m = m * 10 + unsigned(*p - '0');
        }
    }
    if (digits == 0) return false;
    if (p < b && (*p == 'e' || *p == 'E')) {
        ++p;
        bool eneg = false;
        if (p < b && (*p == '+' || *p == '-')) eneg = *p++ == '-';
        if (p >= b || unsigned(*p - '0') >= 10u) return false;
        int e = 0;
        for (; p < b && unsigned(*p - '0') < 10u; ++p) {
            if (e > 100000) return false;
            e = e * 10 + (*p - '0');
        }
        exp10 += eneg ? -e : e;
    }
    if (!trailing_ok(p, b)) return false;
    if (m == 0) {
        *out = neg ? -0.0f : 0.0f;
        return true;
    }
    if (m > (uint64_t(1) << 53) || exp10 < -22 || exp10 > 22) return false;
    const double x = exp10 >= 0 ? double(m) * kPow10[exp10] : double(m) / kPow10[-exp10];
    if (!(x > double(FLT_MIN) && x <= double(FLT_MAX))) return false;
    uint64_t bits;
    std::memcpy(&bits, &x, sizeof(bits));
    if ((bits & ((uint64_t(1) << 29) - 1)) == (uint64_t(1) << 28)) return false;  // on a float midpoint
    const float f = float(x);
    *out = neg ? -f : f;
    return true;
}

inline int reader_threads(int requested) {
    if (requested > 0) return requested;
    const unsigned hw = std::thread::hardware_concurrency();
    return int(std::max(1u, std::min(hw, 64u)));
}

template <class F>
void parallel_for(int count, int threads, F&& body) {
    threads = std::max(1, std::min(threads, count));
    if (threads == 1) {
        for (int i = 0; i < count; ++i) body(i);
        return;
    }
    std::atomic<int> next{0};
    std::vector<std::thread> pool;
    pool.reserve(size_t(threads));
    for (int t = 0; t < threads; ++t)
        pool.emplace_back([&] {
            for (int i; (i = next.fetch_add(1)) < count;) body(i);
        });
    for (auto& th : pool) th.join();
}

}  // namespace detail

// The reference's read_points into out[n * padded_d] (every element written).
// threads <= 0: all hardware threads; chunk_bytes <= 0: an automatic chunk size
// (a test hook: tiny chunks put line boundaries everywhere).
inline void read_points_into(const std::string& path, int64_t n, int d, int padded_d, float* out,
                             int threads = 0, int64_t chunk_bytes = 0) {
    using namespace detail;
    InputBytes in(path);
    const char* data = in.data();
    const size_t size = in.size();
    if (size == 0) throw std::runtime_error("Input is empty");
    const char* header_end = static_cast<const char*>(std::memchr(data, '\n', size));
    if (!header_end) header_end = data + size;
    const size_t columns =
        header_end == data ? 0 : size_t(std::count(data, header_end, ',')) + 1;
    if (columns != size_t(d) && columns != size_t(d) + 1)
        throw std::runtime_error("CSV header must contain d features and optionally one label column");

    const char* body = header_end < data + size ? header_end + 1 : data + size;
    const char* stop = data + size;
    const size_t body_size = size_t(stop - body);
    threads = reader_threads(threads);
    size_t chunk = chunk_bytes > 0 ? size_t(chunk_bytes) : std::max<size_t>(size_t(1) << 20, body_size / (size_t(threads) * 8) + 1);
    const size_t nchunks_max = body_size / chunk + 1;
    // Chunk c holds the lines that start in [start[c], start[c + 1]).
    std::vector<const char*> start;
    start.reserve(nchunks_max + 1);
    start.push_back(body);
    for (size_t c = 1; c < nchunks_max; ++c) {
        const char* at = body + c * chunk;
        if (at <= start.back()) continue;
        const char* nl = static_cast<const char*>(std::memchr(at - 1, '\n', size_t(stop - (at - 1))));
        const char* s = nl ? nl + 1 : stop;
        if (s > start.back() && s < stop) start.push_back(s);
    }
    start.push_back(stop);
    const int nchunks = int(start.size() - 1);
    const bool c_locale = std::strcmp(std::localeconv()->decimal_point, ".") == 0;

    // Pass 1: non-blank lines per chunk.
    std::vector<int64_t> rows_in(size_t(nchunks), 0);
    parallel_for(nchunks, threads, [&](int c) {
        int64_t count = 0;
        for (const char* p = start[size_t(c)]; p < start[size_t(c) + 1];) {
            const char* e = static_cast<const char*>(std::memchr(p, '\n', size_t(stop - p)));
            if (!e) e = stop;
            if (!blank_range(p, e)) ++count;
            p = e + 1;
        }
        rows_in[size_t(c)] = count;
    });
    std::vector<int64_t> first_row(size_t(nchunks) + 1, 0);
    for (int c = 0; c < nchunks; ++c) first_row[size_t(c) + 1] = first_row[size_t(c)] + rows_in[size_t(c)];

    // Pass 2: parse each chunk into its rows; a chunk stops at its first error.
    std::vector<std::string> failure(static_cast<size_t>(nchunks));
    std::atomic<int> first_bad{nchunks};
    parallel_for(nchunks, threads, [&](int c) {
        if (c > first_bad.load(std::memory_order_relaxed)) return;  // a line before this chunk already failed
        int64_t row = first_row[size_t(c)];
        std::string& err = failure[size_t(c)];
        for (const char* p = start[size_t(c)]; p < start[size_t(c) + 1];) {
            const char* e = static_cast<const char*>(std::memchr(p, '\n', size_t(stop - p)));
            if (!e) e = stop;
            const char* line = p;
            p = e + 1;
            if (blank_range(line, e)) continue;
            if (row >= n) {
                err = "CSV contains more rows than --n-samples";
                break;
            }
            if (size_t(std::count(line, e, ',')) + 1 != columns) {
                err = "Wrong column count at data row " + std::to_string(row + 1);
                break;
            }
            float* dst = out + size_t(row) * size_t(padded_d);
            const char* cell = line;
            for (int j = 0; j < d; ++j) {
                const char* comma = static_cast<const char*>(std::memchr(cell, ',', size_t(e - cell)));
                const char* cell_end = comma ? comma : e;
                float v;
                if (!((c_locale && parse_cell_fast(cell, cell_end, &v)) || parse_cell_exact(cell, cell_end, &v))) {
                    err = "Invalid feature at data row " + std::to_string(row + 1) + ", column " + std::to_string(j + 1);
                    break;
                }
                dst[j] = v;
                cell = cell_end + 1;
            }
            if (!err.empty()) break;
            std::fill(dst + d, dst + padded_d, 0.0f);
            ++row;
        }
        if (!err.empty()) {
            int cur = first_bad.load();
            while (c < cur && !first_bad.compare_exchange_weak(cur, c)) {
            }
        }
    });
    for (int c = 0; c < nchunks; ++c)
        if (!failure[size_t(c)].empty()) throw std::runtime_error(failure[size_t(c)]);
    // (as the reference: lines read before a read error are checked first)
    if (in.read_error()) throw std::runtime_error("Error while reading input: " + path);
    if (first_row[size_t(nchunks)] != n) throw std::runtime_error("CSV row count does not match --n-samples");
}

// Raw little-endian float32 rows (n x d, no header) into out[n * padded_d].
inline void read_points_f32_into(const std::string& path, int64_t n, int d, int padded_d, float* out,
                                 int threads = 0) {
    using namespace detail;
    const int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd < 0) throw std::runtime_error("Cannot open input: " + path);
    struct stat st {};
    const bool sized = ::fstat(fd, &st) == 0 && S_ISREG(st.st_mode);
    const uint64_t want = uint64_t(n) * uint64_t(d) * sizeof(float);
    if (!sized || uint64_t(st.st_size) != want) {
        ::close(fd);
        throw std::runtime_error("Binary input must hold exactly n * d float32 values (" + std::to_string(want) +
                                 " bytes): " + path);
    }
    threads = reader_threads(threads);
    const int64_t block_rows = std::max<int64_t>(1, (int64_t(1) << 22) / (int64_t(d) * 4));  // ~4 MB per read
    const int blocks = int((n + block_rows - 1) / block_rows);
    std::vector<std::string> failure(static_cast<size_t>(blocks));
    std::atomic<int> first_bad{blocks};
    parallel_for(blocks, threads, [&](int b) {
        if (b > first_bad.load(std::memory_order_relaxed)) return;
        const int64_t r0 = int64_t(b) * block_rows, r1 = std::min(n, r0 + block_rows);
        std::vector<float> staging;
        float* dst = out + size_t(r0) * size_t(padded_d);
        float* buf = dst;
        if (padded_d != d) {
            staging.resize(size_t(r1 - r0) * size_t(d));
            buf = staging.data();
        }
        size_t left = size_t(r1 - r0) * size_t(d) * sizeof(float);
        off_t off = off_t(uint64_t(r0) * uint64_t(d) * sizeof(float));
        char* to = reinterpret_cast<char*>(buf);
        while (left) {
            const ssize_t got = ::pread(fd, to, left, off);
            if (got < 0 && errno == EINTR) continue;
            if (got <= 0) {
                failure[size_t(b)] = "Error while reading input: " + path;
                break;
            }
            left -= size_t(got);
            off += got;
            to += got;
        }
        if (failure[size_t(b)].empty()) {
            for (int64_t r = r0; r < r1 && failure[size_t(b)].empty(); ++r) {
                const float* src = buf + size_t(r - r0) * size_t(d);
                float* row = dst + size_t(r - r0) * size_t(padded_d);
                for (int j = 0; j < d; ++j)
                    if (!std::isfinite(src[j])) {
                        failure[size_t(b)] =
                            "Invalid feature at data row " + std::to_string(r + 1) + ", column " + std::to_string(j + 1);
                        break;
                    }
                if (padded_d != d) {
                    std::copy(src, src + d, row);
                    std::fill(row + d, row + padded_d, 0.0f);
                }
            }
        }
        if (!failure[size_t(b)].empty()) {
            int cur = first_bad.load();
            while (b < cur && !first_bad.compare_exchange_weak(cur, b)) {
            }
        }
    });
    ::close(fd);
    for (int b = 0; b < blocks; ++b)
        if (!failure[size_t(b)].empty()) throw std::runtime_error(failure[size_t(b)]);
}

inline bool is_f32_path(const std::string& path) {
    return path.size() > 4 && path.compare(path.size() - 4, 4, ".f32") == 0;
}

}  // namespace mxk_cli
