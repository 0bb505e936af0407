// mxkmeans: command-line driver of the B200 MX-KMeans library.
//
// Options, validation, CSV input, label output and the stdout timing record
// follow ParCIS/MX-KMeans src/main.cu:1-134.  Changes: the device check asks for
// compute capability 10.x (B200), the 32-bit index limits on N*D and N*K are
// lifted (the library indexes in 64 bits and never builds an N x K buffer), the
// CSV is parsed on all host threads (same rules and messages), an input path
// ending in .f32 is read as raw float32 rows, and --gpus N row-shards the
// points over N GPUs of this node (one host thread per
// GPU, NCCL allreduce of the per-cluster sums and counts each iteration).
#include <cuda_runtime.h>
#include <getopt.h>

#include <chrono>
#include <cstdio>
#include <filesystem>
#include <iostream>
#include <memory>
#include <string>
#include <thread>
#include <vector>

#include "host_io.hpp"
#include "mxk.h"

namespace {

struct Arguments {
    int64_t n = 0;
    int d = 0, k = 0, runs = 1, warmup = 0, seed = 42, gpus = 1;
    std::string input, output = "labels.csv";
    std::string initialization = "kmeans++";
    mxk_options algorithm{300, 0, 1e-4f, 0};
};

void usage() {
    std::cout << R"(Usage: mxkmeans -n N -d D -k K -i points.csv [options]

Required:
  -n, --n-samples N       Number of input rows
  -d, --dimensions D      Number of feature columns (padded internally to 128)
  -k, --clusters K        Cluster count, at least 4 and a multiple of 4
  -i, --input-file PATH   Dense CSV with a header; optional final label column
                          (a .f32 file: raw little-endian float32, N x D rows)

Options:
  -o, --out-filename PATH Label CSV (default: labels.csv)
  -m, --maxiter N         Maximum Lloyd iterations (default: 300)
  -t, --tol FLOAT         Sum of squared centroid shifts (default: 1e-4)
  -s, --seed N            K-Means++ seed (default: 42)
      --init METHOD      kmeans++ or farthest (default: kmeans++)
  -r, --runs N            Measured repetitions from the same centers (default: 1)
      --warmup N         Unmeasured complete runs (default: 0)
      --fp32-iters N     Initial FP32 Lloyd iterations in each run (default: 0)
      --gpus N           Row-shard the points over N GPUs of this node (default: 1)
      --verbose          Print per-iteration precision counts to stderr
  -h, --help             Show this help

Stdout: CSV with n_samples,dimensions,clusters,mean_seconds,iterations.
Timing includes device workspaces and clustering, excluding CSV I/O,
K-Means++ initialization and the initial host-to-device data transfer.
)";
}

Arguments parse(int argc, char** argv) {
    Arguments a;
    const option options[] = {{"n-samples", required_argument, nullptr, 'n'},
                              {"dimensions", required_argument, nullptr, 'd'},
                              {"clusters", required_argument, nullptr, 'k'},
                              {"input-file", required_argument, nullptr, 'i'},
                              {"out-filename", required_argument, nullptr, 'o'},
                              {"maxiter", required_argument, nullptr, 'm'},
                              {"tol", required_argument, nullptr, 't'},
                              {"seed", required_argument, nullptr, 's'},
                              {"runs", required_argument, nullptr, 'r'},
                              {"warmup", required_argument, nullptr, 1000},
                              {"fp32-iters", required_argument, nullptr, 1001},
                              {"verbose", no_argument, nullptr, 1002},
                              {"init", required_argument, nullptr, 1003},
                              {"gpus", required_argument, nullptr, 1004},
                              {"help", no_argument, nullptr, 'h'},
                              {nullptr, 0, nullptr, 0}};
    int opt;
    while ((opt = getopt_long(argc, argv, "n:d:k:i:o:m:t:s:r:h", options, nullptr)) != -1) {
        switch (opt) {
            case 'n': a.n = mxk_cli::parse_int(optarg); break;
            case 'd': a.d = mxk_cli::parse_int(optarg); break;
            case 'k': a.k = mxk_cli::parse_int(optarg); break;
            case 'i': a.input = optarg; break;
            case 'o': a.output = optarg; break;
            case 'm': a.algorithm.max_iterations = mxk_cli::parse_int(optarg); break;
            case 't': a.algorithm.tolerance = mxk_cli::parse_float(optarg); break;
            case 's': a.seed = mxk_cli::parse_int(optarg); break;
            case 'r': a.runs = mxk_cli::parse_int(optarg); break;
            case 1000: a.warmup = mxk_cli::parse_int(optarg); break;
            case 1001: a.algorithm.fp32_iterations = mxk_cli::parse_int(optarg); break;
            case 1002: a.algorithm.verbose = 1; break;
            case 1003: a.initialization = optarg; break;
            case 1004: a.gpus = mxk_cli::parse_int(optarg); break;
            case 'h': usage(); std::exit(0);
            default: throw std::invalid_argument("Invalid option; use --help");
        }
    }
    if (optind != argc) throw std::invalid_argument("Unexpected positional argument");
    if (a.initialization != "kmeans++" && a.initialization != "farthest")
        throw std::invalid_argument("--init must be kmeans++ or farthest");
    if (a.n <= 0 || a.d <= 0 || a.k < 4 || a.k > a.n || a.k % 4)
        throw std::invalid_argument("Require N > 0, D > 0, 4 <= K <= N, and K divisible by 4");
    if (a.d > INT32_MAX - 127) throw std::invalid_argument("Too many dimensions");
    if (a.runs <= 0 || a.warmup < 0 || a.seed < 0 || int64_t(a.runs) + a.warmup > INT32_MAX)
        throw std::invalid_argument("Require runs > 0, warmup >= 0, seed >= 0, and runs + warmup <= INT_MAX");
    if (a.algorithm.max_iterations <= 0 || a.algorithm.fp32_iterations < 0 || a.algorithm.tolerance < 0)
        throw std::invalid_argument("Require maxiter > 0, fp32-iters >= 0, and tol >= 0");
    if (a.gpus < 1) throw std::invalid_argument("Require --gpus >= 1");
    if (a.input.empty() || a.output.empty()) throw std::invalid_argument("Input and output paths are required");
    if (a.input == a.output || (std::filesystem::exists(a.input) && std::filesystem::exists(a.output) &&
                                std::filesystem::equivalent(a.input, a.output)))
        throw std::invalid_argument("Input and output paths must differ");
    return a;
}

void check(int status) {
    if (status != MXK_OK) throw std::runtime_error(mxk_last_error());
}
void check_cuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// One GPU's shard: rows [row0, row0 + rows) of the padded host matrix.
struct Shard {
    int device = 0;
    int64_t row0 = 0, rows = 0;
    float* points = nullptr;
    float* centroids = nullptr;
    int* labels = nullptr;
    cudaStream_t stream = nullptr;
    void* comm = nullptr;
    int iterations = 0;
    double seconds = 0.0;
    std::string error;
};

}  // namespace

int main(int argc, char** argv) {
    try {
        const Arguments args = parse(argc, argv);
        const int d = (args.d + 127) / 128 * 128;
        int ndev = 0;
        check_cuda(cudaGetDeviceCount(&ndev), "cudaGetDeviceCount");
        if (args.gpus > ndev) throw std::runtime_error("--gpus exceeds the number of visible GPUs");
        for (int g = 0; g < args.gpus; ++g) {
            cudaDeviceProp prop{};
            check_cuda(cudaGetDeviceProperties(&prop, g), "cudaGetDeviceProperties");
            if (prop.major != 10)
                throw std::runtime_error("This build requires an sm_100 Blackwell data-center GPU, such as B200");
        }
        // Every element is written by the reader (features, then zero pads), so
        // the buffer is left uninitialised and first touched by the reader's threads.
        const size_t point_floats = size_t(args.n) * size_t(d);
        std::unique_ptr<float[]> point_buffer(new float[point_floats]);
        if (mxk_cli::is_f32_path(args.input))
            mxk_cli::read_points_f32_into(args.input, args.n, args.d, d, point_buffer.get());
        else
            mxk_cli::read_points_into(args.input, args.n, args.d, d, point_buffer.get());
        const float* points = point_buffer.get();
        // Initial centroids on GPU 0 (mxk_init_*: the same rows as the reference's
        // host_utils.hpp functions pick, at GPU speed).
        std::vector<float> initial(size_t(args.k) * d);
        {
            check_cuda(cudaSetDevice(0), "cudaSetDevice");
            float *dev_points = nullptr, *dev_centroids = nullptr;
            check_cuda(cudaMalloc(&dev_points, sizeof(float) * point_floats), "cudaMalloc");
            check_cuda(cudaMalloc(&dev_centroids, sizeof(float) * initial.size()), "cudaMalloc");
            check_cuda(cudaMemcpy(dev_points, points, sizeof(float) * point_floats, cudaMemcpyHostToDevice),
                       "cudaMemcpy");
            const int st = args.initialization == "farthest"
                               ? mxk_init_farthest(args.n, d, args.k, dev_points, dev_centroids, nullptr)
                               : mxk_init_kmeanspp(args.n, d, args.k, dev_points, dev_centroids,
                                                   uint32_t(args.seed), nullptr);
            if (st == MXK_OK)
                check_cuda(cudaMemcpy(initial.data(), dev_centroids, sizeof(float) * initial.size(),
                                      cudaMemcpyDeviceToHost),
                           "cudaMemcpy");
            cudaFree(dev_points);
            cudaFree(dev_centroids);
            check(st);
        }
        const int G = args.gpus;
        std::vector<Shard> shards(G);
        unsigned char uid[128] = {};
        if (G > 1) check(mxk_comm_unique_id(uid));
        for (int g = 0; g < G; ++g) {
            shards[g].device = g;
            shards[g].row0 = args.n / G * g + std::min<int64_t>(g, args.n % G);
            shards[g].rows = args.n / G + (g < args.n % G ? 1 : 0);
        }
        std::vector<std::thread> threads;
        for (int g = 0; g < G; ++g) {
            threads.emplace_back([&, g] {
                Shard& s = shards[g];
                try {
                    check_cuda(cudaSetDevice(s.device), "cudaSetDevice");
                    check_cuda(cudaStreamCreateWithFlags(&s.stream, cudaStreamNonBlocking), "cudaStreamCreate");
                    check_cuda(cudaMalloc(&s.points, sizeof(float) * size_t(std::max<int64_t>(s.rows, 1)) * d), "cudaMalloc");
                    check_cuda(cudaMalloc(&s.centroids, sizeof(float) * initial.size()), "cudaMalloc");
                    check_cuda(cudaMalloc(&s.labels, sizeof(int) * size_t(std::max<int64_t>(s.rows, 1))), "cudaMalloc");
                    check_cuda(cudaMemcpy(s.points, points + size_t(s.row0) * d, sizeof(float) * size_t(s.rows) * d,
                                          cudaMemcpyHostToDevice),
                               "cudaMemcpy");
                    if (G > 1) check(mxk_comm_init(&s.comm, G, g, uid));
                    mxk_options opts = args.algorithm;
                    if (g != 0) opts.verbose = 0;
                    for (int run = 0; run < args.warmup + args.runs; ++run) {
                        check_cuda(cudaMemcpy(s.centroids, initial.data(), sizeof(float) * initial.size(),
                                              cudaMemcpyHostToDevice),
                                   "cudaMemcpy");
                        check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
                        const auto t0 = std::chrono::steady_clock::now();
                        if (G > 1)
                            check(mxk_kmeans_mixed_sharded(s.comm, s.rows, d, args.k, s.points, s.centroids, s.labels,
                                                           &opts, &s.iterations, s.stream));
                        else
                            check(mxk_kmeans_mixed(s.rows, d, args.k, s.points, s.centroids, s.labels, &opts,
                                                   &s.iterations, s.stream));
                        check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
                        const auto t1 = std::chrono::steady_clock::now();
                        if (run >= args.warmup) s.seconds += std::chrono::duration<double>(t1 - t0).count();
                    }
                } catch (const std::exception& e) {
                    s.error = e.what();
                }
            });
        }
        for (auto& t : threads) t.join();
        for (auto& s : shards)
            if (!s.error.empty()) throw std::runtime_error(s.error);
        std::vector<int> labels(size_t(args.n));
        double seconds = 0.0;
        for (auto& s : shards) {
            check_cuda(cudaSetDevice(s.device), "cudaSetDevice");
            check_cuda(cudaMemcpy(labels.data() + s.row0, s.labels, sizeof(int) * size_t(s.rows), cudaMemcpyDeviceToHost),
                       "cudaMemcpy");
            seconds = std::max(seconds, s.seconds);
            if (s.comm) mxk_comm_destroy(s.comm);
            cudaFree(s.points);
            cudaFree(s.centroids);
            cudaFree(s.labels);
            cudaStreamDestroy(s.stream);
        }
        mxk_cli::write_labels(args.output, labels);
        std::cout << "n_samples,dimensions,clusters,mean_seconds,iterations\n"
                  << args.n << ',' << args.d << ',' << args.k << ',' << seconds / args.runs << ','
                  << shards[0].iterations << '\n';
    } catch (const std::exception& error) {
        std::cerr << "mxkmeans: " << error.what() << '\n';
        return 1;
    }
    return 0;
}
