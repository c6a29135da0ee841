// optimize: command-line CAGRA sort + optimize of a bucket2 kNN graph, with the reference
// tool's options, outputs and exit codes (bucketDemo/buildBucket/src/optimize.cu:215 main):
//
//   optimize -i data.u8bin -g vector_knn.bin -o cagra_graph.bin --output-degree 32 [--skip-sort] [--save-npy]
//
// Steps: read the dataset and the int32 kNN graph, sanitize (-1 / self -> first valid
// neighbour, else (i+1)%N), sort every row by exact L2 unless --skip-sort, rank-based
// detour prune + reverse edges to K, write the uint32 graph (int64 N, int32 K header) and,
// with --save-npy, an int64 .npy beside it.
// Exit status: 0 ok; 2 when the job does not fit the GPU (the free-memory check with
// --gpu-fit-margin, an out-of-memory status from the library, or --force-chunked: the
// reference's signal to fall back to its chunked path); 1 on any other error.
#include <chrono>
#include <cstdio>
#include <filesystem>
#include <string>
#include <vector>

#include "args.hpp"
#include "gta.h"

namespace {

using Clock = std::chrono::steady_clock;

double secs(Clock::time_point t0) { return std::chrono::duration<double>(Clock::now() - t0).count(); }

struct DoesNotFit : std::runtime_error {
    using std::runtime_error::runtime_error;
};

void check(int rc, const char* what)
{
    if (rc == GTA_ENOMEM) throw DoesNotFit(std::string(what) + ": " + gta_last_error());
    if (rc != GTA_OK) throw std::runtime_error(std::string(what) + ": " + gta_last_error());
}

int run(int argc, char** argv)
{
    const std::vector<cli::Opt> opts = {
        {"input", 'i', false, "Original dataset (.fbin/.bin/.u8bin/.i8bin), needed by the L2 sort", ""},
        {"knn-graph", 'g', false, "Input vector_knn.bin (intermediate kNN graph)", ""},
        {"output", 'o', false, "Output CAGRA graph .bin", ""},
        {"output-degree", 0, false, "Target output graph degree K_out (<= input M)", "32"},
        {"skip-sort", 0, true, "Skip the L2 sort (input rows already ascending)", ""},
        {"save-npy", 0, true, "Also write an int64 .npy beside the .bin", ""},
        {"force-chunked", 0, true, "Refuse (exit 2) so that a driver takes its chunked path", ""},
        {"gpu-fit-margin", 0, false, "Multiplier on dataset+graph+output bytes vs free GPU memory", "3.0"},
    };
    cli::Args a("optimize (gta-b200)", opts);
    if (!a.parse(argc, argv)) return 0;
    const std::string input = a.required("input");
    const std::string knn_path = a.required("knn-graph");
    const std::string out_path = a.required("output");
    const int K = static_cast<int>(a.i64("output-degree", 32));
    const bool skip_sort = a.flag("skip-sort");
    const double margin = a.f64("gpu-fit-margin", 3.0);
    if (K <= 0) throw std::runtime_error("--output-degree must be > 0");

    const auto t_all = Clock::now();
    int64_t N = 0, Ng = 0;
    int32_t d = 0, dtype = 0, M = 0;
    check(gta_read_dataset_header(input.c_str(), &N, &d, &dtype), "read dataset header");
    check(gta_read_knn_header(knn_path.c_str(), &Ng, &M), "read kNN header");
    if (Ng != N)
        throw std::runtime_error("KNN graph N (" + std::to_string(Ng) + ") != dataset N (" + std::to_string(N) + ")");
    if (K > M)
        throw std::runtime_error("--output-degree (" + std::to_string(K) + ") > input degree (" + std::to_string(M) + ")");

    const double elem = dtype == GTA_F32 ? 4.0 : 1.0;
    const double need = (skip_sort ? 0.0 : static_cast<double>(N) * d * elem) + static_cast<double>(N) * M * 4.0 +
                        static_cast<double>(N) * K * 4.0;
    int64_t free_b = 0, total_b = 0;
    check(gta_device_memory(&free_b, &total_b), "device memory query");
    std::printf("=== Step 0: fit check: %.2f GB x %.1f vs %.2f GB free\n", need / 1e9, margin, free_b / 1e9);
    if (a.flag("force-chunked")) {
        std::fprintf(stderr, "--force-chunked: refusing; run the chunked prune + reverse-edge path instead\n");
        return 2;
    }
    if (need * margin > static_cast<double>(free_b)) {
        std::fprintf(stderr, "does not fit on the GPU (%.2f GB x %.1f > %.2f GB free)\n", need / 1e9, margin,
                     free_b / 1e9);
        return 2;
    }

    auto t0 = Clock::now();
    std::vector<uint8_t> X;
    if (!skip_sort) {
        X.resize(static_cast<size_t>(N) * d * static_cast<size_t>(elem));
        check(gta_read_dataset(input.c_str(), 0, N, X.data()), "read dataset");
    }
    std::vector<int32_t> knn(static_cast<size_t>(N) * M);
    check(gta_read_knn(knn_path.c_str(), knn.data()), "read kNN graph");
    std::printf("=== Step 1-2: read dataset + kNN graph (N=%lld, M=%d) [%.3fs]\n", static_cast<long long>(N), M, secs(t0));

    t0 = Clock::now();
    std::vector<uint32_t> graph(static_cast<size_t>(N) * K);
    gta_dataset ds{X.data(), N, d, dtype, GTA_L2, 0};
    check(gta_optimize_knn(skip_sort ? nullptr : &ds, knn.data(), N, M, K, graph.data(), 0, nullptr), "optimize");
    std::printf("=== Step 3-4: sanitize%s + CAGRA optimize (prune to K_out=%d) [%.3fs]\n",
                skip_sort ? "" : " + sort", K, secs(t0));

    t0 = Clock::now();
    check(gta_write_graph(out_path.c_str(), graph.data(), N, K), "write graph");
    if (a.flag("save-npy")) {
        std::filesystem::path p(out_path);
        p.replace_extension(".npy");
        check(gta_write_npy_i64(p.string().c_str(), reinterpret_cast<const int32_t*>(graph.data()), N, K), "write npy");
        std::printf("[Write] %s (npy)\n", p.string().c_str());
    }
    std::printf("=== Step 5: write [%.3fs]\nTotal: %.3fs\nOutput: %s\n", secs(t0), secs(t_all), out_path.c_str());
    return 0;
}

}  // namespace

int main(int argc, char** argv)
{
    try {
        return run(argc, argv);
    } catch (const DoesNotFit& e) {
        std::fprintf(stderr, "does not fit: %s\n", e.what());
        return 2;
    } catch (const std::exception& e) {
        std::fprintf(stderr, "FATAL: %s\n", e.what());
        return 1;
    }
}
