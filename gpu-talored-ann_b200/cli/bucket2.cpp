// bucket2: command-line front end of the bucketed kNN-graph build, with the
// reference tool's options and outputs (bucketDemo/buildBucket/src/bucket.cu:9853
// main, :9897-9954 options, :8545-8556 output subdirectory, :9755-9761 outputs).
//
//   bucket2 -i data.u8bin -o out --neighbors-m 64 --fused-optimize-degree 32 [--seed 42] [-t 1]
//
// writes into out/k<knn-k>p<nprobe|knn-k>m<M>t<T>/ what the reference's GPU-resident path
// writes: the bucket-contiguous renumbering of the points (bucket.cu:9253-9456):
// data_reordered.<ext>, inverse_perm.bin (uint32[N], new -> old), bucket_offsets.bin (int32 B,
// uint32[B+1]), bucket_process_order.bin (int32 B, int32[B]), centroid_knn.bin (int64 B,
// int32 K, uint32[B*K]); then, in the reordered id space, vector_knn.bin, vector_dists.bin
// (unless --skip-dists) and neighbors.npy (unless --skip-npy); and with
// --fused-optimize-degree K, final_graph.bin: sanitize + CAGRA prune + reverse edges in the
// reordered space, translated back to the input order (bucket.cu:8434-8480).
// --bucketing reference (the default) is the reference tool's own bucketing (gta_build_bucket2):
// KMeans|| data-point centroids (N x --centroid-ratio), balanced 1-way buckets, every bucket
// searched in the pool of itself and its --nprobe (0: --knn-k) nearest buckets.
// --bucketing top2 is this library's 2-way build: k-means over a sample, every point in its two
// nearest buckets (--n-buckets, default N/3906, i.e. buckets of about 7 800 members).
// The renumbering groups points by their bucket (the nearest one for top2), buckets in the greedy
// order over the centroid kNN graph (--knn-k neighbours, --order-window).  The kNN lists are
// built in the input order and renumbered afterwards, so equal distances stay ordered by input
// id.  The reference's memory / out-of-core / PQ knobs are accepted and ignored.
// Exit status: 0 ok, 1 error ("FATAL: ..." on stderr), like the reference.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <filesystem>
#include <cstdlib>
#include <string>
#include <vector>

#include "args.hpp"
#include "gta.h"

namespace {

using Clock = std::chrono::steady_clock;

double secs(Clock::time_point t0) { return std::chrono::duration<double>(Clock::now() - t0).count(); }

void check(int rc, const char* what)
{
    if (rc != GTA_OK) throw std::runtime_error(std::string(what) + ": " + gta_last_error());
}

size_t elem_bytes(int32_t dtype) { return dtype == GTA_F32 ? 4 : 1; }

// int32 count, then the values (bucket_offsets.bin / bucket_process_order.bin, graph_io.hpp:195-227)
template <typename T>
void write_counted(const char* path, int32_t count, const T* v, size_t n)
{
    FILE* f = std::fopen(path, "wb");
    if (!f) throw std::runtime_error(std::string("cannot open for writing: ") + path);
    const bool ok = std::fwrite(&count, sizeof(count), 1, f) == 1 && std::fwrite(v, sizeof(T), n, f) == n;
    if (std::fclose(f) != 0 || !ok) throw std::runtime_error(std::string("write failed: ") + path);
}

int run(int argc, char** argv)
{
    const std::vector<cli::Opt> opts = {
        {"input", 'i', false, "Input data file (.fbin/.bin/.u8bin/.i8bin)", ""},
        {"output", 'o', false, "Output root directory", ""},
        {"neighbors-m", 0, false, "Per-vector KNN neighbor count M (1..128)", "0"},
        {"fused-optimize-degree", 0, false, "Prune + reverse edges to this degree, write final_graph.bin (0 = off)", "0"},
        {"bucketing", 0, false, "reference (KMeans||, 1-way, own + nprobe pools) or top2 (2-way k-means)", "reference"},
        {"centroid-ratio", 0, false, "reference bucketing: buckets = N x ratio", "0.01"},
        {"n-buckets", 0, false, "top2 bucketing: k-means buckets B (0 = N/3906)", "0"},
        {"kmeans-iters", 0, false, "top2 bucketing: Lloyd iterations", "10"},
        {"sample-rate", 0, false, "top2 bucketing: k-means sample fraction of N (default min(0.1, 1e7/N))", ""},
        {"seed", 0, false, "Random seed", "42"},
        {"iterations", 't', false, "Whole builds with seed+iter, lists dedupe-merged", "1"},
        {"knn-k", 0, false, "Centroid graph degree (bucket order; the pool width when nprobe is 0)", "32"},
        {"nprobe", 0, false, "reference bucketing: neighbour buckets in a pool (0 = knn-k, <= 127)", "0"},
        {"order-window", 0, false, "Window of the bucket processing order (0 = max(4 knn-k, 16))", "0"},
        {"skip-dists", 0, true, "Don't write vector_dists.bin", ""},
        {"skip-npy", 0, true, "Don't write neighbors.npy", ""},
        // accepted for drop-in compatibility, no effect on this build
        {"cpu-limit", 0, false, "(ignored)", ""},
        {"gpu-limit", 0, false, "(ignored)", ""},
        {"bucket-vec-buffer", 0, false, "(ignored)", ""},
        {"use-pq", 0, false, "(ignored)", ""},
        {"kmeans-train-fraction", 0, false, "(ignored)", ""},
        {"bucket-mem-mb", 0, false, "(ignored)", ""},
        {"gpu-bucket-cache-mb", 0, false, "(ignored)", ""},
        {"pq-bits-start", 0, false, "(ignored)", ""},
        {"pq-bits-min", 0, false, "(ignored)", ""},
        {"search-iters", 0, false, "(ignored)", ""},
        {"cache-mb", 0, false, "(ignored)", ""},
        {"out-of-core", 0, true, "(ignored)", ""},
    };
    cli::Args a("bucket2 (gta-b200)", opts);
    if (!a.parse(argc, argv)) return 0;
    const std::string input = a.required("input");
    const std::string root = a.required("output");
    const int M = static_cast<int>(a.i64("neighbors-m", 0));
    const int K = static_cast<int>(a.i64("fused-optimize-degree", 0));
    const int iters = static_cast<int>(a.i64("iterations", 1));
    const int knn_k = static_cast<int>(a.i64("knn-k", 32));
    const int nprobe = static_cast<int>(a.i64("nprobe", 0));
    if (M < 1 || M > 128) throw std::runtime_error("--neighbors-m must be in [1, 128] (the kNN lists are the product)");
    if (K < 0 || K > M) throw std::runtime_error("--fused-optimize-degree must be in [0, neighbors-m]");
    if (iters < 1) throw std::runtime_error("iterations (" + std::to_string(iters) + ") must be >= 1");
    if (nprobe < 0 || nprobe > 127) throw std::runtime_error("nprobe must be in [0, 127] (this build's limit)");
    if (knn_k < 1 || knn_k > 127) throw std::runtime_error("knn-k must be in [1, 127]");
    const std::string bucketing = a.str("bucketing", "reference");
    if (bucketing != "reference" && bucketing != "top2")
        throw std::runtime_error("--bucketing must be reference or top2, not " + bucketing);

    const auto t_all = Clock::now();
    int64_t N = 0;
    int32_t d = 0, dtype = 0;
    check(gta_read_dataset_header(input.c_str(), &N, &d, &dtype), "read header");
    std::printf("[main] %s: N=%lld d=%d dtype=%s\n", input.c_str(), static_cast<long long>(N), d,
                dtype == GTA_F32 ? "f32" : dtype == GTA_U8 ? "u8" : "i8");
    std::vector<uint8_t> X(static_cast<size_t>(N) * d * elem_bytes(dtype));
    auto t0 = Clock::now();
    check(gta_read_dataset(input.c_str(), 0, N, X.data()), "read dataset");
    std::printf("=== Step 1: read dataset [%.3fs]\n", secs(t0));

    const std::string dir = root + "/k" + std::to_string(knn_k) + "p" + std::to_string(nprobe > 0 ? nprobe : knn_k) +
                            "m" + std::to_string(M) + "t" + std::to_string(iters);
    std::filesystem::create_directories(dir);
    std::printf("Output subdir: %s\n", dir.c_str());

    gta_dataset ds{X.data(), N, d, dtype, GTA_L2, 0};
    const uint64_t seed = static_cast<uint64_t>(a.i64("seed", 42));
    std::vector<int32_t> ids(static_cast<size_t>(N) * M);
    std::vector<float> dists(static_cast<size_t>(N) * M);
    std::vector<float> cent;              // B x d
    std::vector<int32_t> bucket_of(static_cast<size_t>(N));
    int64_t B = 0;
    t0 = Clock::now();
    if (bucketing == "reference") {
        const float ratio = static_cast<float>(a.f64("centroid-ratio", 0.01));
        const int64_t n_req = std::max<int64_t>(2, static_cast<int64_t>(static_cast<double>(N) * static_cast<double>(ratio)));
        std::vector<int32_t> cid(static_cast<size_t>(n_req));
        int32_t nb = 0;
        gta_bucket2_params q{};
        q.knn_degree = M;
        q.nprobe = nprobe;
        q.knn_k = knn_k;
        q.rounds = iters;
        q.centroid_ratio = ratio;
        // the reference tool's environment switch for the balanced choice
        const char* rule = std::getenv("BUCKET2_ASSIGN_RULE");
        q.assign_rule = (rule && std::string(rule) == "diskjoin") ? 1 : 0;
        q.seed = seed;
        q.assign_out = bucket_of.data();
        q.centroid_ids_out = cid.data();
        q.n_buckets_out = &nb;
        check(gta_build_bucket2(&ds, &q, ids.data(), dists.data(), nullptr), "reference-bucketing kNN build");
        B = nb;
        cent.resize(static_cast<size_t>(B) * d);  // the centroids are data points
        for (int64_t c = 0; c < B; ++c)
            for (int k = 0; k < d; ++k) {
                const size_t e = static_cast<size_t>(cid[static_cast<size_t>(c)]) * d + k;
                cent[static_cast<size_t>(c) * d + k] =
                    dtype == GTA_F32 ? reinterpret_cast<const float*>(X.data())[e]
                    : dtype == GTA_U8 ? static_cast<float>(X[e]) : static_cast<float>(reinterpret_cast<const int8_t*>(X.data())[e]);
            }
        std::printf("=== Steps 2-6: KMeans|| (%lld buckets), balanced 1-way assignment, pool kNN (nprobe %d, M=%d), "
                    "%d round(s) [%.3fs]\n", static_cast<long long>(B), nprobe > 0 ? nprobe : knn_k, M, iters, secs(t0));
    } else {
        B = a.i64("n-buckets", 0);
        if (B <= 0) B = std::max<int64_t>(2, static_cast<int64_t>(std::llround(static_cast<double>(N) / 3906.0)));
        int64_t sample = 0;
        if (a.has("sample-rate")) sample = std::max<int64_t>(B, static_cast<int64_t>(a.f64("sample-rate", 0.1) * N));
        gta_bucket_params p{};
        p.n_buckets = static_cast<int32_t>(B);
        p.kmeans_iters = static_cast<int32_t>(a.i64("kmeans-iters", 10));
        p.knn_degree = M;
        p.rounds = iters;
        p.kmeans_sample = sample;
        p.seed = seed;
        cent.resize(static_cast<size_t>(B) * d);
        std::vector<int32_t> top2(static_cast<size_t>(N) * 2);
        p.centroids_out = cent.data();
        p.top2_out = top2.data();
        check(gta_build_bucket(&ds, &p, ids.data(), dists.data(), nullptr), "bucketed kNN build");
        for (int64_t i = 0; i < N; ++i) bucket_of[static_cast<size_t>(i)] = top2[static_cast<size_t>(2 * i)];
        std::printf("=== Steps 2-6: k-means (B=%lld), top-2 buckets, per-bucket kNN (M=%d), merge, %d round(s) [%.3fs]\n",
                    static_cast<long long>(B), M, iters, secs(t0));
    }

    // bucket-contiguous renumbering: order of the buckets, new ids, reordered rows and lists
    t0 = Clock::now();
    const int ck = static_cast<int>(std::min<int64_t>({static_cast<int64_t>(knn_k), B - 1, 127}));
    std::vector<int32_t> order(static_cast<size_t>(B)), cknn(static_cast<size_t>(B) * ck);
    check(gta_bucket_order(cent.data(), static_cast<int32_t>(B), d, ck, static_cast<int32_t>(a.i64("order-window", 0)),
                           order.data(), cknn.data(), 0, nullptr),
          "bucket order");
    std::vector<uint32_t> inv(static_cast<size_t>(N));
    std::vector<int64_t> offsets(static_cast<size_t>(B) + 1);
    check(gta_bucket_reorder(bucket_of.data(), N, 1, static_cast<int32_t>(B), order.data(), inv.data(), offsets.data(),
                             0, nullptr),
          "bucket reorder");
    std::vector<uint8_t> Xr(X.size());
    check(gta_permute_rows(X.data(), N, static_cast<int64_t>(d) * static_cast<int64_t>(elem_bytes(dtype)), inv.data(),
                           Xr.data(), 0, nullptr),
          "reorder dataset");
    std::vector<int32_t> ids_new(ids.size());
    std::vector<float> dists_new(dists.size());
    check(gta_permute_graph(ids.data(), N, M, inv.data(), 0, 1, ids_new.data(), 0, nullptr), "renumber kNN lists");
    check(gta_permute_rows(dists.data(), N, 4ll * M, inv.data(), dists_new.data(), 0, nullptr), "reorder distances");
    std::printf("=== Step 4.5: bucket order (centroid kNN k=%d) + renumbering [%.3fs]\n", ck, secs(t0));

    std::vector<uint32_t> graph;
    if (K > 0) {
        graph.resize(static_cast<size_t>(N) * K);
        std::vector<uint32_t> graph_new(graph.size());
        t0 = Clock::now();
        check(gta_optimize_knn(nullptr, ids_new.data(), N, M, K, graph_new.data(), 0, nullptr), "optimize");
        check(gta_permute_graph(reinterpret_cast<const int32_t*>(graph_new.data()), N, K, inv.data(), 1, 0,
                                reinterpret_cast<int32_t*>(graph.data()), 0, nullptr),
              "translate ids");
        std::printf("=== fused optimize (prune + reverse edges to K=%d) + translate ids [%.3fs]\n", K, secs(t0));
    }

    t0 = Clock::now();
    const std::string ext = std::filesystem::path(input).extension().string();
    check(gta_write_dataset((dir + "/data_reordered" + ext).c_str(), Xr.data(), N, d, dtype), "write data_reordered");
    check(gta_write_u32((dir + "/inverse_perm.bin").c_str(), inv.data(), N), "write inverse_perm.bin");
    {
        std::vector<uint32_t> off32(offsets.begin(), offsets.end());
        write_counted((dir + "/bucket_offsets.bin").c_str(), static_cast<int32_t>(B), off32.data(), off32.size());
        write_counted((dir + "/bucket_process_order.bin").c_str(), static_cast<int32_t>(B), order.data(), order.size());
    }
    check(gta_write_graph((dir + "/centroid_knn.bin").c_str(), reinterpret_cast<const uint32_t*>(cknn.data()), B, ck),
          "write centroid_knn.bin");
    check(gta_write_knn((dir + "/vector_knn.bin").c_str(), ids_new.data(), N, M), "write vector_knn.bin");
    if (!a.flag("skip-dists"))
        check(gta_write_knn_dists((dir + "/vector_dists.bin").c_str(), dists_new.data(), N, M), "write vector_dists.bin");
    if (!a.flag("skip-npy"))
        check(gta_write_npy_i64((dir + "/neighbors.npy").c_str(), ids_new.data(), N, M), "write neighbors.npy");
    if (K > 0) check(gta_write_graph((dir + "/final_graph.bin").c_str(), graph.data(), N, K), "write final_graph.bin");
    std::printf("=== write outputs [%.3fs]\n", secs(t0));
    std::printf("Total: %.3fs\n", secs(t_all));
    return 0;
}

}  // namespace

int main(int argc, char** argv)
{
    try {
        return run(argc, argv);
    } catch (const std::exception& e) {
        std::fprintf(stderr, "FATAL: %s\n", e.what());
        return 1;
    }
}
