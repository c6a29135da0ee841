// ref_bridge.cpp -- TEST INFRASTRUCTURE ONLY.
//
// C entry points over the reference's OWN header-only C++ restatements of the
// CAGRA prune and reverse-edge merge, compiled in place from the reference
// tree by oracle/Makefile (REF=<reference root>) into oracle/_ref/libgta_ref.so.
// Nothing from the reference is copied into this repository: the headers are
// included from their original location at build time.
//
//   bucketDemo/buildBucket/src/prune_windowed_core.hpp
//       WindowLookup, sort_row_by_l2 (:134), compute_detour_counts (:190),
//       select_pruned_row (:238)
//   bucketDemo/buildBucket/src/edge_chunk_accumulator.hpp
//       EdgeRecord (:54), build_rank_ordered_csr (:235), TopKReverseStore (:386),
//       merge_rank_ordered_into_row (:471)
//   bucketDemo/buildBucket/src/bucket_order.hpp
//       compute_bucket_processing_order (:143), adjacency_from_flat_graph (:202)
//   bucketDemo/buildBucket/src/translate_graph_ids.hpp
//       translate_graph_to_original_order (:75), translate_npy_to_original_order (:180)
//
// Used to (1) generate the golden fixtures under tests/golden/ and (2) time
// the reference's own CPU prune + reverse-edge code as bench.py's reference
// arm for that stage.
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <vector>

#include "prune_windowed_core.hpp"
#include "edge_chunk_accumulator.hpp"
#include "bucket_order.hpp"
#include "translate_graph_ids.hpp"

#define REF_API extern "C" __attribute__((visibility("default")))

namespace {

// Full-visibility window over an (N, M) int32 candidate table (the exact,
// un-windowed CAGRA rule: every point's row is resident).
prune_windowed::WindowLookup full_window(const int32_t* knn, int64_t N, int32_t M, const float* X, int32_t D)
{
    prune_windowed::WindowLookup w;
    w.reserve(static_cast<size_t>(N));
    static const float zero = 0.0f;
    for (int64_t i = 0; i < N; ++i)
        w.add(static_cast<uint32_t>(i), knn + i * M, X ? X + i * static_cast<int64_t>(D) : &zero);
    return w;
}

}  // namespace

REF_API int ref_detour_counts(const int32_t* knn, int64_t N, int32_t M, int64_t a, uint32_t* out)
{
    try {
        auto w = full_window(knn, N, M, nullptr, 0);
        std::vector<uint32_t> cnt;
        prune_windowed::compute_detour_counts(knn + a * M, M, w, cnt);
        std::memcpy(out, cnt.data(), sizeof(uint32_t) * static_cast<size_t>(M));
        return 0;
    } catch (...) { return 5; }
}

REF_API int ref_select_pruned_row(const int32_t* row, int32_t M, const uint32_t* cnt, int32_t K, uint32_t* out)
{
    try {
        std::vector<uint32_t> c(cnt, cnt + M);
        prune_windowed::select_pruned_row(row, M, c, K, out);
        return 0;
    } catch (...) { return 5; }
}

REF_API int ref_sort_row_by_l2(const float* X, int32_t D, const int32_t* knn, int64_t N, int32_t M, int64_t a,
                               int32_t* out)
{
    try {
        auto w = full_window(knn, N, M, X, D);
        std::vector<int32_t> s;
        prune_windowed::sort_row_by_l2(static_cast<uint32_t>(a), knn + a * M, M, D, w, s);
        std::memcpy(out, s.data(), sizeof(int32_t) * static_cast<size_t>(M));
        return 0;
    } catch (...) { return 5; }
}

// CAGRA optimize over an already distance-sorted, sanitized (N, M) graph:
// full-window detour counts + selection per row, then the reverse-edge
// store (L = K) and the protected merge per row.
REF_API int ref_optimize(const uint32_t* knn_u32, int64_t N, int32_t M, int32_t K, uint32_t* out)
{
    try {
        const int32_t* knn = reinterpret_cast<const int32_t*>(knn_u32);
        auto w = full_window(knn, N, M, nullptr, 0);
        #pragma omp parallel
        {
            std::vector<uint32_t> cnt;
            #pragma omp for schedule(dynamic, 256)
            for (int64_t a = 0; a < N; ++a) {
                prune_windowed::compute_detour_counts(knn + a * M, M, w, cnt);
                prune_windowed::select_pruned_row(knn + a * M, M, cnt, K, out + a * K);
            }
        }
        edge_chunk::TopKReverseStore store;
        store.init(N, static_cast<uint32_t>(K));
        std::vector<edge_chunk::EdgeRecord> recs(static_cast<size_t>(N) * K);
        for (int64_t i = 0; i < N; ++i)
            for (int32_t r = 0; r < K; ++r)
                recs[static_cast<size_t>(i) * K + r] =
                    edge_chunk::EdgeRecord{out[i * K + r], static_cast<uint32_t>(i), static_cast<uint16_t>(r)};
        store.add(recs.data(), recs.size());
        #pragma omp parallel
        {
            std::vector<uint32_t> src(static_cast<size_t>(K));
            #pragma omp for schedule(static)
            for (int64_t j = 0; j < N; ++j) {
                uint32_t c = store.sources(static_cast<uint32_t>(j), src.data());
                edge_chunk::merge_rank_ordered_into_row(out + j * K, src.data(), c, static_cast<uint32_t>(K));
            }
        }
        return 0;
    } catch (...) { return 5; }
}

// build_rank_ordered_csr over (dst, src, rank) triples of one chunk.
REF_API int ref_rank_ordered_csr(const uint32_t* dst, const uint32_t* src, const uint16_t* rank, int64_t n_edges,
                                 uint32_t j_lo, uint32_t chunk_size, uint32_t* row_offsets, uint32_t* csr_src)
{
    try {
        edge_chunk::EdgeVec e(static_cast<size_t>(n_edges));
        for (int64_t i = 0; i < n_edges; ++i) e[static_cast<size_t>(i)] = edge_chunk::EdgeRecord{dst[i], src[i], rank[i]};
        auto csr = edge_chunk::build_rank_ordered_csr(e, j_lo, chunk_size);
        std::memcpy(row_offsets, csr.row_offsets.data(), sizeof(uint32_t) * csr.row_offsets.size());
        std::memcpy(csr_src, csr.src.data(), sizeof(uint32_t) * csr.src.size());
        return 0;
    } catch (...) { return 5; }
}

REF_API void ref_merge_rank_ordered_into_row(uint32_t* row, const uint32_t* src, uint32_t count, uint32_t K)
{
    edge_chunk::merge_rank_ordered_into_row(row, src, count, K);
}

// Bucket processing order of a flat (B, K) uint32 bucket graph.
REF_API int ref_bucket_order(const uint32_t* graph, int64_t B, int32_t K, int32_t window, int32_t* out)
{
    try {
        auto order = bucket_order::compute_bucket_processing_order(
            bucket_order::adjacency_from_flat_graph(graph, B, K), window);
        std::memcpy(out, order.data(), sizeof(int32_t) * order.size());
        return 0;
    } catch (...) { return 5; }
}

// translate_ids on files: a graph .bin (int64 N, int32 K, uint32) or a .npy (int64).
REF_API int ref_translate_graph(const char* graph_path, const char* inv_path, const char* out_path)
{
    try {
        translate_ids::translate_graph_to_original_order(graph_path, inv_path, out_path);
        return 0;
    } catch (...) { return 5; }
}

REF_API int ref_translate_npy(const char* npy_path, const char* inv_path, const char* out_path)
{
    try {
        translate_ids::translate_npy_to_original_order(npy_path, inv_path, out_path);
        return 0;
    } catch (...) { return 5; }
}
