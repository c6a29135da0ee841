// Test infrastructure (the checker, never the product): the reference's own bucket-assignment
// loops, compiled from their lines in the reference source so that the oracle's restatement of
// them can be checked against the reference itself.
//
// Two loops of bucketDemo/buildBucket/src/bucket.cu are not in a header, so the Makefile streams
// each one (nothing is copied into this tree) into one of the functions below through
// REF_FRAGMENT (a path, "/dev/stdin"), with the variables that the loop reads declared as the
// reference declares them:
//   REF_PART_BALANCED: the balanced 1-way choice of batch_assign_with_cagra_anns (:2277-2302),
//     inside the batch loop of :1576-1660 (centroid points preassigned, sizes start at 1,
//     non-centroid points in index order); built without OpenMP, so the loop runs in index
//     order on one thread, the only order of the reference that is reproducible;
//   REF_PART_POOL: the CSR of buckets and the pool segment tables of GpuResidentKnn::run_round
//     (:5317-5347).
#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <stdexcept>
#include <string>
#include <vector>

#ifdef REF_PART_BALANCED
// top2[N x 2] (nearest, second nearest centroid), top2_d[N x 2] their squared distances (read by
// the diskjoin rule), cid[B] the centroids' point ids; batch: points per batch (any value gives
// the same result on one thread).  Writes assign[N].
extern "C" void ref_balanced_assign(const int32_t* top2_in, const float* top2_d_in, int64_t N, int32_t n_c_in,
                                    const int32_t* cid, int32_t diskjoin, int64_t batch, int32_t* assign_out)
{
    constexpr uint32_t TOP_K = 2;
    const int64_t n_centroids = n_c_in;
    const bool rule_dj = diskjoin != 0;
    std::vector<int64_t> assignments(N, -1);
    std::vector<char> is_c(N, 0);
    for (int64_t c = 0; c < n_centroids; ++c) {
        assignments[cid[c]] = c;
        is_c[cid[c]] = 1;
    }
    std::vector<std::atomic<int64_t>> cluster_sizes(n_centroids);
    for (auto& s : cluster_sizes) s.store(1, std::memory_order_relaxed);
    std::vector<int64_t> non_centroid_indices;
    for (int64_t i = 0; i < N; ++i)
        if (!is_c[i]) non_centroid_indices.push_back(i);
    const int64_t N_nc = static_cast<int64_t>(non_centroid_indices.size());
    std::vector<uint32_t> h_top2;
    std::vector<float> h_top2_d;
    for (int64_t batch_start = 0; batch_start < N_nc; batch_start += batch) {
        const int64_t batch_end = std::min(batch_start + batch, N_nc);
        const int64_t batch_size = batch_end - batch_start;
        h_top2.assign(static_cast<size_t>(batch_size) * TOP_K, 0);
        h_top2_d.assign(static_cast<size_t>(batch_size) * TOP_K, 0.f);
        for (int64_t i = 0; i < batch_size; ++i) {
            const int64_t g = non_centroid_indices[batch_start + i];
            for (uint32_t k = 0; k < TOP_K; ++k) {
                h_top2[i * TOP_K + k] = static_cast<uint32_t>(top2_in[g * TOP_K + k]);
                if (top2_d_in) h_top2_d[i * TOP_K + k] = top2_d_in[g * TOP_K + k];
            }
        }
#include REF_FRAGMENT
    }
    for (int64_t i = 0; i < N; ++i) assign_out[i] = static_cast<int32_t>(assignments[i]);
}
#endif

#ifdef REF_PART_POOL
// assign[N] (every point's bucket), centroid_topK[B x P] (each bucket's neighbour buckets).
// Writes offsets[B+1], members[N], seg_bucket[B x (P+1)], seg_ofs[B x (P+1)], pool_size[B].
extern "C" void ref_pool_tables(const int32_t* assign, int64_t N_in, int64_t n_c_in, const uint32_t* centroid_topK,
                                uint32_t P, int64_t* off_out, int32_t* members_out, int32_t* seg_bucket_out,
                                int32_t* seg_ofs_out, int64_t* pool_size_out)
{
    const int64_t N = N_in;
    const int64_t n_centroids = n_c_in;
    std::vector<int64_t> assignments(assign, assign + N);
#include REF_FRAGMENT
    std::copy(offsets.begin(), offsets.end(), off_out);
    std::copy(members.begin(), members.end(), members_out);
    std::copy(seg_bucket.begin(), seg_bucket.end(), seg_bucket_out);
    std::copy(seg_ofs.begin(), seg_ofs.end(), seg_ofs_out);
    std::copy(pool_size.begin(), pool_size.end(), pool_size_out);
}
#endif
