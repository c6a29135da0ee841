// Bucket-contiguous renumbering of a dataset and its graphs (paths relative to the
// reference project root):
//   bucket_reorder      compute_bucket_reorder (bucketDemo/buildBucket/src/bucket.cu:8356-8417):
//                       new ids laid out bucket by bucket in processing order, points of one
//                       bucket in ascending old id; inverse_perm[new] = old
//   permute_rows        the inline dataset reorder bucket2 does in its first build round
//                       (bucket.cu:9253-9403):
//                       row new of the output = row inverse_perm[new] of the input
//   permute_graph       to_original: translate_graph_to_original_order /
//                       translate_npy_to_original_order (translate_graph_ids.hpp:75-200):
//                       row inv[i] of the output = row i with every id v mapped to inv[v];
//                       to new ids: the inverse map (row i = old row inv[i], ids old -> new)
//   bucket_order        compute_bucket_processing_order (bucket_order.hpp:143-200) on the
//                       centroid kNN graph (adjacency_from_flat_graph, :202-218), host code:
//                       it orders B buckets, not points
// Every id read from the caller is range-checked; a bad id or a non-permutation sets the
// device error flag (data check failed) and the offending element is skipped.
#include <cub/cub.cuh>

#include <algorithm>
#include <set>
#include <utility>
#include <vector>

#include "common.cuh"
#include "gta_internal.h"
#include "prof.h"

namespace gta {

namespace {

unsigned grid_for(int64_t n, int per) { return static_cast<unsigned>((n + per - 1) / per); }

// pos_of[order[p]] = p; order must be a permutation of [0, B) (null: identity).
__global__ void order_positions_kernel(const int32_t* __restrict__ order, int32_t B, int32_t* __restrict__ pos_of,
                                       int* err)
{
    const int32_t p = static_cast<int32_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (p >= B) return;
    const int32_t b = order ? order[p] : p;
    if (b < 0 || b >= B) {
        atomicCAS(err, 0, kDevBadIndex);
        return;
    }
    if (atomicExch(&pos_of[b], p) != -1) atomicCAS(err, 0, kDevBadIndex);  // bucket listed twice
}

__global__ void reorder_keys_kernel(const int32_t* __restrict__ assign, int64_t n, int32_t stride, int32_t B,
                                    const int32_t* __restrict__ pos_of, uint32_t* __restrict__ keys,
                                    int32_t* __restrict__ vals, int* err)
{
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int32_t a = assign[i * stride];
    uint32_t key = static_cast<uint32_t>(B);  // unassigned points sort last (and fail the call)
    if (a >= 0 && a < B && pos_of[a] >= 0) key = static_cast<uint32_t>(pos_of[a]);
    else atomicCAS(err, 0, kDevBadIndex);
    keys[i] = key;
    vals[i] = static_cast<int32_t>(i);
}

// offsets[p] = first sorted position whose key is >= p, p in [0, B]
__global__ void key_offsets_kernel(const uint32_t* __restrict__ keys_sorted, int64_t n, int32_t B,
                                   int64_t* __restrict__ offsets)
{
    const int64_t p = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (p > B) return;
    int64_t lo = 0, hi = n;
    while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if (static_cast<int64_t>(keys_sorted[mid]) < p) lo = mid + 1;
        else hi = mid;
    }
    offsets[p] = lo;
}

// One warp per output row; 16-byte moves when rows and bases are 16-byte aligned.
__global__ void permute_rows_kernel(const uint8_t* __restrict__ X, int64_t n, int64_t row_bytes,
                                    const uint32_t* __restrict__ inv, uint8_t* __restrict__ out, int vec16, int* err)
{
    const int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (r >= n) return;
    const uint32_t src = inv[r];
    if (static_cast<int64_t>(src) >= n) {
        if (lane == 0) atomicCAS(err, 0, kDevBadIndex);
        return;
    }
    const uint8_t* s = X + static_cast<int64_t>(src) * row_bytes;
    uint8_t* d = out + r * row_bytes;
    if (vec16) {
        const uint4* s4 = reinterpret_cast<const uint4*>(s);
        uint4* d4 = reinterpret_cast<uint4*>(d);
        for (int64_t k = lane; k < (row_bytes >> 4); k += 32) d4[k] = s4[k];
    } else {
        for (int64_t k = lane; k < row_bytes; k += 32) d[k] = s[k];
    }
}

// perm[inv[i]] = i; inv must be a permutation of [0, n)
__global__ void invert_perm_kernel(const uint32_t* __restrict__ inv, int64_t n, int32_t* __restrict__ perm, int* err)
{
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint32_t v = inv[i];
    if (static_cast<int64_t>(v) >= n) {
        atomicCAS(err, 0, kDevBadIndex);
        return;
    }
    if (atomicExch(&perm[v], static_cast<int32_t>(i)) != -1) atomicCAS(err, 0, kDevBadIndex);
}

// One thread per element.  to_original: out[inv[i]][j] = inv[g[i][j]];
// otherwise out[i][j] = perm[g[inv[i]][j]].  Negative ids stay -1 when keep_padding.
__global__ void permute_graph_kernel(const int32_t* __restrict__ g, int64_t n, int32_t m,
                                     const uint32_t* __restrict__ inv, const int32_t* __restrict__ perm,
                                     int to_original, int keep_padding, int32_t* __restrict__ out, int* err)
{
    const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (e >= n * m) return;
    const int64_t i = e / m;
    const int32_t j = static_cast<int32_t>(e - i * m);
    const uint32_t r = inv[i];
    if (static_cast<int64_t>(r) >= n) {
        atomicCAS(err, 0, kDevBadIndex);
        return;
    }
    const int64_t src_row = to_original ? i : static_cast<int64_t>(r);
    const int64_t dst_row = to_original ? static_cast<int64_t>(r) : i;
    const int32_t v = g[src_row * m + j];
    int32_t mapped = -1;
    if (v < 0) {
        if (!keep_padding) atomicCAS(err, 0, kDevBadIndex);
    } else if (static_cast<int64_t>(v) >= n) {
        atomicCAS(err, 0, kDevBadIndex);
    } else {
        mapped = to_original ? static_cast<int32_t>(inv[v]) : perm[v];
    }
    out[dst_row * m + j] = mapped;
}

}  // namespace

void bucket_reorder(const int32_t* assign, int64_t n, int32_t stride, int32_t B, const int32_t* order,
                    uint32_t* inverse_perm, int64_t* offsets, int* err, cudaStream_t st)
{
    GTA_REQUIRE(n >= 1 && n < (1ll << 31) && B >= 1 && stride >= 1, kInvalid,
                "bucket_reorder: need 1 <= n < 2^31, B >= 1, stride >= 1");
    ProfScope prof("bucket_reorder", 24.0 * static_cast<double>(n), st);
    DevBuf<int32_t> pos_of(static_cast<size_t>(B), st);
    GTA_CUDA(cudaMemsetAsync(pos_of.get(), 0xff, sizeof(int32_t) * static_cast<size_t>(B), st));
    order_positions_kernel<<<grid_for(B, 256), 256, 0, st>>>(order, B, pos_of.get(), err);
    DevBuf<uint32_t> keys_in(static_cast<size_t>(n), st), keys_out(static_cast<size_t>(n), st);
    DevBuf<int32_t> vals_in(static_cast<size_t>(n), st);
    reorder_keys_kernel<<<grid_for(n, 256), 256, 0, st>>>(assign, n, stride, B, pos_of.get(), keys_in.get(),
                                                          vals_in.get(), err);
    int end_bit = 1;
    while ((1ll << end_bit) <= static_cast<int64_t>(B)) ++end_bit;
    int32_t* vals_out = reinterpret_cast<int32_t*>(inverse_perm);
    size_t tmp = 0;
    GTA_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, tmp, keys_in.get(), keys_out.get(), vals_in.get(), vals_out,
                                             static_cast<int>(n), 0, end_bit, st));
    DevBuf<uint8_t> tbuf(tmp, st);
    GTA_CUDA(cub::DeviceRadixSort::SortPairs(tbuf.get(), tmp, keys_in.get(), keys_out.get(), vals_in.get(), vals_out,
                                             static_cast<int>(n), 0, end_bit, st));
    if (offsets) key_offsets_kernel<<<grid_for(B + 1, 256), 256, 0, st>>>(keys_out.get(), n, B, offsets);
    count_launches(offsets ? 3 : 2);
    GTA_CUDA(cudaGetLastError());
}

void permute_rows(const void* X, int64_t n, int64_t row_bytes, const uint32_t* inverse_perm, void* out, int* err,
                  cudaStream_t st)
{
    GTA_REQUIRE(n >= 1 && row_bytes >= 1, kInvalid, "permute_rows: empty input");
    ProfScope prof("permute_rows", (2.0 * row_bytes + 4.0) * static_cast<double>(n), st);
    const bool vec16 = (row_bytes & 15) == 0 && (reinterpret_cast<uintptr_t>(X) & 15u) == 0 &&
                       (reinterpret_cast<uintptr_t>(out) & 15u) == 0;
    permute_rows_kernel<<<grid_for(n * 32, 256), 256, 0, st>>>(static_cast<const uint8_t*>(X), n, row_bytes,
                                                               inverse_perm, static_cast<uint8_t*>(out), vec16 ? 1 : 0,
                                                               err);
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

void permute_graph(const int32_t* g, int64_t n, int32_t m, const uint32_t* inverse_perm, bool to_original,
                   bool keep_padding, int32_t* out, int* err, cudaStream_t st)
{
    GTA_REQUIRE(n >= 1 && n < (1ll << 31) && m >= 1, kInvalid, "permute_graph: need 1 <= n < 2^31, m >= 1");
    ProfScope prof("permute_graph", (12.0 * m + 8.0) * static_cast<double>(n), st);
    DevBuf<int32_t> perm(static_cast<size_t>(n), st);
    GTA_CUDA(cudaMemsetAsync(perm.get(), 0xff, sizeof(int32_t) * static_cast<size_t>(n), st));
    invert_perm_kernel<<<grid_for(n, 256), 256, 0, st>>>(inverse_perm, n, perm.get(), err);  // also validates
    permute_graph_kernel<<<grid_for(n * m, 256), 256, 0, st>>>(g, n, m, inverse_perm, perm.get(), to_original ? 1 : 0,
                                                               keep_padding ? 1 : 0, out, err);
    count_launches(2);
    GTA_CUDA(cudaGetLastError());
}

// Greedy windowed bucket order over the bucket neighbour graph (adj: B x K, entries that are
// negative, >= B or the bucket itself are ignored).  Start: the bucket with the most neighbours
// (lowest id on ties).  Next: among the buckets already touched, the one sharing the most
// neighbour entries with the last `window` placed buckets (sum over placed x in the window and
// over neighbour entries u of x of the entries of v equal to u), highest id on ties; when none
// has been touched, the lowest unplaced id.
void bucket_order(const int32_t* adj, int32_t B, int32_t K, int32_t window, int32_t* order)
{
    GTA_REQUIRE(adj && order && B >= 1 && K >= 0, kInvalid, "bucket_order: bad argument");
    window = std::max(1, window);
    std::vector<std::vector<int32_t>> nb(static_cast<size_t>(B)), rev(static_cast<size_t>(B));
    for (int32_t v = 0; v < B; ++v)
        for (int32_t k = 0; k < K; ++k) {
            const int32_t u = adj[static_cast<size_t>(v) * K + k];
            if (u >= 0 && u < B && u != v) nb[static_cast<size_t>(v)].push_back(u);
        }
    for (int32_t v = 0; v < B; ++v)
        for (int32_t u : nb[static_cast<size_t>(v)]) rev[static_cast<size_t>(u)].push_back(v);
    std::vector<int64_t> score(static_cast<size_t>(B), 0);
    std::vector<char> placed(static_cast<size_t>(B), 0), touched(static_cast<size_t>(B), 0);
    std::set<std::pair<int64_t, int32_t>> ready;  // (score, id) of touched, unplaced buckets
    auto shift = [&](int32_t x, int64_t delta) {
        for (int32_t u : nb[static_cast<size_t>(x)])
            for (int32_t v : rev[static_cast<size_t>(u)]) {
                if (placed[static_cast<size_t>(v)]) continue;
                if (touched[static_cast<size_t>(v)]) ready.erase({score[static_cast<size_t>(v)], v});
                touched[static_cast<size_t>(v)] = 1;
                score[static_cast<size_t>(v)] += delta;
                ready.insert({score[static_cast<size_t>(v)], v});
            }
    };
    int32_t start = 0;
    for (int32_t v = 1; v < B; ++v)
        if (nb[static_cast<size_t>(v)].size() > nb[static_cast<size_t>(start)].size()) start = v;
    int32_t lowest_free = 0;
    order[0] = start;
    placed[static_cast<size_t>(start)] = 1;
    shift(start, +1);
    for (int32_t i = 1; i < B; ++i) {
        if (i > window) shift(order[i - window - 1], -1);
        int32_t pick;
        if (!ready.empty()) {
            auto it = std::prev(ready.end());
            pick = it->second;
            ready.erase(it);
        } else {
            while (placed[static_cast<size_t>(lowest_free)]) ++lowest_free;
            pick = lowest_free;
        }
        order[i] = pick;
        placed[static_cast<size_t>(pick)] = 1;
        shift(pick, +1);
    }
}

}  // namespace gta
