// search.cu -- batched best-first graph search on the device (one warp per query).
//
// Restates bucketDemo/search.py:20-93 graph_search_single (paths relative to the
// reference root) so that a graph's search recall can be measured at device
// speed with the reference's own rule:
//   * the given entry points (drawn and de-duplicated on the host, ascending)
//     are visited in order;
//   * the candidate with the smallest (distance, id) is expanded next, until its
//     distance exceeds the worst of the best list once that list holds ef entries;
//   * the best list is an array in insertion order: appended while short, else
//     its first maximum is overwritten by a strictly smaller distance;
//   * neighbours outside [0, N) or already visited are skipped, the others are
//     handled in row order.
// The candidate set keeps only what can still be expanded: a candidate farther
// than the current worst of a full best list could only end the search when
// popped, which an empty candidate set does as well, so it is not stored (and
// candidates that fall behind a shrinking worst are dropped when the set is
// compacted).  Every warp-level step is data-parallel except the best-list and
// candidate updates, which run in row order exactly as the reference does.
// Distances: the exact fp32 chain over ascending dimensions (exact integers for
// 8-bit data).
#include <cfloat>
#include <cmath>

#include "common.cuh"
#include "gta_internal.h"
#include "prof.h"

namespace gta {

namespace {

constexpr int kSearchWarps = 3;       // queries per CTA (one per warp)
constexpr int kVisitCap = 16384;      // visited-set slots per query
constexpr int kVisitMax = 12288;      // load limit of the visited set (3/4)
constexpr int kCandCap = 640;         // candidate slots per query
constexpr uint32_t kNoId = 0xFFFFFFFFu;

struct SearchArgs {
    const void* base;
    int dtype;
    int64_t n;
    int d;
    const uint32_t* graph;
    int kg;
    const void* queries;
    int64_t nq;
    const int32_t* entries;
    int ne;
    int topk;
    int ef;
    int32_t* out_ids;
    float* out_dists;
    int* err;
};

__device__ __forceinline__ uint32_t visit_hash(uint32_t v) { return (v * 2654435761u) >> 8; }

template <typename T>
__device__ __forceinline__ float row_dist(const float* __restrict__ q, const T* __restrict__ x, int d)
{
    float acc = 0.0f;
    for (int i = 0; i < d; ++i) {
        const float t = q[i] - to_f32(x[i]);
        acc = fmaf(t, t, acc);
    }
    return acc;
}

// 8-bit rows with d % 16 == 0 (16-byte aligned): 16-byte loads, the same ascending chain.
template <>
__device__ __forceinline__ float row_dist<uint8_t>(const float* __restrict__ q, const uint8_t* __restrict__ x, int d)
{
    float acc = 0.0f;
    if ((d & 15) == 0 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0) {
        const uint4* x4 = reinterpret_cast<const uint4*>(x);
        for (int b = 0; b < (d >> 4); ++b) {
            const uint4 v = x4[b];
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int k = 0; k < 16; ++k) {
                const float t = q[b * 16 + k] - static_cast<float>((w[k >> 2] >> (8 * (k & 3))) & 0xffu);
                acc = fmaf(t, t, acc);
            }
        }
        return acc;
    }
    for (int i = 0; i < d; ++i) {
        const float t = q[i] - static_cast<float>(x[i]);
        acc = fmaf(t, t, acc);
    }
    return acc;
}

// Warp-wide argmin (by (d, id)) or argmax-first (by d, then lowest position) helpers.
__device__ __forceinline__ void warp_min_pair(float& d, uint32_t& id, int& pos)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float od = __shfl_xor_sync(0xffffffffu, d, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, id, o);
        const int op = __shfl_xor_sync(0xffffffffu, pos, o);
        if (od < d || (od == d && oi < id)) { d = od; id = oi; pos = op; }
    }
}

__device__ __forceinline__ void warp_max_first(float& d, int& pos)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float od = __shfl_xor_sync(0xffffffffu, d, o);
        const int op = __shfl_xor_sync(0xffffffffu, pos, o);
        if (od > d || (od == d && op < pos)) { d = od; pos = op; }
    }
}

template <typename T>
__global__ void __launch_bounds__(kSearchWarps * 32) search_kernel(const SearchArgs a)
{
    extern __shared__ __align__(16) uint8_t sm[];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const size_t per_warp = static_cast<size_t>(kVisitCap) * 4 + static_cast<size_t>(kCandCap) * 8 +
                            static_cast<size_t>(a.ef) * 8 + static_cast<size_t>(a.d) * 4;
    uint8_t* mine = sm + w * per_warp;
    uint32_t* vis = reinterpret_cast<uint32_t*>(mine);
    float* cd = reinterpret_cast<float*>(vis + kVisitCap);
    uint32_t* ci = reinterpret_cast<uint32_t*>(cd + kCandCap);
    float* bd = reinterpret_cast<float*>(ci + kCandCap);
    uint32_t* bi = reinterpret_cast<uint32_t*>(bd + a.ef);
    float* qv = reinterpret_cast<float*>(bi + a.ef);
    const T* base = static_cast<const T*>(a.base);
    const T* queries = static_cast<const T*>(a.queries);
    const uint32_t vmask = kVisitCap - 1;

    for (int64_t q = static_cast<int64_t>(blockIdx.x) * kSearchWarps + w; q < a.nq;
         q += static_cast<int64_t>(gridDim.x) * kSearchWarps) {
        for (int i = lane; i < kVisitCap; i += 32) vis[i] = kNoId;
        for (int i = lane; i < a.d; i += 32) qv[i] = to_f32(queries[q * a.d + i]);
        __syncwarp();
        int n_vis = 0, cn = 0, bs = 0;
        float wd = -FLT_MAX;  // worst distance of the best list (meaningful once bs >= ef)
        int wpos = 0;
        bool overflow = false;

        // Visits the chunk's candidate ids (one per lane, kNoId = none) in lane order.
        auto visit_chunk = [&](uint32_t v) {
            // first occurrence within the chunk only
            const unsigned valid = __ballot_sync(0xffffffffu, v != kNoId);
            const unsigned same = __match_any_sync(0xffffffffu, v);
            bool lead = v != kNoId && (__ffs(same & valid) - 1) == lane;
            // visited-set lookup and insert (ids in the chunk are now distinct)
            bool fresh = false;
            if (lead) {
                for (uint32_t h = visit_hash(v) & vmask;; h = (h + 1) & vmask) {
                    const uint32_t old = atomicCAS(&vis[h], kNoId, v);
                    if (old == kNoId) { fresh = true; break; }
                    if (old == v) break;
                }
            }
            const unsigned fm = __ballot_sync(0xffffffffu, fresh);
            n_vis += __popc(fm);
            if (n_vis > kVisitMax) overflow = true;
            float dv = 0.0f;
            if (fresh) dv = row_dist(qv, base + static_cast<int64_t>(v) * a.d, a.d);
            // the reference's sequential updates, in lane (= row) order
            for (unsigned m = fm; m != 0u; m &= m - 1u) {
                const int src = __ffs(m) - 1;
                const float d = __shfl_sync(0xffffffffu, dv, src);
                const uint32_t id = __shfl_sync(0xffffffffu, v, src);
                const bool was_full = bs >= a.ef;
                if (!was_full || d <= wd) {
                    if (cn >= kCandCap && was_full) {  // compact: drop what can no longer be expanded
                        int keep = 0;
                        for (int base_i = 0; base_i < cn; base_i += 32) {
                            const int i = base_i + lane;
                            const bool k = i < cn && cd[i] <= wd;
                            const float kd = i < cn ? cd[i] : 0.0f;
                            const uint32_t ki = i < cn ? ci[i] : 0u;
                            const unsigned km = __ballot_sync(0xffffffffu, k);
                            __syncwarp();
                            if (k) {
                                const int at = keep + __popc(km & ((1u << lane) - 1u));
                                cd[at] = kd;
                                ci[at] = ki;
                            }
                            keep += __popc(km);
                            __syncwarp();
                        }
                        cn = keep;
                    }
                    if (cn >= kCandCap) {
                        overflow = true;
                    } else {
                        if (lane == 0) { cd[cn] = d; ci[cn] = id; }
                        ++cn;
                    }
                }
                if (!was_full) {
                    if (lane == 0) { bd[bs] = d; bi[bs] = id; }
                    if (bs == 0 || d > wd) { wd = d; wpos = bs; }
                    ++bs;
                } else if (d < wd) {
                    if (lane == 0) { bd[wpos] = d; bi[wpos] = id; }
                    __syncwarp();
                    float md = -FLT_MAX;
                    int mp = 0x7fffffff;
                    for (int i = lane; i < bs; i += 32)
                        if (bd[i] > md) { md = bd[i]; mp = i; }
                    warp_max_first(md, mp);
                    wd = md;
                    wpos = mp;
                }
                __syncwarp();
            }
        };

        // entry points, in the given (ascending) order
        for (int e0 = 0; e0 < a.ne && !overflow; e0 += 32) {
            const int e = e0 + lane;
            int32_t s = e < a.ne ? a.entries[q * a.ne + e] : -1;
            const uint32_t v = (s >= 0 && static_cast<int64_t>(s) < a.n) ? static_cast<uint32_t>(s) : kNoId;
            visit_chunk(v);
        }
        // best-first expansion
        while (cn > 0 && !overflow) {
            float md = FLT_MAX;
            uint32_t mi = kNoId;
            int mp = -1;
            for (int i = lane; i < cn; i += 32)
                if (cd[i] < md || (cd[i] == md && ci[i] < mi)) { md = cd[i]; mi = ci[i]; mp = i; }
            warp_min_pair(md, mi, mp);
            __syncwarp();
            if (lane == 0) { cd[mp] = cd[cn - 1]; ci[mp] = ci[cn - 1]; }  // remove the popped candidate
            --cn;
            __syncwarp();
            if (bs >= a.ef && md > wd) break;
            const uint32_t* nb = a.graph + static_cast<int64_t>(mi) * a.kg;
            for (int j0 = 0; j0 < a.kg && !overflow; j0 += 32) {
                const int j = j0 + lane;
                const uint32_t v = j < a.kg ? nb[j] : kNoId;
                visit_chunk((v != kNoId && static_cast<int64_t>(v) < a.n) ? v : kNoId);
            }
        }
        if (overflow && lane == 0) atomicCAS(a.err, 0, kDevOverflow);
        // the best list sorted by (distance, id): each entry's rank by counting
        __syncwarp();
        for (int i = lane; i < bs; i += 32) {
            const float di = bd[i];
            const uint32_t ii = bi[i];
            int rank = 0;
            for (int j = 0; j < bs; ++j) rank += (bd[j] < di) || (bd[j] == di && bi[j] < ii);
            if (rank < a.topk) {
                a.out_ids[q * a.topk + rank] = static_cast<int32_t>(ii);
                a.out_dists[q * a.topk + rank] = di;
            }
        }
        for (int r = bs + lane; r < a.topk; r += 32) {
            a.out_ids[q * a.topk + r] = -1;
            a.out_dists[q * a.topk + r] = INFINITY;
        }
        __syncwarp();
    }
}

}  // namespace

void graph_search(const void* base, int dtype, int64_t n, int d, const uint32_t* graph, int kg, const void* queries,
                  int64_t nq, const int32_t* entries, int ne, int topk, int ef, int32_t* out_ids, float* out_dists,
                  int* err, cudaStream_t st)
{
    GTA_REQUIRE(n >= 1 && d >= 1 && d <= 1024 && kg >= 1 && ne >= 1 && topk >= 1 && ef >= topk && ef <= 256, kInvalid,
                "search: need 1 <= topk <= ef <= 256, d <= 1024");
    if (nq == 0) return;
    SearchArgs a{base, dtype, n, d, graph, kg, queries, nq, entries, ne, topk, ef, out_ids, out_dists, err};
    const size_t per_warp = static_cast<size_t>(kVisitCap) * 4 + static_cast<size_t>(kCandCap) * 8 +
                            static_cast<size_t>(ef) * 8 + static_cast<size_t>(d) * 4;
    const size_t smem = per_warp * kSearchWarps;
    int dev = 0, n_sm = 0;
    GTA_CUDA(cudaGetDevice(&dev));
    GTA_CUDA(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev));
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>((nq + kSearchWarps - 1) / kSearchWarps, n_sm));
    ProfScope prof("search", static_cast<double>(nq), st);
    switch (dtype) {
        case 0:
            GTA_CUDA(cudaFuncSetAttribute(search_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
            search_kernel<float><<<grid, kSearchWarps * 32, smem, st>>>(a);
            break;
        case 1:
            GTA_CUDA(cudaFuncSetAttribute(search_kernel<uint8_t>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
            search_kernel<uint8_t><<<grid, kSearchWarps * 32, smem, st>>>(a);
            break;
        case 2:
            GTA_CUDA(cudaFuncSetAttribute(search_kernel<int8_t>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
            search_kernel<int8_t><<<grid, kSearchWarps * 32, smem, st>>>(a);
            break;
        default: throw Error(kInvalid, "search: unknown dtype");
    }
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

}  // namespace gta
