// Kernels of the reference-bucketing build (the bucketing of the reference's bucket2 tool;
// paths relative to the reference project root):
//   KMeans|| data-point centroids   select_centroids_on_gpu_kmeans_parallel
//                                   (bucketDemo/buildBucket/src/bucket.cu:2833-3217): a random first
//                                   point, three rounds that take each point with probability
//                                   0.5 * n_centroids * d(x)^2 / psi (kmeans_par_sample_kernel :2548),
//                                   psi estimated on a strided subsample (:2999-3016), then a uniform
//                                   subsample of the candidates down to n_centroids (:3150-3172)
//   balanced 1-way assignment       batch_assign_with_cagra_anns (:1552, the choice at :2276-2301):
//                                   nearest or second-nearest centroid, the second when its bucket
//                                   holds fewer than 0.8 x the first's points (or, with the diskjoin
//                                   rule of :2290-2292, fewer points and d2 < 1.2 d1); centroid
//                                   points stay in their own bucket, every bucket starts at size 1
//                                   (:1655-1660)
//   own + nprobe pools              GpuResidentKnn::run_round (:5310-5365): the pool of bucket c is
//                                   c's members followed by those of its nprobe nearest buckets
// Randomness comes from splitmix64 streams keyed by the seed (the reference's raft / mt19937
// streams cannot be reproduced).  The balanced choice runs in the reference loop's sequential
// order (each point sees every earlier point's choice): the reference's result on one OpenMP
// thread; with more threads its relaxed-atomic interleaving is not reproducible.
#include <cub/cub.cuh>

#include <algorithm>
#include <cstdint>

#include "../../include/gta.h"
#include "common.cuh"
#include "gta_internal.h"
#include "prof.h"

namespace gta {

namespace {

// take point i in round r when it is not yet a candidate and u < l * d(x)^2 / psi
__global__ void kpar_sample_kernel(const float* __restrict__ min_d, int64_t n, uint64_t seed, int round, double lk,
                                   const double* __restrict__ psi, uint8_t* __restrict__ chosen,
                                   uint8_t* __restrict__ sel)
{
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const double u = static_cast<double>(kpar_uniform_bits(seed, round, static_cast<uint64_t>(i))) * 0x1.0p-53;
    const bool take = !chosen[i] && u < (lk * static_cast<double>(min_d[i])) / *psi;
    sel[i] = take ? 1 : 0;
    if (take) chosen[i] = 1;
}

// psi = (sum of min_d[j * stride], j < sub_n) * n / sub_n, in a fixed order: lane l sums
// j = l, l + 32, ... ascending, then a shuffle tree 16, 8, 4, 2, 1 (fp64)
__global__ void kpar_psi_kernel(const float* __restrict__ min_d, int64_t n, int64_t stride, int64_t sub_n,
                                double* __restrict__ psi)
{
    const int lane = threadIdx.x;
    double s = 0.0;
    for (int64_t j = lane; j < sub_n; j += 32) s += static_cast<double>(min_d[j * stride]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_down_sync(0xffffffffu, s, o);
    if (lane == 0) *psi = s * (static_cast<double>(n) / static_cast<double>(sub_n));
}

__global__ void min_update_kernel(float* __restrict__ min_d, const float* __restrict__ d_new, int64_t n)
{
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) min_d[i] = fminf(min_d[i], d_new[i]);
}

// The balanced choice in the reference's sequential order: every non-centroid point, in index
// order, decides against the sizes left by all earlier points.  One warp takes 32 points at a
// time; lane i waits for the earlier lanes of its group that share one of its two buckets, and
// the lanes whose earlier sharers have decided choose together (their buckets are disjoint, so
// none of them sees another's update).  Sizes live in shared memory when they fit.
// rule 0: c2 when size(c2) < 0.8 size(c1) (double); rule 1 (diskjoin): c2 when
// size(c2) < size(c1) and d2 < 1.2f d1 (d: the two centroids' squared distances).
template <bool kShared>
__global__ void __launch_bounds__(32)
    balanced_assign_kernel(const int32_t* __restrict__ top2, const float* __restrict__ top2_d,
                           const int32_t* __restrict__ nc_ids, int64_t n_nc, int32_t n_c, int rule,
                           int32_t* __restrict__ g_sizes, int32_t* __restrict__ assign, int* err)
{
    extern __shared__ int32_t s_sizes[];
    volatile int32_t* sizes = kShared ? s_sizes : g_sizes;
    const int lane = threadIdx.x;
    if (kShared) {
        for (int32_t c = lane; c < n_c; c += 32) s_sizes[c] = g_sizes[c];
        __syncwarp();
    }
    // the group's points, loaded one group ahead
    auto load = [&](int64_t b0, int32_t& i, int32_t& c1, int32_t& c2, float& d1, float& d2) {
        const int64_t j = b0 + lane;
        i = -1; c1 = c2 = -1; d1 = d2 = 0.f;
        if (j < n_nc) {
            i = nc_ids[j];
            c1 = top2[2 * static_cast<int64_t>(i)];
            c2 = top2[2 * static_cast<int64_t>(i) + 1];
            if (rule == 1) {
                d1 = top2_d[2 * static_cast<int64_t>(i)];
                d2 = top2_d[2 * static_cast<int64_t>(i) + 1];
            }
        }
    };
    int32_t ni, nc1, nc2;
    float nd1, nd2;
    load(0, ni, nc1, nc2, nd1, nd2);
    for (int64_t b0 = 0; b0 < n_nc; b0 += 32) {
        const int32_t i = ni, c1 = nc1, c2 = nc2;
        const float d1 = nd1, d2 = nd2;
        if (b0 + 32 < n_nc) load(b0 + 32, ni, nc1, nc2, nd1, nd2);
        const bool valid = i >= 0 && c1 >= 0 && c1 < n_c && c2 >= 0 && c2 < n_c;
        if (i >= 0 && !valid) atomicCAS(err, 0, kDevBadIndex);
        // the earlier lanes of the group that share a bucket with this one
        unsigned dep = 0;
        for (int t = 0; t < 31; ++t) {
            const int32_t a = __shfl_sync(0xffffffffu, valid ? c1 : -1, t);
            const int32_t b = __shfl_sync(0xffffffffu, valid ? c2 : -1, t);
            if (t < lane && a >= 0 && (a == c1 || a == c2 || b == c1 || b == c2)) dep |= 1u << t;
        }
        unsigned pending = __ballot_sync(0xffffffffu, valid);
        while (pending) {
            const bool ready = ((pending >> lane) & 1u) && (dep & pending) == 0;
            int32_t chosen = -1;
            if (ready) {
                const int32_t s1 = sizes[c1], s2 = sizes[c2];
                const bool take2 = rule == 1 ? (s2 < s1 && d2 < 1.2f * d1)
                                             : (static_cast<double>(s2) < 0.8 * static_cast<double>(s1));
                chosen = take2 ? c2 : c1;
                assign[i] = chosen;
            }
            __syncwarp();
            if (ready) sizes[chosen] = sizes[chosen] + 1;  // the ready lanes' buckets are disjoint
            __syncwarp();
            pending &= ~__ballot_sync(0xffffffffu, ready);
        }
    }
}

__global__ void centroid_self_assign_kernel(const int32_t* __restrict__ cid, int32_t n_c, int32_t* __restrict__ assign,
                                            uint8_t* __restrict__ is_c, int32_t* __restrict__ sizes)
{
    const int32_t c = static_cast<int32_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (c >= n_c) return;
    assign[cid[c]] = c;
    is_c[cid[c]] = 1;
    sizes[c] = 1;
}

// pool_ids[pool_off[c] + seg_ofs[c][j] + k] = members[offsets[seg_b[c][j]] + k]
__global__ void pool_fill_kernel(const int32_t* __restrict__ members, const int64_t* __restrict__ offsets,
                                 const int32_t* __restrict__ seg_b, const int64_t* __restrict__ seg_dst, int32_t S,
                                 int32_t c_lo, int32_t n_buckets, int32_t* __restrict__ pool_ids)
{
    const int64_t s = blockIdx.x;  // (bucket - c_lo) * S + segment
    if (s >= static_cast<int64_t>(n_buckets) * S) return;
    const int32_t b = seg_b[(c_lo * static_cast<int64_t>(S)) + s];
    if (b < 0) return;
    const int64_t lo = offsets[b], len = offsets[b + 1] - lo;
    const int64_t dst = seg_dst[s];
    for (int64_t k = threadIdx.x; k < len; k += blockDim.x) pool_ids[dst + k] = members[lo + k];
}

// mem_row of a 1-way build: point members[i] owns list row i; no second membership
__global__ void one_way_rows_kernel(const int32_t* __restrict__ members, int64_t n, int64_t* __restrict__ mem_row)
{
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int64_t p = members[i];
    mem_row[2 * p] = i;
    mem_row[2 * p + 1] = -1;
}

__global__ void flag_not_kernel(const uint8_t* __restrict__ f, int64_t n, uint8_t* __restrict__ out)
{
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) out[i] = f[i] ? 0 : 1;
}

unsigned grid_of(int64_t n, int per) { return static_cast<unsigned>((n + per - 1) / per); }

}  // namespace

void kpar_psi(const float* min_d, int64_t n, double* psi, cudaStream_t st)
{
    const int64_t stride = std::max<int64_t>(1, n / kKparPsiTarget);
    const int64_t sub_n = n / stride;
    kpar_psi_kernel<<<1, 32, 0, st>>>(min_d, n, stride, sub_n, psi);
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

void kpar_sample(const float* min_d, int64_t n, uint64_t seed, int round, double lk, const double* psi, uint8_t* chosen,
                 uint8_t* sel, cudaStream_t st)
{
    kpar_sample_kernel<<<grid_of(n, 256), 256, 0, st>>>(min_d, n, seed, round, lk, psi, chosen, sel);
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

int64_t select_flagged(const uint8_t* flags, int64_t n, int32_t* out, cudaStream_t st)
{
    GTA_REQUIRE(n < (1ll << 31), kInvalid, "select_flagged: n must be below 2^31");
    DevBuf<int32_t> iota_b(static_cast<size_t>(n), st);
    sample_ids(n, n, 0, iota_b.get(), st);  // n of n: the identity
    DevBuf<int64_t> cnt(1, st);
    size_t tmp = 0;
    GTA_CUDA(cub::DeviceSelect::Flagged(nullptr, tmp, iota_b.get(), flags, out, cnt.get(), static_cast<int>(n), st));
    DevBuf<uint8_t> tb(tmp, st);
    GTA_CUDA(cub::DeviceSelect::Flagged(tb.get(), tmp, iota_b.get(), flags, out, cnt.get(), static_cast<int>(n), st));
    int64_t h = 0;
    GTA_CUDA(cudaMemcpyAsync(&h, cnt.get(), sizeof(int64_t), cudaMemcpyDeviceToHost, st));
    GTA_CUDA(cudaStreamSynchronize(st));
    return h;
}

void min_update(float* min_d, const float* d_new, int64_t n, cudaStream_t st)
{
    min_update_kernel<<<grid_of(n, 256), 256, 0, st>>>(min_d, d_new, n);
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

void balanced_assign(const int32_t* top2, const float* top2_d, int rule, const int32_t* cid, int32_t n_c, int64_t n,
                     int32_t* assign, int* err, cudaStream_t st)
{
    ProfScope prof("balanced_assign", 12.0 * static_cast<double>(n), st);
    GTA_REQUIRE(rule == 0 || (rule == 1 && top2_d), kInvalid, "balanced_assign: unknown rule");
    DevBuf<int32_t> sizes(static_cast<size_t>(n_c), st);
    DevBuf<uint8_t> is_c(static_cast<size_t>(n), st), not_c(static_cast<size_t>(n), st);
    GTA_CUDA(cudaMemsetAsync(is_c.get(), 0, static_cast<size_t>(n), st));
    centroid_self_assign_kernel<<<grid_of(n_c, 256), 256, 0, st>>>(cid, n_c, assign, is_c.get(), sizes.get());
    flag_not_kernel<<<grid_of(n, 256), 256, 0, st>>>(is_c.get(), n, not_c.get());
    count_launches(2);
    DevBuf<int32_t> nc_ids(static_cast<size_t>(n), st);
    const int64_t n_nc = select_flagged(not_c.get(), n, nc_ids.get(), st);
    const size_t smem = sizeof(int32_t) * static_cast<size_t>(n_c);
    if (smem <= 200u * 1024u) {
        GTA_CUDA(cudaFuncSetAttribute(balanced_assign_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(smem)));
        balanced_assign_kernel<true><<<1, 32, smem, st>>>(top2, top2_d, nc_ids.get(), n_nc, n_c, rule, sizes.get(),
                                                          assign, err);
    } else {
        balanced_assign_kernel<false><<<1, 32, 0, st>>>(top2, top2_d, nc_ids.get(), n_nc, n_c, rule, sizes.get(),
                                                        assign, err);
    }
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

void pool_fill(const int32_t* members, const int64_t* offsets, const int32_t* seg_b, const int64_t* seg_dst, int32_t S,
               int32_t c_lo, int32_t n_buckets, int32_t* pool_ids, cudaStream_t st)
{
    if (n_buckets <= 0) return;
    pool_fill_kernel<<<static_cast<unsigned>(static_cast<int64_t>(n_buckets) * S), 128, 0, st>>>(
        members, offsets, seg_b, seg_dst, S, c_lo, n_buckets, pool_ids);
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

void one_way_rows(const int32_t* members, int64_t n, int64_t* mem_row, cudaStream_t st)
{
    one_way_rows_kernel<<<grid_of(n, 256), 256, 0, st>>>(members, n, mem_row);
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

}  // namespace gta
