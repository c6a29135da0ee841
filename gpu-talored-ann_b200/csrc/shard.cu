// The sharded (multi-GPU) build's data movement on the device: which rows and lists a rank sends
// to which rank, packed into per-rank contiguous blocks for one all-to-all, and the tables the
// receiving side needs.  The reference's multi-GPU plan (bucketDemo/buildBucket/src/bucket.cu:
// row-sharded k-means, buckets on owner GPUs, points and lists exchanged, merge on the point's
// owner) sends the same data; here the packing is a stable multi-destination partition:
//
//   masks[i]    bit r set when item i goes to rank r (a membership goes to every rank holding a
//               piece of its bucket; a list row to the owner of its point, if this rank computed it)
//   partition   perm lists, rank by rank, the items carrying that rank's bit, each rank's items in
//               item order (block counts, a host prefix over (rank, block), then a scatter that
//               ranks items inside a block with warp ballots)
//   pack        one warp per sent item copies its payload (a dataset row, or a list row) and meta
//
// Every id read from the caller is range-checked; a bad one sets the device error flag (data
// check failed) and the item is dropped.
#include <algorithm>
#include <vector>

#include "common.cuh"
#include "gta_internal.h"
#include "prof.h"

namespace gta {

namespace {

constexpr int kPartThreads = 256;
constexpr int kPartItems = 2048;  // items per partition block
constexpr int kMaxRanks = 64;     // one bit per rank in a mask

unsigned blocks_for(int64_t n, int per) { return static_cast<unsigned>((n + per - 1) / per); }

__global__ void __launch_bounds__(kPartThreads)
    part_count_kernel(const uint64_t* __restrict__ masks, int64_t n, int world, int n_blk, int64_t* __restrict__ cnt)
{
    __shared__ int s_cnt[kMaxRanks];
    for (int r = threadIdx.x; r < world; r += blockDim.x) s_cnt[r] = 0;
    __syncthreads();
    const int64_t base = static_cast<int64_t>(blockIdx.x) * kPartItems;
    for (int k = threadIdx.x; k < kPartItems; k += blockDim.x) {
        const int64_t i = base + k;
        if (i >= n) break;
        uint64_t m = masks[i];
        while (m) {
            const int r = __ffsll(static_cast<long long>(m)) - 1;
            m &= m - 1;
            atomicAdd(&s_cnt[r], 1);
        }
    }
    __syncthreads();
    for (int r = threadIdx.x; r < world; r += blockDim.x) cnt[static_cast<int64_t>(r) * n_blk + blockIdx.x] = s_cnt[r];
}

// off[r * n_blk + b]: the first position of block b's items for rank r
__global__ void __launch_bounds__(kPartThreads)
    part_scatter_kernel(const uint64_t* __restrict__ masks, int64_t n, int world, int n_blk,
                        const int64_t* __restrict__ off, int64_t* __restrict__ perm)
{
    constexpr int kWarps = kPartThreads / 32;
    __shared__ int s_warp[kWarps][kMaxRanks];
    __shared__ int s_run[kMaxRanks];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const unsigned lt = (1u << lane) - 1u;
    for (int r = threadIdx.x; r < world; r += blockDim.x) s_run[r] = 0;
    const int64_t base = static_cast<int64_t>(blockIdx.x) * kPartItems;
    for (int c = 0; c < kPartItems; c += kPartThreads) {
        const int64_t i = base + c + threadIdx.x;
        const uint64_t m = i < n ? masks[i] : 0ull;
        for (int r = 0; r < world; ++r) {
            const unsigned b = __ballot_sync(0xffffffffu, (m >> r) & 1ull);
            if (lane == 0) s_warp[warp][r] = __popc(b);
        }
        __syncthreads();
        for (int r = 0; r < world; ++r) {
            const unsigned b = __ballot_sync(0xffffffffu, (m >> r) & 1ull);
            if ((m >> r) & 1ull) {
                int before = s_run[r];
                for (int w = 0; w < warp; ++w) before += s_warp[w][r];
                perm[off[static_cast<int64_t>(r) * n_blk + blockIdx.x] + before + __popc(b & lt)] = i;
            }
        }
        __syncthreads();
        for (int r = threadIdx.x; r < world; r += blockDim.x) {
            int t = 0;
            for (int w = 0; w < kWarps; ++w) t += s_warp[w][r];
            s_run[r] += t;
        }
        __syncthreads();
    }
}

// the grouped row's bucket: the last b with offsets[b] <= j
__device__ __forceinline__ int32_t bucket_of_row(const int64_t* __restrict__ offsets, int32_t B, int64_t j)
{
    int32_t lo = 0, hi = B - 1;
    while (lo < hi) {
        const int32_t mid = (lo + hi + 1) >> 1;
        if (offsets[mid] <= j) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

// membership m = 2p + s of local point p goes to every holder of its bucket top2[m]
__global__ void membership_masks_kernel(const int32_t* __restrict__ top2, int64_t n_mem, int32_t B,
                                        const uint64_t* __restrict__ holders, int world, uint64_t* __restrict__ masks,
                                        int* err)
{
    const int64_t m = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (m >= n_mem) return;
    const int32_t b = top2[m];
    uint64_t mk = 0;
    if (b >= 0 && b < B) mk = holders[b];
    const uint64_t valid = world == 64 ? ~0ull : ((1ull << world) - 1ull);
    if (mk == 0 || (mk & ~valid)) {  // no holder, or a holder past the last rank
        atomicCAS(err, 0, kDevBadIndex);
        mk = 0;
    }
    masks[m] = mk;
}

// grouped row j goes to the owner of its point when it lies in this rank's range of its bucket
__global__ void list_masks_kernel(const int32_t* __restrict__ order, const int32_t* __restrict__ gid, int64_t n_r,
                                  const int64_t* __restrict__ offsets, int32_t B, const int64_t* __restrict__ row_lo,
                                  const int64_t* __restrict__ row_hi, const int64_t* __restrict__ starts, int world,
                                  uint64_t* __restrict__ masks, int* err)
{
    const int64_t j = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (j >= n_r) return;
    const int32_t b = bucket_of_row(offsets, B, j);
    const int64_t rel = j - offsets[b];
    uint64_t mk = 0;
    if (rel >= row_lo[b] && rel < row_hi[b]) {
        const int32_t o = order[j];
        const int64_t g = (o >= 0 && o < n_r) ? gid[o] : -1;
        if (g < starts[0] || g >= starts[world]) {
            atomicCAS(err, 0, kDevBadIndex);
        } else {
            int r = 0;
            while (r + 1 < world && starts[r + 1] <= g) ++r;
            mk = 1ull << r;
        }
    }
    masks[j] = mk;
}

__device__ __forceinline__ void copy_row(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int64_t bytes,
                                         int lane)
{
    const bool v16 = ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) | bytes) & 15) == 0;
    if (v16) {
        const uint4* s = reinterpret_cast<const uint4*>(src);
        uint4* d = reinterpret_cast<uint4*>(dst);
        for (int64_t k = lane; k < bytes / 16; k += 32) d[k] = s[k];
    } else {
        for (int64_t k = lane; k < bytes; k += 32) dst[k] = src[k];
    }
}

__global__ void pack_memberships_kernel(const int64_t* __restrict__ perm, int64_t total, const uint8_t* __restrict__ X,
                                        int64_t row_bytes, int64_t row0, const int32_t* __restrict__ top2,
                                        uint8_t* __restrict__ send_rows, int32_t* __restrict__ send_meta)
{
    const int64_t pos = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (pos >= total) return;
    const int64_t m = perm[pos];
    const int64_t p = m >> 1;
    copy_row(X + p * row_bytes, send_rows + pos * row_bytes, row_bytes, lane);
    if (lane == 0) {
        send_meta[3 * pos] = static_cast<int32_t>(row0 + p);
        send_meta[3 * pos + 1] = top2[m];
        send_meta[3 * pos + 2] = top2[m ^ 1];
    }
}

__global__ void pack_lists_kernel(const int64_t* __restrict__ perm, int64_t total, const int32_t* __restrict__ lid,
                                  const float* __restrict__ ldist, int32_t M, const int32_t* __restrict__ order,
                                  const int32_t* __restrict__ gid, const int64_t* __restrict__ offsets, int32_t B,
                                  int32_t* __restrict__ send_ids, float* __restrict__ send_dists,
                                  int32_t* __restrict__ send_meta)
{
    const int64_t pos = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (pos >= total) return;
    const int64_t j = perm[pos];
    for (int t = lane; t < M; t += 32) {
        send_ids[pos * M + t] = lid[j * M + t];
        send_dists[pos * M + t] = ldist[j * M + t];
    }
    if (lane == 0) {
        send_meta[2 * pos] = gid[order[j]];
        send_meta[2 * pos + 1] = bucket_of_row(offsets, B, j);
    }
}

// mem_row[2p + slot] = i for received list i of local point p: slot 0 for the lower of the
// point's two buckets
__global__ void member_rows_kernel(const int32_t* __restrict__ meta, int64_t n_b, int64_t row0, int64_t n_local,
                                   const int32_t* __restrict__ top2, int64_t* __restrict__ mem_row, int* err)
{
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n_b) return;
    const int64_t p = static_cast<int64_t>(meta[2 * i]) - row0;
    const int32_t b = meta[2 * i + 1];
    if (p < 0 || p >= n_local) {
        atomicCAS(err, 0, kDevBadIndex);
        return;
    }
    const int32_t t0 = top2[2 * p], t1 = top2[2 * p + 1];
    if (b != t0 && b != t1) {
        atomicCAS(err, 0, kDevBadIndex);
        return;
    }
    mem_row[2 * p + (b != min(t0, t1) ? 1 : 0)] = i;
}

// seed[gid] = the M-th distance of each computed row whose bucket is the lower of its point's two
__global__ void lower_seeds_kernel(const float* __restrict__ ldist, int32_t M, int64_t n_r,
                                   const int32_t* __restrict__ order, const int32_t* __restrict__ gid,
                                   const int64_t* __restrict__ offsets, const int32_t* __restrict__ partner, int32_t B,
                                   const int64_t* __restrict__ row_lo, const int64_t* __restrict__ row_hi, int64_t N,
                                   float* __restrict__ seed, int* err)
{
    const int64_t j = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (j >= n_r) return;
    const int32_t b = bucket_of_row(offsets, B, j);
    const int64_t rel = j - offsets[b];
    if (rel < row_lo[b] || rel >= row_hi[b] || partner[j] <= b) return;
    const int32_t o = order[j];
    const int64_t g = (o >= 0 && o < n_r) ? gid[o] : -1;
    if (g < 0 || g >= N) {
        atomicCAS(err, 0, kDevBadIndex);
        return;
    }
    seed[g] = ldist[j * M + M - 1];
}

__global__ void fill_kernel(float* __restrict__ p, int64_t n, float v)
{
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) p[i] = v;
}

}  // namespace

void stable_partition(const uint64_t* masks, int64_t n, int world, DevBuf<int64_t>& perm, std::vector<int64_t>& counts,
                      cudaStream_t st)
{
    GTA_REQUIRE(world >= 1 && world <= kMaxRanks, kInvalid, "partition: 1 to 64 ranks");
    counts.assign(static_cast<size_t>(world), 0);
    if (n == 0) return;
    const int n_blk = static_cast<int>(blocks_for(n, kPartItems));
    DevBuf<int64_t> cnt(static_cast<size_t>(world) * n_blk, st);
    part_count_kernel<<<n_blk, kPartThreads, 0, st>>>(masks, n, world, n_blk, cnt.get());
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
    std::vector<int64_t> h(static_cast<size_t>(world) * n_blk);
    GTA_CUDA(cudaMemcpyAsync(h.data(), cnt.get(), sizeof(int64_t) * h.size(), cudaMemcpyDeviceToHost, st));
    GTA_CUDA(cudaStreamSynchronize(st));
    int64_t acc = 0;
    for (int r = 0; r < world; ++r) {
        const int64_t start = acc;
        for (int b = 0; b < n_blk; ++b) {
            const int64_t c = h[static_cast<size_t>(r) * n_blk + b];
            h[static_cast<size_t>(r) * n_blk + b] = acc;
            acc += c;
        }
        counts[static_cast<size_t>(r)] = acc - start;
    }
    perm = DevBuf<int64_t>(static_cast<size_t>(std::max<int64_t>(acc, 1)), st);
    if (acc == 0) return;
    GTA_CUDA(cudaMemcpyAsync(cnt.get(), h.data(), sizeof(int64_t) * h.size(), cudaMemcpyHostToDevice, st));
    // (a pageable source: the copy is staged before cudaMemcpyAsync returns)
    part_scatter_kernel<<<n_blk, kPartThreads, 0, st>>>(masks, n, world, n_blk, cnt.get(), perm.get());
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

void shard_pack_memberships(const ShardPackMem& a, std::vector<int64_t>& counts, cudaStream_t st)
{
    const int64_t n_mem = 2 * a.n_local;
    DevBuf<uint64_t> masks(static_cast<size_t>(std::max<int64_t>(n_mem, 1)), st);
    DevBuf<int64_t> perm;
    if (n_mem > 0) {
        ProfScope prof("shard_pack", 8.0 * static_cast<double>(n_mem), st);
        membership_masks_kernel<<<blocks_for(n_mem, 256), 256, 0, st>>>(a.top2, n_mem, a.B, a.holders, a.world,
                                                                         masks.get(), a.err);
        count_launches(1);
        GTA_CUDA(cudaGetLastError());
    }
    stable_partition(masks.get(), n_mem, a.world, perm, counts, st);
    if (!a.send_rows) return;
    int64_t total = 0;
    for (int64_t c : counts) total += c;
    GTA_REQUIRE(total <= a.capacity, kInvalid, "shard_pack_memberships: send buffers too small");
    if (total == 0) return;
    ProfScope prof("shard_pack", static_cast<double>(total) * (2.0 * a.row_bytes + 12.0), st);
    pack_memberships_kernel<<<blocks_for(total * 32, 256), 256, 0, st>>>(
        perm.get(), total, static_cast<const uint8_t*>(a.X), a.row_bytes, a.row0, a.top2,
        static_cast<uint8_t*>(a.send_rows), a.send_meta);
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

void shard_pack_lists(const ShardPackLists& a, std::vector<int64_t>& counts, cudaStream_t st)
{
    DevBuf<uint64_t> masks(static_cast<size_t>(std::max<int64_t>(a.n_r, 1)), st);
    DevBuf<int64_t> lo(static_cast<size_t>(a.B), st), hi(static_cast<size_t>(a.B), st),
        starts(static_cast<size_t>(a.world) + 1, st);
    GTA_CUDA(cudaMemcpyAsync(lo.get(), a.row_lo, sizeof(int64_t) * a.B, cudaMemcpyHostToDevice, st));
    GTA_CUDA(cudaMemcpyAsync(hi.get(), a.row_hi, sizeof(int64_t) * a.B, cudaMemcpyHostToDevice, st));
    GTA_CUDA(cudaMemcpyAsync(starts.get(), a.starts, sizeof(int64_t) * (a.world + 1), cudaMemcpyHostToDevice, st));
    DevBuf<int64_t> perm;
    if (a.n_r > 0) {
        list_masks_kernel<<<blocks_for(a.n_r, 256), 256, 0, st>>>(a.order, a.gid, a.n_r, a.offsets, a.B, lo.get(),
                                                                   hi.get(), starts.get(), a.world, masks.get(), a.err);
        count_launches(1);
        GTA_CUDA(cudaGetLastError());
    }
    stable_partition(masks.get(), a.n_r, a.world, perm, counts, st);
    if (!a.send_ids) return;
    int64_t total = 0;
    for (int64_t c : counts) total += c;
    GTA_REQUIRE(total <= a.capacity, kInvalid, "shard_pack_lists: send buffers too small");
    if (total == 0) return;
    ProfScope prof("shard_pack", static_cast<double>(total) * (16.0 * a.M + 16.0), st);
    pack_lists_kernel<<<blocks_for(total * 32, 256), 256, 0, st>>>(perm.get(), total, a.lid, a.ldist, a.M, a.order,
                                                                   a.gid, a.offsets, a.B, a.send_ids, a.send_dists,
                                                                   a.send_meta);
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

void shard_member_rows(const int32_t* meta, int64_t n_b, int64_t row0, int64_t n_local, const int32_t* top2,
                       int64_t* mem_row, int* err, cudaStream_t st)
{
    GTA_CUDA(cudaMemsetAsync(mem_row, 0xFF, sizeof(int64_t) * 2 * static_cast<size_t>(n_local), st));
    if (n_b == 0) return;
    member_rows_kernel<<<blocks_for(n_b, 256), 256, 0, st>>>(meta, n_b, row0, n_local, top2, mem_row, err);
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

void shard_lower_seeds(const float* ldist, int32_t M, int64_t n_r, const int32_t* order, const int32_t* gid,
                       const int64_t* offsets, const int32_t* partner, int32_t B, const int64_t* row_lo_h,
                       const int64_t* row_hi_h, int64_t N, float* seed, int* err, cudaStream_t st)
{
    if (N > 0) {
        fill_kernel<<<blocks_for(N, 256), 256, 0, st>>>(seed, N, INFINITY);
        count_launches(1);
        GTA_CUDA(cudaGetLastError());
    }
    if (n_r == 0) return;
    DevBuf<int64_t> lo(static_cast<size_t>(B), st), hi(static_cast<size_t>(B), st);
    GTA_CUDA(cudaMemcpyAsync(lo.get(), row_lo_h, sizeof(int64_t) * B, cudaMemcpyHostToDevice, st));
    GTA_CUDA(cudaMemcpyAsync(hi.get(), row_hi_h, sizeof(int64_t) * B, cudaMemcpyHostToDevice, st));
    lower_seeds_kernel<<<blocks_for(n_r, 256), 256, 0, st>>>(ldist, M, n_r, order, gid, offsets, partner, B, lo.get(),
                                                             hi.get(), N, seed, err);
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

}  // namespace gta
