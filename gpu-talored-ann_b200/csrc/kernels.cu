// kernels.cu -- the integer / byte kernels of the bucketed kNN + CAGRA build.
//
// All of them are HBM- or latency-bound; none is reshaped into a GEMM.
// Reference behaviour (paths relative to the reference root):
//   merge_memberships  bucketDemo/buildBucket/src/bucket.cu:5025-5131 resident_merge(_warp)_kernel
//   sanitize           bucketDemo/buildBucket/src/optimize.cu:95-133
//   prune_detour       bucketDemo/buildBucket/src/prune_windowed_core.hpp:190-263 (full window),
//                      prune_windowed_gpu.cu:178-330 (warp per point, id->rank hash, detour stamp)
//   reverse_merge      bucketDemo/buildBucket/src/edge_chunk_accumulator.hpp:386-494,
//                      optimize_chunked.cu:372 kern_scatter_rank / :1450 kern_e_merge
//   sort_rows_l2       bucketDemo/buildBucket/src/prune_windowed_core.hpp:134-175
//   centroid_update    bucketDemo/build_bucket.py:255-261
//   kmeanspp_init      bucketDemo/build_bucket.py:189-229 (D^2 sampling on a pool of min(N, 20B))
#include <cub/cub.cuh>
#include <cuda_bf16.h>

#include <cmath>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "gta_internal.h"
#include "prof.h"

namespace gta {

namespace {

constexpr uint32_t kEmpty = 0xFFFFFFFFu;

__device__ __forceinline__ uint64_t splitmix64(uint64_t x)
{
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ double uniform01(uint64_t seed, uint64_t t)
{
    return static_cast<double>(splitmix64(seed * 0x2545F4914F6CDD1Dull + t) >> 11) * (1.0 / 9007199254740992.0);
}

template <typename T> __device__ __forceinline__ float ld_f32(const T* p) { return static_cast<float>(*p); }
template <> __device__ __forceinline__ float ld_f32<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }

template <typename Tout> __device__ __forceinline__ Tout from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
// 8-bit operand rows: the values are the dataset's own bytes (0 .. 255), held exactly
template <> __device__ __forceinline__ uint8_t from_f32<uint8_t>(float v) { return static_cast<uint8_t>(v); }

__device__ __forceinline__ float exact_l2_f(const float* __restrict__ a, const float* __restrict__ b, int d)
{
    float acc = 0.0f;
    for (int i = 0; i < d; ++i) {
        const float t = a[i] - b[i];
        acc = fmaf(t, t, acc);
    }
    return acc;
}

// ---------------------------------------------------------------- conversion
// four consecutive elements as f32 (the caller guarantees the alignment of the access)
__device__ __forceinline__ void load4_f32(const float* p, float (&v)[4])
{
    const float4 q = *reinterpret_cast<const float4*>(p);
    v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
}
__device__ __forceinline__ void load4_f32(const uint8_t* p, float (&v)[4])
{
    const uchar4 q = *reinterpret_cast<const uchar4*>(p);
    v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
}
__device__ __forceinline__ void load4_f32(const int8_t* p, float (&v)[4])
{
    const char4 q = *reinterpret_cast<const char4*>(p);
    v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
}
__device__ __forceinline__ void load4_f32(const __nv_bfloat16* p, float (&v)[4])
{
    for (int u = 0; u < 4; ++u) v[u] = __bfloat162float(p[u]);
}
__device__ __forceinline__ void store4_from_f32(float* p, const float (&v)[4])
{
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}
__device__ __forceinline__ void store4_from_f32(uint8_t* p, const float (&v)[4])
{
    *reinterpret_cast<uchar4*>(p) = make_uchar4(static_cast<uint8_t>(v[0]), static_cast<uint8_t>(v[1]),
                                                static_cast<uint8_t>(v[2]), static_cast<uint8_t>(v[3]));
}
__device__ __forceinline__ void store4_from_f32(__nv_bfloat16* p, const float (&v)[4])
{
    __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]), b = __floats2bfloat162_rn(v[2], v[3]);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t*>(&a);
    u.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = u;
}

template <typename Tin, typename Tout>
__global__ void convert_rows_kernel(const Tin* __restrict__ X, int d, const int32_t* __restrict__ row_ids,
                                    int64_t n_out, Tout* __restrict__ out, int d_pad, float* __restrict__ norms, int vec4)
{
    const int lane = threadIdx.x & 31;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= n_out) return;
    const int64_t src = row_ids ? static_cast<int64_t>(row_ids[row]) : row;
    const Tin* x = X + src * d;
    Tout* o = out ? out + row * d_pad : nullptr;
    // squared norm: per-lane fma chains, then a butterfly sum (exact for 8-bit rows, where every
    // partial sum is an integer below 2^24)
    float acc = 0.0f;
    if (vec4) {  // d % 4 == 0, rows 4-element aligned: four elements per lane and access
        for (int g = lane; 4 * g < d_pad; g += 32) {
            float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            if (4 * g < d) load4_f32(x + 4 * g, v);
#pragma unroll
            for (int u = 0; u < 4; ++u) acc = fmaf(v[u], v[u], acc);
            if (o) store4_from_f32(o + 4 * g, v);
        }
    } else {
        for (int i = lane; i < d_pad; i += 32) {
            const float v = i < d ? ld_f32(x + i) : 0.0f;
            acc = fmaf(v, v, acc);
            if (o) o[i] = from_f32<Tout>(v);
        }
    }
    if (norms) {
#pragma unroll
        for (int m = 16; m > 0; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
        if (lane == 0) norms[row] = acc;
    }
}

template <typename Tin>
void convert_dispatch_out(const Tin* X, int d, const int32_t* ids, int64_t n, void* out, int out_elem, int d_pad,
                          float* norms, cudaStream_t st)
{
    const int wpb = 8;
    const unsigned grid = static_cast<unsigned>((n + wpb - 1) / wpb);
    const size_t in_align = sizeof(Tin) * 4, out_align = static_cast<size_t>(elem_bytes(out_elem)) * 4;
    const int vec4 = (d % 4 == 0) && (d_pad % 4 == 0) && (reinterpret_cast<uintptr_t>(X) % in_align == 0) &&
                     (reinterpret_cast<uintptr_t>(out) % out_align == 0);
    if (out_elem == kElemU8) {
        GTA_REQUIRE(sizeof(Tin) == 1 && static_cast<Tin>(-1) > 0, kInvalid, "convert_rows: 8-bit operand rows need u8 data");
        convert_rows_kernel<Tin, uint8_t><<<grid, wpb * 32, 0, st>>>(X, d, ids, n, static_cast<uint8_t*>(out), d_pad,
                                                                      norms, vec4);
    } else if (out_elem == kElemBF16)
        convert_rows_kernel<Tin, __nv_bfloat16><<<grid, wpb * 32, 0, st>>>(X, d, ids, n,
                                                                            static_cast<__nv_bfloat16*>(out), d_pad, norms,
                                                                            vec4);
    else
        convert_rows_kernel<Tin, float><<<grid, wpb * 32, 0, st>>>(X, d, ids, n, static_cast<float*>(out), d_pad, norms,
                                                                    vec4);
    count_launches(1);
}

// Rows of a shard holding global rows [row0, row0 + n): out[j] = X[ids[j] - row0]
// as f32 (d columns), a zero row where ids[j] lies outside the shard.
template <typename Tin>
__global__ void gather_range_kernel(const Tin* __restrict__ X, int d, int64_t row0, int64_t n,
                                    const int32_t* __restrict__ ids, int64_t n_ids, float* __restrict__ out)
{
    const int lane = threadIdx.x & 31;
    const int64_t j = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (j >= n_ids) return;
    const int64_t src = static_cast<int64_t>(ids[j]) - row0;
    const bool in = src >= 0 && src < n;
    const Tin* x = X + (in ? src : 0) * d;
    float* o = out + j * d;
    for (int i = lane; i < d; i += 32) o[i] = in ? ld_f32(x + i) : 0.0f;
}

__global__ void gather_i32_kernel(const int32_t* __restrict__ src, const int32_t* __restrict__ idx, int64_t n,
                                  int32_t* __restrict__ out)
{
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) out[i] = src[idx[i]];
}

// ---------------------------------------------------------------- sampling
__global__ void sample_ids_kernel(int64_t N, int64_t n_s, uint64_t seed, int32_t* out)
{
    const int64_t j = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (j >= n_s) return;
    const int64_t lo = (j * N) / n_s, hi = ((j + 1) * N) / n_s;
    const uint64_t h = splitmix64((seed * 0x100000001B3ull) ^ static_cast<uint64_t>(j));
    out[j] = static_cast<int32_t>(lo + static_cast<int64_t>(h % static_cast<uint64_t>(hi - lo)));
}

// ---------------------------------------------------------------- k-means++
constexpr int kKppThreads = 256;

__global__ void kpp_first_kernel(const float* __restrict__ pool, int64_t pool_n, int d_pad, uint64_t seed,
                                 float* __restrict__ C)
{
    const int64_t i = static_cast<int64_t>(uniform01(seed, 0) * static_cast<double>(pool_n));
    const int64_t c = i < pool_n ? i : pool_n - 1;
    for (int k = threadIdx.x; k < d_pad; k += blockDim.x) C[k] = pool[c * d_pad + k];
}

// One D^2-sampling step: fold centroid t into min_d2, then the last block to
// finish draws centroid t+1 with probability proportional to min_d2.  Every
// block sums its chunk as 256 contiguous per-thread runs combined in thread
// order, and the draw repeats exactly that order inside the chosen block, so
// the pick is reproducible run to run.
__device__ __forceinline__ double kpp_run_sum(const float* __restrict__ v, int64_t a, int64_t b)
{
    double s = 0.0;
    for (int64_t i = a; i < b; ++i) s += static_cast<double>(v[i]);
    return s;
}

__global__ void __launch_bounds__(kKppThreads) kpp_step_kernel(const float* __restrict__ pool, int64_t pool_n, int d,
                                                               int d_pad, float* __restrict__ C, int t, int B,
                                                               float* __restrict__ min_d2, double* __restrict__ bsum,
                                                               unsigned* __restrict__ counter, uint64_t seed, int64_t chunk)
{
    extern __shared__ float cen[];
    __shared__ double part[kKppThreads];
    __shared__ bool last;
    __shared__ int s_blk;
    __shared__ double s_resid;
    __shared__ int64_t s_pick;
    const int tid = threadIdx.x;
    for (int k = tid; k < d; k += blockDim.x) cen[k] = C[static_cast<int64_t>(t) * d_pad + k];
    __syncthreads();
    const int64_t lo = static_cast<int64_t>(blockIdx.x) * chunk;
    const int64_t hi = min(pool_n, lo + chunk);
    for (int64_t i = lo + tid; i < hi; i += blockDim.x) {
        const float dd = exact_l2_f(pool + i * d_pad, cen, d);
        min_d2[i] = (t == 0) ? dd : fminf(min_d2[i], dd);
    }
    __syncthreads();
    const int64_t per = (hi - lo + kKppThreads - 1) / kKppThreads;
    {
        const int64_t a = min(hi, lo + tid * per), e = min(hi, a + per);
        part[tid] = kpp_run_sum(min_d2, a, e);
    }
    __syncthreads();
    if (tid == 0) {
        double s = 0.0;
        for (int w = 0; w < kKppThreads; ++w) s += part[w];
        bsum[blockIdx.x] = s;
        __threadfence();
        last = (atomicAdd(counter, 1u) == gridDim.x - 1);
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (tid == 0) {
        *counter = 0;
        s_blk = -1;
        if (t + 1 < B) {
            double total = 0.0;
            for (unsigned b = 0; b < gridDim.x; ++b) total += bsum[b];
            const double u = uniform01(seed, static_cast<uint64_t>(t) + 1);
            s_pick = min(pool_n - 1, static_cast<int64_t>(u * static_cast<double>(pool_n)));
            s_blk = -2;
            if (total > 0.0) {
                const double target = u * total;
                double cum = 0.0;
                unsigned b = 0;
                for (; b + 1 < gridDim.x; ++b) {
                    if (cum + bsum[b] > target) break;
                    cum += bsum[b];
                }
                s_blk = static_cast<int>(b);
                s_resid = target - cum;
            }
        }
    }
    __syncthreads();
    if (s_blk == -1) return;
    if (s_blk >= 0) {
        const int64_t lo2 = static_cast<int64_t>(s_blk) * chunk, hi2 = min(pool_n, lo2 + chunk);
        const int64_t per2 = (hi2 - lo2 + kKppThreads - 1) / kKppThreads;
        {
            const int64_t a = min(hi2, lo2 + tid * per2), e = min(hi2, a + per2);
            part[tid] = kpp_run_sum(min_d2, a, e);
        }
        __syncthreads();
        if (tid == 0) {
            double cum = 0.0;
            int w = 0;
            for (; w + 1 < kKppThreads; ++w) {
                if (cum + part[w] > s_resid) break;
                cum += part[w];
            }
            const int64_t a = min(hi2, lo2 + w * per2), e = min(hi2, a + per2);
            int64_t pick = (e > a) ? e - 1 : hi2 - 1;
            for (int64_t i = a; i < e; ++i) {
                cum += static_cast<double>(min_d2[i]);
                if (cum > s_resid) { pick = i; break; }
            }
            s_pick = pick;
        }
    }
    __syncthreads();
    const int64_t pick = s_pick;
    for (int k = tid; k < d_pad; k += blockDim.x) C[static_cast<int64_t>(t + 1) * d_pad + k] = pool[pick * d_pad + k];
}

// The whole D^2 sampling in one cooperative launch: one thread per pool point,
// every CTA co-resident, a bounded grid barrier per centroid instead of a
// kernel launch.  Step t folds centroid t into each point's min distance
// (kept in a register), each CTA writes the fp64 inclusive prefix of its
// points' weights and its total, and after the barrier every CTA draws the
// same centroid t+1: the CTA whose cumulative total first exceeds u * total,
// then the point whose prefix first exceeds the remainder.  Sums are fixed-order
// scans, so the picks are reproducible run to run and on every GPU.
constexpr int kKppCoopThreads = 256;

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p)
{
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Grid barrier of a cooperative launch; gives up after the wait budget and
// raises the abort flag that every CTA polls.  Returns false on abort.
__device__ bool coop_barrier(unsigned* arrive, unsigned target, int* abort_flag, int* err, int* s_ok)
{
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(arrive, 1u);
        const long long t0 = clock64();
        int ok = 1;
        for (uint32_t it = 0; ld_acquire_u32(arrive) < target; ++it) {
            if ((it & 15u) != 15u) continue;  // poll hot; check abort and the budget every 16 polls
            if (*reinterpret_cast<volatile int*>(abort_flag)) { ok = 0; break; }
            if (clock64() - t0 > kWaitBudgetCycles) {
                atomicExch(abort_flag, 1);
                if (err) atomicCAS(err, 0, kDevTimeoutGrid);
                ok = 0;
                break;
            }
        }
        __threadfence();
        *s_ok = ok;
    }
    __syncthreads();
    return *s_ok != 0;
}

// Inclusive fp64 prefix sum over the CTA's threads (fixed order).
__device__ __forceinline__ double block_incl_scan(double v, double* s_warp)
{
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const double u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
    }
    if (lane == 31) s_warp[w] = v;
    __syncthreads();
    if (w == 0) {
        double t = lane < (kKppCoopThreads / 32) ? s_warp[lane] : 0.0;
#pragma unroll
        for (int o = 1; o < kKppCoopThreads / 32; o <<= 1) {
            const double u = __shfl_up_sync(0xffffffffu, t, o);
            if (lane >= o) t += u;
        }
        if (lane < kKppCoopThreads / 32) s_warp[lane] = t;
    }
    __syncthreads();
    const double off = w > 0 ? s_warp[w - 1] : 0.0;
    __syncthreads();
    return v + off;
}

// With `resident` 1, each CTA keeps its 256 pool rows in shared memory, transposed
// (dimension-major, so thread t reads column t without bank conflicts).  With `resident` 2
// (rows too long for that), the rows pass through shared memory kKppDims dimensions at a time,
// transposed the same way (row stride kKppStride: conflict-free both ways), every warp loading
// 32 rows' slices with coalesced loads; each thread's chain still runs over the dimensions in
// ascending order, so the distances are those of exact_l2_f bit for bit.
constexpr int kKppDims = 64;
constexpr int kKppStride = kKppCoopThreads + 1;

__global__ void __launch_bounds__(kKppCoopThreads)
    kpp_coop_kernel(const float* __restrict__ pool, int64_t pool_n, int d, int d_pad, float* __restrict__ C, int B,
                    uint64_t seed, double* __restrict__ gpre, double* __restrict__ gtot, unsigned* arrive,
                    int* abort_flag, int* err, int resident)
{
    extern __shared__ float cen[];
    float* rows_t = cen + d_pad;  // resident: [d][256]
    __shared__ double s_warp[kKppCoopThreads / 32];
    __shared__ int64_t s_pick;
    __shared__ int s_blk, s_ok;
    __shared__ double s_resid;
    const int tid = threadIdx.x;
    const int G = gridDim.x;
    const int64_t i = static_cast<int64_t>(blockIdx.x) * kKppCoopThreads + tid;
    const bool valid = i < pool_n;
    float md = INFINITY;
    if (resident == 1)
        for (int k = 0; k < d; ++k) rows_t[k * kKppCoopThreads + tid] = valid ? pool[i * d_pad + k] : 0.0f;
    if (tid == 0) {
        const int64_t f = static_cast<int64_t>(uniform01(seed, 0) * static_cast<double>(pool_n));
        s_pick = f < pool_n ? f : pool_n - 1;
    }
    for (int t = 0; t < B; ++t) {
        __syncthreads();
        const int64_t pick = s_pick;
        for (int k = tid; k < d; k += kKppCoopThreads) cen[k] = pool[pick * d_pad + k];
        if (blockIdx.x == 0)
            for (int k = tid; k < d_pad; k += kKppCoopThreads)
                C[static_cast<int64_t>(t) * d_pad + k] = pool[pick * d_pad + k];
        __syncthreads();
        if (t + 1 >= B) break;
        if (valid) {
            float dd;
            if (resident == 1) {  // the same fp32 chain as exact_l2_f, operands from shared memory
                dd = 0.0f;
                for (int k = 0; k < d; ++k) {
                    const float t = rows_t[k * kKppCoopThreads + tid] - cen[k];
                    dd = fmaf(t, t, dd);
                }
                md = fminf(md, dd);
            } else if (resident == 0) {
                dd = exact_l2_f(pool + i * d_pad, cen, d);
                md = fminf(md, dd);
            }
        }
        if (resident == 2) {
            // every thread of the CTA stages (the barriers below), the valid ones add
            const int warp = tid >> 5, lane = tid & 31;
            float dd = 0.0f;
            for (int k0 = 0; k0 < d; k0 += kKppDims) {
                const int nk = d - k0 < kKppDims ? d - k0 : kKppDims;
#pragma unroll 8
                for (int p = 0; p < 32; ++p) {
                    const int col = warp * 32 + p;  // this CTA's point
                    const int64_t ip = static_cast<int64_t>(blockIdx.x) * kKppCoopThreads + col;
                    const float* src = pool + (ip < pool_n ? ip : 0) * d_pad + k0;
                    const float v0 = (ip < pool_n && lane < nk) ? src[lane] : 0.0f;
                    const float v1 = (ip < pool_n && lane + 32 < nk) ? src[lane + 32] : 0.0f;
                    rows_t[lane * kKppStride + col] = v0;
                    rows_t[(lane + 32) * kKppStride + col] = v1;
                }
                __syncthreads();
                if (valid) {
                    for (int c = 0; c < nk; ++c) {
                        const float t = rows_t[c * kKppStride + tid] - cen[k0 + c];
                        dd = fmaf(t, t, dd);
                    }
                }
                __syncthreads();
            }
            if (valid) md = fminf(md, dd);
        }
        const double incl = block_incl_scan(valid ? static_cast<double>(md) : 0.0, s_warp);
        const int par = t & 1;
        gpre[static_cast<int64_t>(par) * G * kKppCoopThreads + static_cast<int64_t>(blockIdx.x) * kKppCoopThreads + tid] = incl;
        if (tid == kKppCoopThreads - 1) gtot[par * G + blockIdx.x] = incl;
        if (!coop_barrier(arrive, static_cast<unsigned>(t + 1) * static_cast<unsigned>(G), abort_flag, err, &s_ok)) return;
        // the draw, identical in every CTA: first the CTA, then the point inside it
        const double u = uniform01(seed, static_cast<uint64_t>(t) + 1);
        const double tot_b = tid < G ? __ldcg(gtot + par * G + tid) : 0.0;
        const double cum_b = block_incl_scan(tot_b, s_warp);
        if (tid == kKppCoopThreads - 1) {
            s_resid = cum_b;  // the grand total (threads past G add zeros)
            s_blk = -1;
        }
        __syncthreads();
        const double total = s_resid;
        const double target = u * total;
        __syncthreads();
        if (total > 0.0 && tid < G && cum_b > target && (tid == 0 || cum_b - tot_b <= target)) {
            s_blk = tid;
            s_resid = target - (cum_b - tot_b);
        }
        if (tid == 0 && !(total > 0.0)) s_pick = min(pool_n - 1, static_cast<int64_t>(u * static_cast<double>(pool_n)));
        __syncthreads();
        const int blk = s_blk;
        if (total > 0.0) {
            if (blk < 0) {
                // rounding left the target past every cumulative total: the last CTA
                if (tid == 0) { s_blk = G - 1; s_resid = 0.0; }
                __syncthreads();
            }
            const int b = s_blk;
            const double resid = s_resid;
            const int64_t j = static_cast<int64_t>(b) * kKppCoopThreads + tid;
            const int64_t rem = pool_n - static_cast<int64_t>(b) * kKppCoopThreads;
            const int cnt = static_cast<int>(rem < kKppCoopThreads ? rem : kKppCoopThreads);
            const double pre = tid < cnt ? __ldcg(gpre + static_cast<int64_t>(par) * G * kKppCoopThreads + j) : 0.0;
            const double prev = (tid > 0 && tid < cnt) ? __ldcg(gpre + static_cast<int64_t>(par) * G * kKppCoopThreads + j - 1)
                                                       : 0.0;
            if (tid == 0) s_pick = static_cast<int64_t>(b) * kKppCoopThreads + cnt - 1;  // fallback: the CTA's last point
            __syncthreads();
            if (tid < cnt && pre > resid && (tid == 0 || prev <= resid)) s_pick = j;
        }
    }
}

// ---------------------------------------------------------------- Lloyd update
__global__ void seg_offsets_kernel(const int32_t* __restrict__ keys_sorted, int64_t n, int32_t B,
                                   int64_t* __restrict__ offsets)
{
    const int64_t b = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (b > B) return;
    int64_t lo = 0, hi = n;  // first index with key >= b
    while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if (keys_sorted[mid] < b) lo = mid + 1;
        else hi = mid;
    }
    offsets[b] = lo;
}

// One thread per (centroid, dimension): the members' values added in ascending member order in
// fp64, then divided by the count (the oracle's rule, bit for bit).  The chain of a large centroid
// is long (C3: tens of thousands of members), so a thread keeps loads in flight ahead of its
// additions: the values of the next kSumBatch members (their ids already in registers) and the
// ids of the batch after that are issued before the current batch is added.
constexpr int kSumBatch = 32;

__global__ void __launch_bounds__(128)
    centroid_sum_kernel(const float* __restrict__ Xs, int d, int d_pad, const int32_t* __restrict__ order,
                        const int64_t* __restrict__ offsets, const float* __restrict__ C_in, float* __restrict__ C_out)
{
    const int b = blockIdx.x;
    const int k = static_cast<int>(blockIdx.y) * blockDim.x + threadIdx.x;
    if (k >= d_pad) return;
    const int64_t lo = offsets[b], hi = offsets[b + 1];
    const int64_t cnt = hi - lo;
    const int64_t o = static_cast<int64_t>(b) * d_pad + k;
    if (k >= d) {
        C_out[o] = 0.0f;
        return;
    }
    if (cnt == 0) {
        C_out[o] = C_in[o];
        return;
    }
    double s = 0.0;
    int64_t j = lo;
    const int64_t end_full = lo + cnt / kSumBatch * kSumBatch;  // members in whole batches
    if (end_full > lo) {
        int32_t ids[kSumBatch];  // the ids of the batch whose values are loaded next
        float cur[kSumBatch];    // the values of the batch added next
#pragma unroll
        for (int u = 0; u < kSumBatch; ++u) ids[u] = order[lo + u];
#pragma unroll
        for (int u = 0; u < kSumBatch; ++u) cur[u] = Xs[static_cast<int64_t>(ids[u]) * d_pad + k];
        if (lo + kSumBatch < end_full) {
#pragma unroll
            for (int u = 0; u < kSumBatch; ++u) ids[u] = order[lo + kSumBatch + u];
        }
        for (; j + kSumBatch < end_full; j += kSumBatch) {
            float nxt[kSumBatch];  // the batch starting at j + kSumBatch
#pragma unroll
            for (int u = 0; u < kSumBatch; ++u) nxt[u] = Xs[static_cast<int64_t>(ids[u]) * d_pad + k];
            if (j + 2 * kSumBatch < end_full) {
#pragma unroll
                for (int u = 0; u < kSumBatch; ++u) ids[u] = order[j + 2 * kSumBatch + u];
            }
#pragma unroll
            for (int u = 0; u < kSumBatch; ++u) s += static_cast<double>(cur[u]);
#pragma unroll
            for (int u = 0; u < kSumBatch; ++u) cur[u] = nxt[u];
        }
#pragma unroll
        for (int u = 0; u < kSumBatch; ++u) s += static_cast<double>(cur[u]);  // the batch at end_full - kSumBatch
        j = end_full;
    }
    for (; j < hi; ++j) s += static_cast<double>(Xs[static_cast<int64_t>(order[j]) * d_pad + k]);
    C_out[o] = static_cast<float>(s / static_cast<double>(cnt));
}

// Integer-valued rows (8-bit data): every partial sum is an integer below 2^53, so fp64 adds
// are exact in any order and the sums equal the ascending-order sums bit for bit.  A CTA
// takes kSumRange consecutive sorted members (one thread per dimension), accumulates runs of
// one centroid in registers and adds each run to the centroid's sums atomically.
constexpr int kSumRange = 256;

__global__ void centroid_sum_int_kernel(const float* __restrict__ Xs, int d, int d_pad, const int32_t* __restrict__ order,
                                        const int32_t* __restrict__ keys_sorted, int64_t n, int32_t B,
                                        double* __restrict__ sums)
{
    const int64_t lo = static_cast<int64_t>(blockIdx.x) * kSumRange;
    const int64_t hi = lo + kSumRange < n ? lo + kSumRange : n;
    for (int k = threadIdx.x; k < d; k += blockDim.x) {
        int32_t cur = keys_sorted[lo];
        double acc = 0.0;
        for (int64_t j = lo; j < hi; ++j) {
            const int32_t a = keys_sorted[j];
            if (a != cur) {
                if (cur >= 0 && cur < B) atomicAdd(&sums[static_cast<int64_t>(cur) * d + k], acc);
                cur = a;
                acc = 0.0;
            }
            acc += static_cast<double>(Xs[static_cast<int64_t>(order[j]) * d_pad + k]);
        }
        if (cur >= 0 && cur < B) atomicAdd(&sums[static_cast<int64_t>(cur) * d + k], acc);
    }
}

__global__ void centroid_means_int_kernel(const double* __restrict__ sums, const int64_t* __restrict__ offsets,
                                          const float* __restrict__ C_in, int32_t B, int d, int d_pad,
                                          float* __restrict__ C_out)
{
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<int64_t>(B) * d_pad) return;
    const int64_t b = i / d_pad;
    const int k = static_cast<int>(i - b * d_pad);
    const int64_t cnt = offsets[b + 1] - offsets[b];
    if (k >= d) C_out[i] = 0.0f;
    else C_out[i] = cnt > 0 ? static_cast<float>(sums[b * d + k] / static_cast<double>(cnt)) : C_in[i];
}

// Per-centroid fp64 sums (members in sorted order) and counts of a shard.
__global__ void centroid_partial_kernel(const float* __restrict__ Xs, int d, int d_pad,
                                        const int32_t* __restrict__ order, const int64_t* __restrict__ offsets,
                                        double* __restrict__ sums, long long* __restrict__ counts)
{
    const int b = blockIdx.x;
    const int64_t lo = offsets[b], hi = offsets[b + 1];
    if (threadIdx.x == 0) counts[b] = hi - lo;
    for (int k = threadIdx.x; k < d; k += blockDim.x) {
        double s = 0.0;
        for (int64_t j = lo; j < hi; ++j) s += static_cast<double>(Xs[static_cast<int64_t>(order[j]) * d_pad + k]);
        sums[static_cast<int64_t>(b) * d + k] = s;
    }
}

__global__ void centroid_means_kernel(const double* __restrict__ sums, const long long* __restrict__ counts,
                                      const float* __restrict__ C_in, int32_t B, int d, float* __restrict__ C_out)
{
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<int64_t>(B) * d) return;
    const long long c = counts[i / d];
    C_out[i] = c > 0 ? static_cast<float>(sums[i] / static_cast<double>(c)) : C_in[i];
}

__global__ void iota_kernel(int32_t* out, int64_t n)
{
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) out[i] = static_cast<int32_t>(i);
}

// ---------------------------------------------------------------- memberships
// Membership i = (point i/2, way i%2).  Sort key = bucket * B + the point's
// other bucket: inside a bucket, members that share their second bucket (one
// boundary region of the Voronoi diagram) become contiguous, in point order.
// An id outside [0, B), or both ways naming one bucket, is recorded in *err and
// gets the key past every bucket, so no later kernel indexes with it.
__global__ void membership_pairs_kernel(const int32_t* __restrict__ top2, int64_t N, int32_t B,
                                        uint32_t* __restrict__ keys, int32_t* __restrict__ vals, int* err)
{
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= 2 * N) return;
    const int32_t a = top2[i], o = top2[i ^ 1];
    const bool ok = a >= 0 && a < B && o >= 0 && o < B && a != o;
    if (!ok) atomicCAS(err, 0, kDevBadIndex);
    keys[i] = ok ? static_cast<uint32_t>(a) * static_cast<uint32_t>(B) + static_cast<uint32_t>(o) : 0xffffffffu;
    vals[i] = static_cast<int32_t>(i >> 1);
}

// Records in *err any id outside [0, hi).
__global__ void check_ids_kernel(const int32_t* __restrict__ ids, int64_t n, int32_t hi, int* err)
{
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n && (ids[i] < 0 || ids[i] >= hi)) atomicCAS(err, 0, kDevBadIndex);
}

__global__ void seg_offsets_scaled_kernel(const uint32_t* __restrict__ keys_sorted, int64_t n, int32_t B,
                                          int64_t* __restrict__ offsets)
{
    const int64_t b = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (b > B) return;
    const uint64_t want = static_cast<uint64_t>(b) * static_cast<uint64_t>(B);
    int64_t lo = 0, hi = n;  // first index with key >= b * B
    while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if (static_cast<uint64_t>(keys_sorted[mid]) < want) lo = mid + 1;
        else hi = mid;
    }
    offsets[b] = lo;
}

// first index of bucket b's memberships whose partner is above b (keys b * B + partner)
__global__ void phase_split_kernel(const uint32_t* __restrict__ keys_sorted, int64_t n, int32_t B,
                                   int64_t* __restrict__ split)
{
    const int64_t b = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (b >= B) return;
    const uint64_t want = static_cast<uint64_t>(b) * static_cast<uint64_t>(B) + static_cast<uint64_t>(b);
    int64_t lo = 0, hi = n;
    while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if (static_cast<uint64_t>(keys_sorted[mid]) < want) lo = mid + 1;
        else hi = mid;
    }
    split[b] = lo;
}

__global__ void partner_kernel(const uint32_t* __restrict__ keys_sorted, int64_t n, int32_t B,
                               int32_t* __restrict__ partner)
{
    const int64_t j = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (j >= n) return;
    const uint32_t k = keys_sorted[j];
    partner[j] = k < static_cast<uint32_t>(B) * static_cast<uint32_t>(B) ? static_cast<int32_t>(k % static_cast<uint32_t>(B))
                                                                          : -1;
}

// split[b] = first grouped row of bucket b whose partner is above b (rows of a bucket ascend
// by partner)
__global__ void split_from_partner_kernel(const int32_t* __restrict__ partner, const int64_t* __restrict__ offsets,
                                          int32_t B, int64_t* __restrict__ split)
{
    const int64_t b = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (b >= B) return;
    int64_t lo = offsets[b], hi = offsets[b + 1];
    while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if (partner[mid] <= static_cast<int32_t>(b)) lo = mid + 1;
        else hi = mid;
    }
    split[b] = lo;
}

__global__ void seeds_from_lists_kernel(const float* __restrict__ list_d, const int64_t* __restrict__ mem_row,
                                        int64_t N, int M, int64_t j0, int64_t n_rows, float* __restrict__ seed)
{
    const int64_t p = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (p >= N) return;
    const int64_t r = mem_row[2 * p] - j0;
    seed[p] = (r >= 0 && r < n_rows) ? list_d[r * M + (M - 1)] : INFINITY;
}

__global__ void mem_rows_kernel(const uint32_t* __restrict__ keys_sorted, const int32_t* __restrict__ members,
                                const int32_t* __restrict__ top2, int64_t n2, int32_t B, int64_t* __restrict__ mem_row)
{
    const int64_t j = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (j >= n2) return;
    const uint32_t bkt = keys_sorted[j] / static_cast<uint32_t>(B);
    if (bkt >= static_cast<uint32_t>(B)) return;  // an invalid membership (recorded by membership_pairs_kernel)
    const int64_t p = members[j];
    const int32_t lo_b = min(top2[2 * p], top2[2 * p + 1]);
    const int way = static_cast<int32_t>(bkt) == lo_b ? 0 : 1;
    mem_row[2 * p + way] = j;
}

// ---------------------------------------------------------------- merge
// Warp per point.  Output positions follow the two-pointer rule of the
// reference: running entry i lands at i + #{kept new j : bd[j] < ad[i]},
// kept new entry j at rank_j + #{i : ad[i] <= bd[j]}; a new id already in
// the running list is dropped.  Lists are ascending, padded with -1 / +inf.
constexpr int kMergeWarps = 8;
constexpr int kMaxM = 128;

// One warp merges the running list a (na valid entries used) with the new list b: b's entries
// whose id is already in a are dropped, the rest merged by distance with a's entries first on
// equal distance; out may alias a (both lists are staged in shared memory first).  Both lists are
// ascending, so every output position is a binary search in the other list; a's ids sit in a
// small open-addressing table for the duplicate test.
constexpr int kMergeHash = 512;  // >= 4 * kMaxM slots

__device__ __forceinline__ void merge_warp(const int32_t* an, const float* ad, bool va, const int32_t* bn,
                                           const float* bd, bool vb, int M, int32_t* on, float* od, int32_t* s_an,
                                           int32_t* s_bn, float* s_ad, float* s_bd, int* s_pref, uint32_t* s_hash)
{
    const int lane = threadIdx.x & 31;
    int na = va ? M : 0, nb = vb ? M : 0;
    for (int k = lane; k < M; k += 32) {
        const int32_t x = va ? an[k] : -1, y = vb ? bn[k] : -1;
        s_an[k] = x; s_ad[k] = va ? ad[k] : INFINITY; s_bn[k] = y; s_bd[k] = vb ? bd[k] : INFINITY;
        if (x < 0) na = min(na, k);
        if (y < 0) nb = min(nb, k);
    }
    for (int h = lane; h < kMergeHash; h += 32) s_hash[h] = kEmpty;
    for (int off = 16; off > 0; off >>= 1) {
        na = min(na, __shfl_xor_sync(0xffffffffu, na, off));
        nb = min(nb, __shfl_xor_sync(0xffffffffu, nb, off));
    }
    __syncwarp();
    constexpr uint32_t hmask = kMergeHash - 1;
    for (int k = lane; k < na; k += 32) {  // a's ids (>= 0) into the table
        const uint32_t id = static_cast<uint32_t>(s_an[k]);
        for (uint32_t h = (id * 2654435761u) >> 7 & hmask;; h = (h + 1) & hmask) {
            const uint32_t old = atomicCAS(&s_hash[h], kEmpty, id);
            if (old == kEmpty || old == id) break;
        }
    }
    __syncwarp();
    // kept new entries: s_pref[j] = number kept among b[0 .. j)
    int base = 0;
    for (int g = 0; g < (M + 31) / 32; ++g) {
        const int j = g * 32 + lane;
        bool keep = false;
        if (j < nb) {
            const uint32_t id = static_cast<uint32_t>(s_bn[j]);
            keep = true;
            for (uint32_t h = (id * 2654435761u) >> 7 & hmask;; h = (h + 1) & hmask) {
                const uint32_t key = s_hash[h];
                if (key == kEmpty) break;
                if (key == id) { keep = false; break; }
            }
        }
        const unsigned m = __ballot_sync(0xffffffffu, keep);
        const int before = base + __popc(m & ((1u << lane) - 1u));
        if (j < M) s_pref[j] = keep ? before : -1 - before;  // a dropped entry stores -(kept before it) - 1
        base += __popc(m);
    }
    __syncwarp();
    const int n_keep = base;
    auto kept_before = [&](int p) {  // number of kept new entries among b[0 .. p)
        if (p >= nb) return n_keep;
        const int v = s_pref[p];
        return v >= 0 ? v : -1 - v;
    };
    for (int i = lane; i < na; i += 32) {
        const float x = s_ad[i];
        int lo = 0, hi = nb;  // first b entry with distance >= x
        while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (s_bd[mid] < x) lo = mid + 1;
            else hi = mid;
        }
        const int pos = i + kept_before(lo);
        if (pos < M) { on[pos] = s_an[i]; od[pos] = x; }
    }
    for (int j = lane; j < nb; j += 32) {
        const int k = s_pref[j];
        if (k < 0) continue;
        const float x = s_bd[j];
        int lo = 0, hi = na;  // first a entry with distance > x
        while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (s_ad[mid] <= x) lo = mid + 1;
            else hi = mid;
        }
        const int pos = k + lo;
        if (pos < M) { on[pos] = s_bn[j]; od[pos] = x; }
    }
    for (int q = na + n_keep + lane; q < M; q += 32) { on[q] = -1; od[q] = INFINITY; }
    __syncwarp();
}

__global__ void __launch_bounds__(kMergeWarps * 32)
    merge_kernel(const int32_t* __restrict__ run_n, const float* __restrict__ run_d, const int32_t* __restrict__ new_n,
                 const float* __restrict__ new_d, const int64_t* __restrict__ mem_row, int64_t N, int M,
                 int32_t* __restrict__ out_n, float* __restrict__ out_d)
{
    // mem_row entries outside [0, 2N) (a membership that was never built) read as empty lists
    __shared__ int32_t s_an[kMergeWarps][kMaxM], s_bn[kMergeWarps][kMaxM];
    __shared__ float s_ad[kMergeWarps][kMaxM], s_bd[kMergeWarps][kMaxM];
    __shared__ int s_rank[kMergeWarps][kMaxM];
    __shared__ uint32_t s_hash[kMergeWarps][kMergeHash];
    const int w = threadIdx.x >> 5;
    const int64_t p = static_cast<int64_t>(blockIdx.x) * kMergeWarps + w;
    if (p >= N) return;
    const int64_t ra = mem_row ? mem_row[2 * p] : p;
    const int64_t rb = mem_row ? mem_row[2 * p + 1] : p;
    const bool va = !mem_row || (ra >= 0 && ra < 2 * N), vb = !mem_row || (rb >= 0 && rb < 2 * N);
    merge_warp(run_n + (va ? ra : 0) * M, run_d + (va ? ra : 0) * M, va, new_n + (vb ? rb : 0) * M,
               new_d + (vb ? rb : 0) * M, vb, M, out_n + p * M, out_d + p * M, s_an[w], s_bn[w], s_ad[w], s_bd[w],
               s_rank[w], s_hash[w]);
}

// A batch of membership rows j0 .. j0 + n - 1 (lists at row j - j0 of bl / bd) into the per-point
// lists out: pass 0 copies every row that is its point's first (lower-bucket) membership, pass 1
// merges every row that is the second into what the first left there (the order of
// merge_memberships, so a bucket-batched build equals the one-pass build).
__global__ void __launch_bounds__(kMergeWarps * 32)
    merge_batch_kernel(const int32_t* __restrict__ bl, const float* __restrict__ bd, const int32_t* __restrict__ members,
                       const int64_t* __restrict__ mem_row, int64_t j0, int64_t n, int64_t N, int M, int pass,
                       int32_t* __restrict__ out_n, float* __restrict__ out_d)
{
    __shared__ int32_t s_an[kMergeWarps][kMaxM], s_bn[kMergeWarps][kMaxM];
    __shared__ float s_ad[kMergeWarps][kMaxM], s_bd[kMergeWarps][kMaxM];
    __shared__ int s_rank[kMergeWarps][kMaxM];
    __shared__ uint32_t s_hash[kMergeWarps][kMergeHash];
    const int w = threadIdx.x >> 5;
    const int64_t r = static_cast<int64_t>(blockIdx.x) * kMergeWarps + w;
    if (r >= n) return;
    const int64_t j = j0 + r;
    const int64_t pt = members[j];
    if (pt < 0 || pt >= N) return;
    const bool first = mem_row[2 * pt] == j;
    if ((pass == 0) != first) return;
    int32_t* on = out_n + pt * M;
    float* od = out_d + pt * M;
    // pass 0: merge with an empty running list (= the list itself); pass 1: with the running one
    merge_warp(on, od, pass == 1, bl + r * M, bd + r * M, true, M, on, od, s_an[w], s_bn[w], s_ad[w], s_bd[w],
               s_rank[w], s_hash[w]);
}

// ---------------------------------------------------------------- sanitize
// Rows [row0, row0 + n_rows) of an N-point graph (global ids), one warp per row.
__global__ void sanitize_kernel(const int32_t* __restrict__ knn, int64_t n_rows, int64_t row0, int64_t N, int M,
                                uint32_t* __restrict__ out)
{
    const int lane = threadIdx.x & 31;
    const int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= n_rows) return;
    const int64_t i = row0 + r;
    const int32_t* row = knn + r * M;
    uint32_t fallback = static_cast<uint32_t>((i + 1) % N);
    for (int g = 0; g < M; g += 32) {
        const int j = g + lane;
        const int32_t v = j < M ? row[j] : -1;
        const bool ok = v >= 0 && static_cast<int64_t>(v) < N && static_cast<int64_t>(v) != i;
        const unsigned m = __ballot_sync(0xffffffffu, ok);
        if (m) { fallback = static_cast<uint32_t>(__shfl_sync(0xffffffffu, v, __ffs(m) - 1)); break; }
    }
    for (int j = lane; j < M; j += 32) {
        const int32_t v = row[j];
        const bool ok = v >= 0 && static_cast<int64_t>(v) < N && static_cast<int64_t>(v) != i;
        out[r * M + j] = ok ? static_cast<uint32_t>(v) : fallback;
    }
}

// ---------------------------------------------------------------- detour prune
constexpr int kPruneWarps = 8;

// Warp per row a (processed in `order` when given: rows of one bucket region
// together, so the neighbour rows they gather stay in L2).  Row a's candidates
// go into a shared-memory id -> rank hash table sized 8x the row (load factor
// <= 1/8); duplicates of an id keep separate slots.  Lane l takes the closer
// candidates D = row[kAD] with kAD = l, l+32, ...: it reads D's whole row and
// looks every entry up, setting bit kAB of its mask for each later rank kAB >
// kAD whose candidate appears there (a set: a pair (kAD, kAB) counts once even
// when D's row repeats an id).  The detour count of kAB is the number of masks
// holding bit kAB, summed over the warp with ballots; no per-candidate
// cross-lane reduction is needed.

__device__ __forceinline__ uint32_t hash_id(uint32_t id, uint32_t mask) { return (id * 2654435761u) >> 7 & mask; }

// Per warp in dynamic shared memory: the id -> rank hash of the row (cap 64-bit slots, id in
// the high word, rank in the low word; all ones = empty), the row, its detour counts and the
// count histogram / next free position of every count.
__host__ __device__ __forceinline__ uint32_t prune_cap(int M)
{
    uint32_t cap = 64;
    while (cap < 8u * static_cast<uint32_t>(M)) cap <<= 1;
    return cap;
}

// bytes of one warp's region, a multiple of 16 so that every warp's 64-bit slots stay aligned
__host__ __device__ __forceinline__ uint32_t prune_per_warp(int M)
{
    return (prune_cap(M) * 8u + 12u * static_cast<uint32_t>(M) + 15u) & ~15u;
}

__global__ void __launch_bounds__(kPruneWarps * 32)
    prune_kernel(const uint32_t* __restrict__ g, int64_t N, int M, int K, const int32_t* __restrict__ order,
                 int64_t row0, int64_t n_rows, uint32_t* __restrict__ out, int* err)
{
    extern __shared__ __align__(16) uint8_t prune_smem[];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const uint32_t cap = prune_cap(M);
    const uint32_t mask = cap - 1;
    const size_t per_warp = prune_per_warp(M);
    uint64_t* s_slot = reinterpret_cast<uint64_t*>(prune_smem + w * per_warp);
    uint32_t* s_row = reinterpret_cast<uint32_t*>(s_slot + cap);
    uint32_t* s_cnt = s_row + M;
    uint32_t* s_next = s_cnt + M;
    const int64_t gw = static_cast<int64_t>(blockIdx.x) * kPruneWarps + w;
    if (gw >= n_rows) return;
    // rows row0 .. row0 + n_rows - 1 of the graph, visited in `order` (local indices)
    const int64_t orow = order ? static_cast<int64_t>(order[gw]) : gw;
    const int64_t a = row0 + orow;
    for (uint32_t h = lane; h < cap; h += 32) s_slot[h] = ~0ull;
    const uint32_t* ra = g + a * M;
    for (int k = lane; k < M; k += 32) {
        s_row[k] = ra[k];
        s_cnt[k] = 0;
        s_next[k] = 0;
    }
    __syncwarp();
    // A repeated id (sanitize pads with the row's first neighbour) gets a slot per rank; every
    // slot holding the id that a later copy passes is flagged (kDupFlag), so a lookup goes on
    // past a match only when more copies follow along the probe chain.
    constexpr uint64_t kDupFlag = 1ull << 31;
    for (int k = lane; k < M; k += 32) {
        const uint32_t id = s_row[k];
        const uint64_t mine = (static_cast<uint64_t>(id) << 32) | static_cast<uint32_t>(k);
        for (uint32_t h = hash_id(id, mask);; h = (h + 1) & mask) {
            unsigned long long* sp = reinterpret_cast<unsigned long long*>(&s_slot[h]);
            const unsigned long long old = atomicCAS(sp, ~0ull, mine);
            if (old == ~0ull) break;
            if (static_cast<uint32_t>(old >> 32) == id) atomicOr(sp, kDupFlag);
        }
    }
    __syncwarp();
    // Lane l takes kAD = l + 32 j and marks in a mask every later rank kAB whose id appears in
    // row(row[kAD]) (each (D, B) pair once); at load factor <= 1/8 almost every lookup ends at
    // its first slot, so the probe loop is the rare path.
    constexpr int kJ = kMaxM / 32;
    const int n_j = (M - 1 + 31) / 32;
    const bool vec = (M & 3) == 0;
#pragma unroll
    for (int j = 0; j < kJ; ++j) {
        const int kAD = lane + 32 * j;
        if (j >= n_j || kAD >= M - 1) continue;
        const uint32_t dd = s_row[kAD];
        if (static_cast<int64_t>(dd) >= N) {
            atomicCAS(err, 0, kDevBadIndex);
            continue;
        }
        const uint32_t* rd = g + static_cast<int64_t>(dd) * M;
        uint64_t m0 = 0, m1 = 0;
        auto look = [&](uint32_t v) {
            // ids of the graph are < N < 2^31; anything else (all ones included, which would
            // read as the high word of an empty slot) is in no row
            if (static_cast<int64_t>(v) >= N) return;
            uint32_t h = hash_id(v, mask);
            for (;;) {
                uint64_t sl = s_slot[h];
                while (static_cast<uint32_t>(sl >> 32) != v) {
                    if (sl == ~0ull) return;
                    h = (h + 1) & mask;
                    sl = s_slot[h];
                }
                const int kAB = static_cast<int>(static_cast<uint32_t>(sl) & 0x7fu);
                if (kAB > kAD) {
                    const uint64_t bit = 1ull << (kAB & 63);
                    if (kAB < 64) m0 |= bit;
                    else m1 |= bit;
                }
                if (!(sl & kDupFlag)) return;
                h = (h + 1) & mask;
            }
        };
        if ((M & 15) == 0) {
            // 16 ids per batch: four 16-byte loads in flight before the lookups that use them
            const uint4* rd4 = reinterpret_cast<const uint4*>(rd);
            for (int e16 = 0; e16 < (M >> 4); ++e16) {
                uint4 x[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) x[u] = __ldg(rd4 + 4 * e16 + u);
#pragma unroll
                for (int u = 0; u < 4; ++u) { look(x[u].x); look(x[u].y); look(x[u].z); look(x[u].w); }
            }
        } else if (vec) {
            const uint4* rd4 = reinterpret_cast<const uint4*>(rd);
            for (int e4 = 0; e4 < (M >> 2); ++e4) {
                const uint4 x = rd4[e4];
                look(x.x); look(x.y); look(x.z); look(x.w);
            }
        } else {
            for (int e = 0; e < M; ++e) look(rd[e]);
        }
        // detour counts: one shared-memory increment per marked (D, B) pair
        while (m0) {
            atomicAdd(&s_cnt[__ffsll(static_cast<long long>(m0)) - 1], 1u);
            m0 &= m0 - 1;
        }
        while (m1) {
            atomicAdd(&s_cnt[64 + __ffsll(static_cast<long long>(m1)) - 1], 1u);
            m1 &= m1 - 1;
        }
    }
    __syncwarp();
    // position of entry k = #{k' : (cnt[k'], k') < (cnt[k], k)}: counts histogram -> exclusive
    // prefix = first position of each count; entries of equal count in ascending k
    for (int k = lane; k < M; k += 32) atomicAdd(&s_next[s_cnt[k]], 1u);
    __syncwarp();
    uint32_t carry = 0;
    for (int c0 = 0; c0 < M; c0 += 32) {
        const uint32_t v = c0 + lane < M ? s_next[c0 + lane] : 0u;
        uint32_t incl = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
        }
        if (c0 + lane < M) s_next[c0 + lane] = carry + incl - v;
        carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    __syncwarp();
    const unsigned lt = (1u << lane) - 1u;
    for (int k0 = 0; k0 < M; k0 += 32) {
        const int k = k0 + lane;
        const bool has = k < M;
        const uint32_t c = has ? s_cnt[k] : 0xFFFFFFFFu;
        const unsigned grp = __match_any_sync(0xffffffffu, c);
        const uint32_t base = has ? s_next[c] : 0u;
        __syncwarp();
        if (has) {
            const uint32_t pos = base + static_cast<uint32_t>(__popc(grp & lt));
            if (pos < static_cast<uint32_t>(K)) out[orow * K + pos] = s_row[k];
            if ((grp & lt) == 0u) s_next[c] = base + static_cast<uint32_t>(__popc(grp));  // the group's first lane
        }
        __syncwarp();
    }
}

size_t prune_smem_bytes(int M) { return static_cast<size_t>(kPruneWarps) * prune_per_warp(M); }

// Received memberships grouped by (bucket, other bucket), stable in arrival order.
__global__ void group_keys_kernel(const int32_t* __restrict__ bucket, const int32_t* __restrict__ other, int64_t n,
                                  int32_t B, uint32_t* __restrict__ keys, int32_t* __restrict__ vals)
{
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    keys[i] = static_cast<uint32_t>(bucket[i]) * static_cast<uint32_t>(B) + static_cast<uint32_t>(other[i]);
    vals[i] = static_cast<int32_t>(i);
}

// Rows grouped by (nearest bucket, second bucket): the processing order that
// keeps a warp's neighbour rows in L2 (same grouping as the memberships).
__global__ void locality_keys_kernel(const int32_t* __restrict__ top2, int64_t N, int32_t B, uint32_t* __restrict__ keys,
                                     int32_t* __restrict__ vals)
{
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= N) return;
    keys[i] = static_cast<uint32_t>(top2[2 * i]) * static_cast<uint32_t>(B) + static_cast<uint32_t>(top2[2 * i + 1]);
    vals[i] = static_cast<int32_t>(i);
}

// ---------------------------------------------------------------- reverse edges
// The reverse list of destination j: the sources i with j in pruned(i), ordered by
// (rank of j in row i, i) and capped at K (edge_chunk_accumulator.hpp:386-469
// TopKReverseStore, :235-284 build_rank_ordered_csr).  One edge is one key
// rank << src_bits | src, so ascending keys are exactly that order; the key is 32 bits
// wide whenever bits(N - 1) + bits(K - 1) <= 32 (every configuration up to 2^27 rows at
// K = 32), else 64 bits.

__device__ __forceinline__ void report_error(int* err, int code)
{
    if (err) atomicCAS(err, 0, code);
}

// One warp per source row of the whole pruned graph (N x K, global ids); destinations
// in [lo, hi) are counted at local index dst - lo.  An id >= N is reported as
// kDevBadIndex (the entry point returns GTA_EDATA) and dropped.
__global__ void rev_count_kernel(const uint32_t* __restrict__ pruned, int64_t N, int K, int64_t lo, int64_t hi,
                                 unsigned long long* __restrict__ indeg, int* __restrict__ err)
{
    const int lane = threadIdx.x & 31;
    const int64_t src = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    if (src >= N) return;
    for (int r = lane; r < K; r += 32) {
        const int64_t dst = pruned[src * K + r];
        if (dst >= N) {
            report_error(err, kDevBadIndex);
            continue;
        }
        if (dst >= lo && dst < hi) atomicAdd(&indeg[dst - lo], 1ull);
    }
}

// Each edge's key into its destination's segment of the CSR (slot order within a
// segment is arbitrary; the merge sorts it).
template <typename KeyT>
__global__ void rev_scatter_kernel(const uint32_t* __restrict__ pruned, int64_t N, int K, int64_t lo, int64_t hi,
                                   int src_bits, const uint64_t* __restrict__ off, uint32_t* __restrict__ cursor,
                                   KeyT* __restrict__ keys)
{
    const int lane = threadIdx.x & 31;
    const int64_t src = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    if (src >= N) return;
    for (int r = lane; r < K; r += 32) {
        const int64_t dst = pruned[src * K + r];
        if (dst < lo || dst >= hi) continue;  // hi <= N: out-of-range ids were reported by the count
        const uint64_t pos = off[dst - lo] + atomicAdd(&cursor[dst - lo], 1u);
        keys[pos] = (static_cast<KeyT>(r) << src_bits) | static_cast<KeyT>(src);
    }
}

// One compare-exchange stage of a warp-wide bitonic network over 32 R keys held as
// v[r] = element 32 r + lane: partners at distance j, direction set by bit k.
template <typename KeyT, int R>
__device__ __forceinline__ void bitonic_stage(KeyT (&v)[R], int lane, int k, int j)
{
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int e = 32 * r + lane;
        const bool up = (e & k) == 0;
        if (j >= 32) {
            const int rp = r ^ (j >> 5);
            if (rp > r) {
                const KeyT a = v[r], b = v[rp];
                const KeyT mn = a < b ? a : b, mx = a < b ? b : a;
                v[r] = up ? mn : mx;
                v[rp] = up ? mx : mn;
            }
        } else {
            const KeyT o = __shfl_xor_sync(0xffffffffu, v[r], j);
            const bool take_min = ((lane & j) == 0) == up;
            v[r] = take_min ? (o < v[r] ? o : v[r]) : (o > v[r] ? o : v[r]);
        }
    }
}

template <typename KeyT, int R>
__device__ __forceinline__ void warp_sort_keys(KeyT (&v)[R], int lane)
{
#pragma unroll
    for (int k = 2; k <= 32 * R; k <<= 1)
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) bitonic_stage<KeyT, R>(v, lane, k, j);
}

// best <- the 32 R smallest of (best, c), both ascending: the element-wise minimum of
// best and reversed c is bitonic and holds them; one merge pass sorts it.
template <typename KeyT, int R>
__device__ __forceinline__ void warp_merge_lowest(KeyT (&best)[R], const KeyT (&c)[R], int lane)
{
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const KeyT t = __shfl_sync(0xffffffffu, c[R - 1 - r], 31 - lane);
        best[r] = t < best[r] ? t : best[r];
    }
#pragma unroll
    for (int j = 16 * R; j > 0; j >>= 1) bitonic_stage<KeyT, R>(best, lane, 32 * R, j);
}

constexpr int kRevWarps = 8;

// One warp per destination j (rows [row0, row0 + n_rows) of the pruned graph):
//  1. the min(len, K) smallest keys of j's segment, ascending, by a register bitonic
//     sort of 32 R keys per chunk and a keep-lowest merge across chunks (K <= 32 R);
//  2. the protected merge of edge_chunk_accumulator.hpp:471-494 merge_rank_ordered_into_row
//     (sources inserted weakest first after the first K/2 forward edges, an id already in
//     the row moved instead of repeated, the last entry dropped when the row is full), in
//     its closed form: the first K/2 entries stay; then the reverse sources strongest first,
//     each kept only if it is not among the first K/2 and not a repeat of a stronger one;
//     then the remaining forward entries in order, less the first copy of every kept source;
//     the row cut at K.  (Serial insertion is a move-to-front list of capacity K - K/2, whose
//     final content is its distinct accesses by recency followed by what was never touched.)
template <typename KeyT, int R>
__global__ void __launch_bounds__(kRevWarps * 32)
    rev_merge_kernel(const uint32_t* __restrict__ pruned, int64_t row0, int64_t n_rows, int K, int src_bits,
                     const uint64_t* __restrict__ off, const KeyT* __restrict__ keys, uint32_t* __restrict__ out)
{
    __shared__ uint32_t s_src[kRevWarps][32 * R], s_row[kRevWarps][32 * R], s_out[kRevWarps][32 * R];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int64_t j = static_cast<int64_t>(blockIdx.x) * kRevWarps + w;
    if (j >= n_rows) return;
    const KeyT kNone = ~static_cast<KeyT>(0);
    const uint64_t lo = off[j];
    const int64_t len = static_cast<int64_t>(off[j + 1] - lo);
    uint32_t* row = s_row[w];
    uint32_t* sel = s_out[w];
    for (int k = lane; k < K; k += 32) row[k] = pruned[(row0 + j) * K + k];
    KeyT best[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int64_t e = 32 * r + lane;
        best[r] = e < len ? keys[lo + e] : kNone;
    }
    warp_sort_keys<KeyT, R>(best, lane);
    for (int64_t c0 = 32 * R; c0 < len; c0 += 32 * R) {
        KeyT c[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int64_t e = c0 + 32 * r + lane;
            c[r] = e < len ? keys[lo + e] : kNone;
        }
        warp_sort_keys<KeyT, R>(c, lane);
        warp_merge_lowest<KeyT, R>(best, c, lane);
    }
    const KeyT src_mask = (static_cast<KeyT>(1) << src_bits) - 1;
#pragma unroll
    for (int r = 0; r < R; ++r) s_src[w][32 * r + lane] = static_cast<uint32_t>(best[r] & src_mask);
    __syncwarp();
    const int n_keep = static_cast<int>(len < K ? len : K);
    const int np = K / 2;
    const unsigned lt = (1u << lane) - 1u;
    // reverse sources, strongest first: not protected, first occurrence
    int nu = 0;
    for (int g0 = 0; g0 < n_keep; g0 += 32) {
        const int t = g0 + lane;
        const uint32_t src = t < n_keep ? s_src[w][t] : kEmpty;
        bool keep = t < n_keep;
        for (int p = 0; p < np; ++p) keep &= row[p] != src;
        for (int p = 0; p < g0; ++p) keep &= s_src[w][p] != src;
        keep &= (__ffs(__match_any_sync(0xffffffffu, src)) - 1) == lane;
        const unsigned b = __ballot_sync(0xffffffffu, keep);
        const int pos = np + nu + __popc(b & lt);
        if (keep && pos < K) sel[pos] = src;
        nu += __popc(b);
    }
    __syncwarp();
    if (nu < K - np) {
        // the forward entries after the protected ones, less the first copy of each kept source
        int nr = 0;
        for (int g0 = np; g0 < K; g0 += 32) {
            const int q = g0 + lane;
            const uint32_t o = q < K ? row[q] : kEmpty;
            bool in_sel = false;
            for (int i = 0; i < nu; ++i) in_sel |= sel[np + i] == o;
            bool first = true;
            for (int p = np; p < g0; ++p) first &= row[p] != o;
            first &= (__ffs(__match_any_sync(0xffffffffu, o)) - 1) == lane;
            const bool keep = q < K && !(in_sel && first);
            const unsigned b = __ballot_sync(0xffffffffu, keep);
            const int pos = np + nu + nr + __popc(b & lt);
            if (keep && pos < K) sel[pos] = o;
            nr += __popc(b);
        }
        __syncwarp();
    }
    for (int k = lane; k < K; k += 32) out[j * K + k] = k < np ? row[k] : sel[k];
}

// ---------------------------------------------------------------- row sort by exact distance
__global__ void sort_rows_kernel(const float* __restrict__ X, int d, int d_pad, const int32_t* __restrict__ knn,
                                 int64_t N, int M, int32_t* __restrict__ out)
{
    __shared__ uint64_t s_keys[4][kMaxM];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int64_t i = static_cast<int64_t>(blockIdx.x) * 4 + w;
    if (i >= N) return;
    int np2 = 1;
    while (np2 < M) np2 <<= 1;
    for (int k = lane; k < np2; k += 32) {
        uint64_t key = ~0ull;
        if (k < M) {
            const int32_t id = knn[i * M + k];
            if (id >= 0 && static_cast<int64_t>(id) < N) {
                const float dd = exact_l2_f(X + i * d_pad, X + static_cast<int64_t>(id) * d_pad, d);
                key = (static_cast<uint64_t>(f2key(dd)) << 32) | static_cast<uint32_t>(k);
            }
        }
        s_keys[w][k] = key;
    }
    __syncwarp();
    for (int k = 2; k <= np2; k <<= 1)
        for (int jj = k >> 1; jj > 0; jj >>= 1) {
            for (int t = lane; t < (np2 >> 1); t += 32) {
                const int a = 2 * jj * (t / jj) + (t % jj), l = a + jj;
                const bool up = (a & k) == 0;
                const uint64_t x = s_keys[w][a], y = s_keys[w][l];
                if ((x > y) == up) { s_keys[w][a] = y; s_keys[w][l] = x; }
            }
            __syncwarp();
        }
    for (int k = lane; k < M; k += 32) {
        const uint64_t key = s_keys[w][k];
        out[i * M + k] = key == ~0ull ? -1 : knn[i * M + static_cast<int>(key & 0xffffffffu)];
    }
}

__global__ void max_sqrt_kernel(const float* __restrict__ v, int64_t n, unsigned* __restrict__ out)
{
    float m = 0.0f;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        m = fmaxf(m, sqrtf(fmaxf(v[i], 0.0f)));
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(m));
}

unsigned blocks_for(int64_t n, int per) { return static_cast<unsigned>((n + per - 1) / per); }

}  // namespace

// ============================================================================ host launchers
void convert_rows(const void* X, int dtype, int d, const int32_t* row_ids, int64_t n_out, void* out, int out_elem,
                  int d_pad, float* norms, cudaStream_t st)
{
    if (n_out == 0) return;
    switch (dtype) {
        case 0: convert_dispatch_out(static_cast<const float*>(X), d, row_ids, n_out, out, out_elem, d_pad, norms, st); break;
        case 1: convert_dispatch_out(static_cast<const uint8_t*>(X), d, row_ids, n_out, out, out_elem, d_pad, norms, st); break;
        case 2: convert_dispatch_out(static_cast<const int8_t*>(X), d, row_ids, n_out, out, out_elem, d_pad, norms, st); break;
        default: throw Error(kInvalid, "convert_rows: unknown dtype");
    }
    GTA_CUDA(cudaGetLastError());
}

void sample_ids(int64_t N, int64_t n_s, uint64_t seed, int32_t* out, cudaStream_t st)
{
    if (n_s >= N) {
        iota_kernel<<<blocks_for(N, 256), 256, 0, st>>>(out, N);
        count_launches(1);
    } else {
        sample_ids_kernel<<<blocks_for(n_s, 256), 256, 0, st>>>(N, n_s, seed, out);
        count_launches(1);
    }
    GTA_CUDA(cudaGetLastError());
}

void kmeanspp_init(const float* pool, const float* /*pool_norm*/, int64_t pool_n, int d, int d_pad, int32_t B,
                   uint64_t seed, float* C, int* err, cudaStream_t st)
{
    GTA_REQUIRE(pool_n >= 1 && B >= 1, kInvalid, "kmeans++: empty pool");
    {
        // one cooperative launch when every CTA fits on the device at once
        const int G = static_cast<int>((pool_n + kKppCoopThreads - 1) / kKppCoopThreads);
        int dev = 0, n_sm = 0, per_sm = 0, coop = 0;
        GTA_CUDA(cudaGetDevice(&dev));
        GTA_CUDA(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev));
        GTA_CUDA(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev));
        // pool rows resident in shared memory when they fit (d <= 200: about 200 KB per CTA), else
        // staged through it kKppDims dimensions at a time
        const size_t staged = sizeof(float) * (static_cast<size_t>(d_pad) + static_cast<size_t>(kKppDims) * kKppStride);
        int resident = d <= 200 ? 1 : (staged <= 227 * 1024 ? 2 : 0);
        size_t smem1 = resident == 1 ? sizeof(float) * static_cast<size_t>(d_pad) * (1 + kKppCoopThreads)
                                     : (resident == 2 ? staged : sizeof(float) * static_cast<size_t>(d_pad));
        if (smem1 > 227 * 1024) {
            // one centroid row alone does not fit either: the per-centroid launches below
            resident = 0;
            smem1 = sizeof(float) * static_cast<size_t>(d_pad);
        }
        // the attribute covers the layout chosen here and the staged one it may fall back to
        GTA_CUDA(cudaFuncSetAttribute(kpp_coop_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(std::min<size_t>(std::max(smem1, staged), 227 * 1024))));
        GTA_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kpp_coop_kernel, kKppCoopThreads, smem1));
        if (resident == 1 && G > per_sm * n_sm) {
            resident = staged <= 227 * 1024 ? 2 : 0;
            smem1 = resident == 2 ? staged : sizeof(float) * static_cast<size_t>(d_pad);
            GTA_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kpp_coop_kernel, kKppCoopThreads, smem1));
        }
        if (coop && smem1 <= 227 * 1024 && G <= per_sm * n_sm && G <= kKppCoopThreads) {
            DevBuf<double> gpre(static_cast<size_t>(2) * G * kKppCoopThreads, st), gtot(static_cast<size_t>(2) * G, st);
            DevBuf<unsigned> arrive(2, st);
            GTA_CUDA(cudaMemsetAsync(arrive.get(), 0, 2 * sizeof(unsigned), st));
            GTA_CUDA(cudaMemsetAsync(C, 0, sizeof(float) * static_cast<size_t>(B) * d_pad, st));
            unsigned* arr = arrive.get();
            int* abort_flag = reinterpret_cast<int*>(arrive.get() + 1);
            double* gp = gpre.get();
            double* gt = gtot.get();
            void* args[] = {const_cast<float**>(&pool), &pool_n, &d, &d_pad, &C, &B, &seed, &gp, &gt, &arr, &abort_flag, &err,
                            &resident};
            GTA_CUDA(cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(kpp_coop_kernel), dim3(G),
                                                 dim3(kKppCoopThreads), args, smem1, st));
            count_launches(1);
            return;
        }
    }
    const int64_t chunk = std::max<int64_t>(256, (pool_n + 295) / 296);
    const unsigned grid = static_cast<unsigned>((pool_n + chunk - 1) / chunk);
    DevBuf<float> min_d2(static_cast<size_t>(pool_n), st);
    DevBuf<double> bsum(grid, st);
    DevBuf<unsigned> counter(1, st);
    GTA_CUDA(cudaMemsetAsync(counter.get(), 0, sizeof(unsigned), st));
    GTA_CUDA(cudaMemsetAsync(C, 0, sizeof(float) * static_cast<size_t>(B) * d_pad, st));
    kpp_first_kernel<<<1, 128, 0, st>>>(pool, pool_n, d_pad, seed, C);
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
    const size_t smem = sizeof(float) * static_cast<size_t>(d);
    for (int t = 0; t < B; ++t) {
        kpp_step_kernel<<<grid, kKppThreads, smem, st>>>(pool, pool_n, d, d_pad, C, t, B, min_d2.get(), bsum.get(),
                                                         counter.get(), seed, chunk);
        count_launches(1);
    }
    GTA_CUDA(cudaGetLastError());
}

void check_ids(const int32_t* ids, int64_t n, int32_t hi, int* err, cudaStream_t st)
{
    if (n == 0) return;
    check_ids_kernel<<<blocks_for(n, 256), 256, 0, st>>>(ids, n, hi, err);
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

void centroid_update(const float* Xs, int64_t n_s, int d, int d_pad, const int32_t* assign, const float* C_in,
                     int32_t B, float* C_out, float* C_norm, int* err, cudaStream_t st, bool integer_rows)
{
    check_ids(assign, n_s, B, err, st);
    DevBuf<int32_t> keys_out(n_s, st), idx_in(n_s, st), idx_out(n_s, st);
    DevBuf<int64_t> offsets(static_cast<size_t>(B) + 1, st);
    iota_kernel<<<blocks_for(n_s, 256), 256, 0, st>>>(idx_in.get(), n_s);
    count_launches(1);
    int end_bit = 1;
    while ((1ll << end_bit) < B) ++end_bit;
    size_t tmp = 0;
    GTA_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, tmp, assign, keys_out.get(), idx_in.get(), idx_out.get(),
                                             static_cast<int>(n_s), 0, end_bit, st));
    DevBuf<uint8_t> tbuf(tmp, st);
    GTA_CUDA(cub::DeviceRadixSort::SortPairs(tbuf.get(), tmp, assign, keys_out.get(), idx_in.get(), idx_out.get(),
                                             static_cast<int>(n_s), 0, end_bit, st));
    seg_offsets_kernel<<<blocks_for(B + 1, 256), 256, 0, st>>>(keys_out.get(), n_s, B, offsets.get());
    count_launches(1);
    ProfScope prof("kmeans_update", 4.0 * static_cast<double>(n_s) * d, st);
    if (integer_rows && n_s > 0) {
        DevBuf<double> sums(static_cast<size_t>(B) * d, st);
        GTA_CUDA(cudaMemsetAsync(sums.get(), 0, sizeof(double) * static_cast<size_t>(B) * d, st));
        centroid_sum_int_kernel<<<blocks_for(n_s, kSumRange), 128, 0, st>>>(Xs, d, d_pad, idx_out.get(), keys_out.get(),
                                                                            n_s, B, sums.get());
        centroid_means_int_kernel<<<blocks_for(static_cast<int64_t>(B) * d_pad, 256), 256, 0, st>>>(
            sums.get(), offsets.get(), C_in, B, d, d_pad, C_out);
        count_launches(2);
    } else {
        const dim3 grid(static_cast<unsigned>(B), static_cast<unsigned>((d_pad + 127) / 128));
        centroid_sum_kernel<<<grid, 128, 0, st>>>(Xs, d, d_pad, idx_out.get(), offsets.get(), C_in, C_out);
        count_launches(1);
    }
    if (C_norm) convert_rows(C_out, 0, d_pad, nullptr, B, C_out, kElemF32, d_pad, C_norm, st);
    GTA_CUDA(cudaGetLastError());
}

void group_by_key(const int32_t* keys, int64_t n, int32_t B, int32_t* order, int64_t* offsets, int* err, cudaStream_t st)
{
    GTA_REQUIRE(n >= 1 && n < (1ll << 31) && B >= 1, kInvalid, "group_by_key: need 1 <= n < 2^31, B >= 1");
    check_ids(keys, n, B, err, st);
    DevBuf<int32_t> keys_out(static_cast<size_t>(n), st), idx_in(static_cast<size_t>(n), st);
    iota_kernel<<<blocks_for(n, 256), 256, 0, st>>>(idx_in.get(), n);
    count_launches(1);
    int end_bit = 1;
    while ((1ll << end_bit) < B) ++end_bit;
    size_t tmp = 0;
    GTA_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, tmp, keys, keys_out.get(), idx_in.get(), order,
                                             static_cast<int>(n), 0, end_bit, st));
    DevBuf<uint8_t> tbuf(tmp, st);
    GTA_CUDA(cub::DeviceRadixSort::SortPairs(tbuf.get(), tmp, keys, keys_out.get(), idx_in.get(), order,
                                             static_cast<int>(n), 0, end_bit, st));
    seg_offsets_kernel<<<blocks_for(B + 1, 256), 256, 0, st>>>(keys_out.get(), n, B, offsets);
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

void build_memberships(const int32_t* top2, int64_t N, int32_t B, int32_t* members, int64_t* offsets,
                       int64_t* mem_row, int* err, cudaStream_t st, int64_t* split, int32_t* partner)
{
    const int64_t n2 = 2 * N;
    GTA_REQUIRE(n2 < (1ll << 31), kInvalid, "memberships: more than 2^31 memberships on one device");
    GTA_REQUIRE(static_cast<int64_t>(B) * B < (1ll << 32), kInvalid, "memberships: n_buckets must be below 65536");
    DevBuf<uint32_t> keys_in(n2, st), keys_out(n2, st);
    DevBuf<int32_t> vals_in(n2, st);
    ProfScope prof("memberships", 24.0 * static_cast<double>(n2), st);
    membership_pairs_kernel<<<blocks_for(n2, 256), 256, 0, st>>>(top2, N, B, keys_in.get(), vals_in.get(), err);
    count_launches(1);
    int end_bit = 1;
    while ((1ll << end_bit) < static_cast<int64_t>(B) * B) ++end_bit;
    size_t tmp = 0;
    GTA_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, tmp, keys_in.get(), keys_out.get(), vals_in.get(), members,
                                             static_cast<int>(n2), 0, end_bit, st));
    DevBuf<uint8_t> tbuf(tmp, st);
    GTA_CUDA(cub::DeviceRadixSort::SortPairs(tbuf.get(), tmp, keys_in.get(), keys_out.get(), vals_in.get(), members,
                                             static_cast<int>(n2), 0, end_bit, st));
    seg_offsets_scaled_kernel<<<blocks_for(B + 1, 256), 256, 0, st>>>(keys_out.get(), n2, B, offsets);
    count_launches(1);
    GTA_CUDA(cudaMemsetAsync(mem_row, 0xff, sizeof(int64_t) * static_cast<size_t>(n2), st));  // -1: not built
    mem_rows_kernel<<<blocks_for(n2, 256), 256, 0, st>>>(keys_out.get(), members, top2, n2, B, mem_row);
    count_launches(1);
    if (split) {
        phase_split_kernel<<<blocks_for(B, 256), 256, 0, st>>>(keys_out.get(), n2, B, split);
        count_launches(1);
    }
    if (partner) {
        partner_kernel<<<blocks_for(n2, 256), 256, 0, st>>>(keys_out.get(), n2, B, partner);
        count_launches(1);
    }
    GTA_CUDA(cudaGetLastError());
}

void split_from_partner(const int32_t* partner, const int64_t* offsets, int32_t B, int64_t* split, cudaStream_t st)
{
    split_from_partner_kernel<<<blocks_for(B, 256), 256, 0, st>>>(partner, offsets, B, split);
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

void seeds_from_lists(const float* list_d, const int64_t* mem_row, int64_t N, int M, int64_t j0, int64_t n_rows,
                      float* seed, cudaStream_t st)
{
    seeds_from_lists_kernel<<<blocks_for(N, 256), 256, 0, st>>>(list_d, mem_row, N, M, j0, n_rows, seed);
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

void merge_memberships(const int32_t* list_n, const float* list_d, const int64_t* mem_row, int64_t N, int M,
                       int32_t* out_n, float* out_d, cudaStream_t st)
{
    GTA_REQUIRE(M >= 1 && M <= kMaxM, kInvalid, "merge: M must be in [1, 128]");
    ProfScope prof("merge", 24.0 * M * static_cast<double>(N), st);
    merge_kernel<<<blocks_for(N, kMergeWarps), kMergeWarps * 32, 0, st>>>(list_n, list_d, list_n, list_d, mem_row, N, M,
                                                                          out_n, out_d);
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

void merge_membership_batch(const int32_t* bl, const float* bd, const int32_t* members, const int64_t* mem_row,
                            int64_t j0, int64_t n, int64_t N, int M, int32_t* out_n, float* out_d, cudaStream_t st,
                            int passes)
{
    GTA_REQUIRE(M >= 1 && M <= kMaxM, kInvalid, "merge: M must be in [1, 128]");
    if (n <= 0) return;
    for (int pass = 0; pass < 2; ++pass) {
        if (!((passes >> pass) & 1)) continue;
        merge_batch_kernel<<<blocks_for(n, kMergeWarps), kMergeWarps * 32, 0, st>>>(bl, bd, members, mem_row, j0, n, N, M,
                                                                                     pass, out_n, out_d);
        count_launches(1);
    }
    GTA_CUDA(cudaGetLastError());
}

void merge_lists(const int32_t* run_n, const float* run_d, const int32_t* new_n, const float* new_d, int64_t N,
                 int M, int32_t* out_n, float* out_d, cudaStream_t st)
{
    GTA_REQUIRE(M >= 1 && M <= kMaxM, kInvalid, "merge: M must be in [1, 128]");
    merge_kernel<<<blocks_for(N, kMergeWarps), kMergeWarps * 32, 0, st>>>(run_n, run_d, new_n, new_d, nullptr, N, M,
                                                                          out_n, out_d);
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

void sanitize(const int32_t* knn, int64_t N, int M, uint32_t* out, cudaStream_t st)
{
    ProfScope prof("sanitize", 8.0 * M * static_cast<double>(N), st);
    sanitize_kernel<<<blocks_for(N, 8), 256, 0, st>>>(knn, N, 0, N, M, out);
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

void prune_detour(const uint32_t* g, int64_t N, int M, int K, const int32_t* order, uint32_t* out, int* err,
                  cudaStream_t st)
{
    GTA_REQUIRE(M >= 2 && M <= kMaxM && K >= 1 && K <= M, kInvalid, "prune: need 1 <= K <= M <= 128");
    ProfScope prof("prune", (4.0 * M * (M + 1) + 4.0 * K) * static_cast<double>(N), st);
    const size_t smem = prune_smem_bytes(M);
    GTA_CUDA(cudaFuncSetAttribute(prune_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    prune_kernel<<<blocks_for(N, kPruneWarps), kPruneWarps * 32, smem, st>>>(g, N, M, K, order, 0, N, out, err);
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

void locality_order(const int32_t* top2, int64_t N, int32_t B, int32_t* order, cudaStream_t st)
{
    GTA_REQUIRE(static_cast<int64_t>(B) * B < (1ll << 32), kInvalid, "locality order: n_buckets must be below 65536");
    DevBuf<uint32_t> keys_in(N, st), keys_out(N, st);
    DevBuf<int32_t> vals_in(N, st);
    locality_keys_kernel<<<blocks_for(N, 256), 256, 0, st>>>(top2, N, B, keys_in.get(), vals_in.get());
    count_launches(1);
    int end_bit = 1;
    while ((1ll << end_bit) < static_cast<int64_t>(B) * B) ++end_bit;
    size_t tmp = 0;
    GTA_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, tmp, keys_in.get(), keys_out.get(), vals_in.get(), order,
                                             static_cast<int>(N), 0, end_bit, st));
    DevBuf<uint8_t> tbuf(tmp, st);
    GTA_CUDA(cub::DeviceRadixSort::SortPairs(tbuf.get(), tmp, keys_in.get(), keys_out.get(), vals_in.get(), order,
                                             static_cast<int>(N), 0, end_bit, st));
    GTA_CUDA(cudaGetLastError());
}

namespace {

int bits_for(uint64_t x) { return x ? 64 - __builtin_clzll(x) : 0; }

// Where one reverse-edge merge keeps its scratch: in-degrees (u64, rows + 1), CSR offsets
// (u64, rows + 1), cursors (u32, rows), edge keys (N * K keys of key_bytes) and the scan's
// temporary storage.
struct RevScratch {
    unsigned long long* indeg;
    uint64_t* off;
    uint32_t* cursor;
    void* keys;
    void* scan_tmp;
    size_t scan_bytes;
};

// bytes of one edge key: 4 when rank and source fit together in 32 bits
int rev_key_bytes(int64_t N, int K)
{
    return std::max(1, bits_for(static_cast<uint64_t>(N - 1))) + bits_for(static_cast<uint64_t>(K - 1)) <= 32 ? 4 : 8;
}

size_t rev_scan_bytes(int64_t n_rows)
{
    size_t tmp = 0;
    GTA_CUDA(cub::DeviceScan::ExclusiveSum(nullptr, tmp, static_cast<unsigned long long*>(nullptr),
                                           static_cast<uint64_t*>(nullptr), static_cast<int>(n_rows + 1)));
    return tmp;
}

template <typename KeyT>
void rev_scatter_merge(const uint32_t* pruned, int64_t N, int K, int64_t lo, int64_t n_rows, int src_bits,
                       const RevScratch& s, uint32_t* out, cudaStream_t st)
{
    KeyT* keys = static_cast<KeyT*>(s.keys);
    rev_scatter_kernel<KeyT><<<blocks_for(N, 8), 256, 0, st>>>(pruned, N, K, lo, lo + n_rows, src_bits, s.off,
                                                               s.cursor, keys);
    const unsigned grid = blocks_for(n_rows, kRevWarps);
    if (K <= 32)
        rev_merge_kernel<KeyT, 1><<<grid, kRevWarps * 32, 0, st>>>(pruned, lo, n_rows, K, src_bits, s.off, keys, out);
    else if (K <= 64)
        rev_merge_kernel<KeyT, 2><<<grid, kRevWarps * 32, 0, st>>>(pruned, lo, n_rows, K, src_bits, s.off, keys, out);
    else
        rev_merge_kernel<KeyT, 4><<<grid, kRevWarps * 32, 0, st>>>(pruned, lo, n_rows, K, src_bits, s.off, keys, out);
    count_launches(2);
}

// Reverse-edge merge of the destinations [lo, lo + n_rows) of the pruned graph (N x K,
// global ids) into out (n_rows x K): in-degree count (ids >= N reported in *err), offsets
// by an exclusive scan, keys scattered into each destination's segment, one warp per
// destination for its K smallest keys and the protected merge.
void reverse_merge_core(const uint32_t* pruned, int64_t N, int K, int64_t lo, int64_t n_rows, uint32_t* out,
                        const RevScratch& s, int* err, cudaStream_t st)
{
    const int src_bits = std::max(1, bits_for(static_cast<uint64_t>(N - 1)));
    GTA_CUDA(cudaMemsetAsync(s.indeg, 0, sizeof(unsigned long long) * (n_rows + 1), st));
    GTA_CUDA(cudaMemsetAsync(s.cursor, 0, sizeof(uint32_t) * n_rows, st));
    rev_count_kernel<<<blocks_for(N, 8), 256, 0, st>>>(pruned, N, K, lo, lo + n_rows, s.indeg, err);
    count_launches(1);
    size_t tmp = s.scan_bytes;
    GTA_CUDA(cub::DeviceScan::ExclusiveSum(s.scan_tmp, tmp, s.indeg, s.off, static_cast<int>(n_rows + 1), st));
    if (rev_key_bytes(N, K) == 4)
        rev_scatter_merge<uint32_t>(pruned, N, K, lo, n_rows, src_bits, s, out, st);
    else
        rev_scatter_merge<unsigned long long>(pruned, N, K, lo, n_rows, src_bits, s, out, st);
    GTA_CUDA(cudaGetLastError());
}

// the same merge with its scratch from the call's workspace
void reverse_merge_ws(const uint32_t* pruned, int64_t N, int K, int64_t lo, int64_t n_rows, uint32_t* out, int* err,
                      cudaStream_t st)
{
    const size_t scan_bytes = rev_scan_bytes(n_rows);
    DevBuf<unsigned long long> indeg(static_cast<size_t>(n_rows) + 1, st);
    DevBuf<uint64_t> off(static_cast<size_t>(n_rows) + 1, st);
    DevBuf<uint32_t> cursor(static_cast<size_t>(n_rows), st);
    // every edge of the graph may point into the range: keys for all of them
    DevBuf<uint8_t> keys(static_cast<size_t>(N) * K * rev_key_bytes(N, K), st);
    DevBuf<uint8_t> scan(scan_bytes, st);
    const RevScratch s{indeg.get(), off.get(), cursor.get(), keys.get(), scan.get(), scan_bytes};
    reverse_merge_core(pruned, N, K, lo, n_rows, out, s, err, st);
}

}  // namespace

void reverse_merge(const uint32_t* pruned, int64_t N, int K, uint32_t* out, int* err, cudaStream_t st)
{
    GTA_REQUIRE(N >= 1 && K >= 1 && K <= kMaxM, kInvalid, "reverse: need n >= 1 and K in [1, 128]");
    ProfScope prof("reverse", 32.0 * K * static_cast<double>(N), st);
    reverse_merge_ws(pruned, N, K, 0, N, out, err, st);
}

// ---------------------------------------------------------------- reverse-edge merge without allocation
// Scratch of gta_reverse_merge_noalloc: one file-scope device array, resident on
// every GPU that loads the library until the process exits.  Layout (each region
// 256-byte aligned): in-degrees (u64, rows + 1), offsets (u64, rows + 1),
// cursors (u32, rows), edge keys (up to 8 bytes each, edges), scan temporary
// storage, and the call's device error word.
namespace {
constexpr int64_t kNoAllocMaxRows = 1ll << 17;
constexpr int64_t kNoAllocMaxEdges = 1ll << 21;
constexpr size_t kNoAllocScanBytes = 1u << 20;
constexpr size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }
constexpr size_t kNoAllocIndegOff = 0;
constexpr size_t kNoAllocOffOff = kNoAllocIndegOff + align256(sizeof(unsigned long long) * (kNoAllocMaxRows + 1));
constexpr size_t kNoAllocCursorOff = kNoAllocOffOff + align256(sizeof(uint64_t) * (kNoAllocMaxRows + 1));
constexpr size_t kNoAllocKeysOff = kNoAllocCursorOff + align256(sizeof(uint32_t) * kNoAllocMaxRows);
constexpr size_t kNoAllocScanOff = kNoAllocKeysOff + align256(sizeof(uint64_t) * kNoAllocMaxEdges);
constexpr size_t kNoAllocErrOff = kNoAllocScanOff + kNoAllocScanBytes;
constexpr size_t kNoAllocBytes = kNoAllocErrOff + 256;

static __device__ __align__(256) unsigned char g_rev_scratch[kNoAllocBytes];

// Device address of the scratch array in the current context.  The host-side name
// g_rev_scratch is only a stand-in, so the address is looked up with the caller's
// device current, on every call (a cached address would go stale after a device
// reset or in another context of the same device).
unsigned char* noalloc_scratch()
{
    void* ptr = nullptr;
    GTA_CUDA(cudaGetSymbolAddress(&ptr, g_rev_scratch));
    return static_cast<unsigned char*>(ptr);
}
}  // namespace

int64_t reverse_merge_noalloc_max_rows() { return kNoAllocMaxRows; }
int64_t reverse_merge_noalloc_max_edges() { return kNoAllocMaxEdges; }

void reverse_merge_noalloc(const uint32_t* pruned, int64_t N, int K, uint32_t* out, cudaStream_t st)
{
    GTA_REQUIRE(pruned && out && N >= 1 && K >= 1 && K <= kMaxM, kInvalid,
                "reverse_merge_noalloc: need non-null buffers, n >= 1 and 1 <= k <= 128");
    GTA_REQUIRE(N <= kNoAllocMaxRows && N * K <= kNoAllocMaxEdges, kInvalid,
                "reverse_merge_noalloc: graph too large for the fixed scratch (at most " +
                    std::to_string(kNoAllocMaxRows) + " rows and " + std::to_string(kNoAllocMaxEdges) +
                    " edges); use gta_reverse_merge");
    unsigned char* base = noalloc_scratch();
    const size_t scan_bytes = rev_scan_bytes(N);
    GTA_REQUIRE(scan_bytes <= kNoAllocScanBytes, kInvalid, "reverse_merge_noalloc: scan scratch exceeds its reserve");
    const RevScratch s{reinterpret_cast<unsigned long long*>(base + kNoAllocIndegOff),
                       reinterpret_cast<uint64_t*>(base + kNoAllocOffOff),
                       reinterpret_cast<uint32_t*>(base + kNoAllocCursorOff), base + kNoAllocKeysOff,
                       base + kNoAllocScanOff, kNoAllocScanBytes};
    // the array keeps the previous call's contents: the error word (and, in the core, the
    // counters) start from zero
    int* err = reinterpret_cast<int*>(base + kNoAllocErrOff);
    GTA_CUDA(cudaMemsetAsync(err, 0, sizeof(int), st));
    reverse_merge_core(pruned, N, K, 0, N, out, s, err, st);
    int h = 0;
    GTA_CUDA(cudaMemcpyAsync(&h, err, sizeof(int), cudaMemcpyDeviceToHost, st));
    GTA_CUDA(cudaStreamSynchronize(st));
    GTA_REQUIRE(h == 0, kData, "reverse_merge_noalloc: a neighbour id is outside [0, n)");
}

// ============================================================================ shard variants
void gather_range(const void* X, int dtype, int d, int64_t row0, int64_t n, const int32_t* ids, int64_t n_ids,
                  float* out, cudaStream_t st)
{
    if (n_ids == 0) return;
    const unsigned grid = static_cast<unsigned>((n_ids + 7) / 8);
    switch (dtype) {
        case 0: gather_range_kernel<<<grid, 256, 0, st>>>(static_cast<const float*>(X), d, row0, n, ids, n_ids, out); break;
        case 1: gather_range_kernel<<<grid, 256, 0, st>>>(static_cast<const uint8_t*>(X), d, row0, n, ids, n_ids, out); break;
        case 2: gather_range_kernel<<<grid, 256, 0, st>>>(static_cast<const int8_t*>(X), d, row0, n, ids, n_ids, out); break;
        default: throw Error(kInvalid, "gather_rows: unknown dtype");
    }
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

void gather_i32(const int32_t* src, const int32_t* idx, int64_t n, int32_t* out, cudaStream_t st)
{
    if (n == 0) return;
    gather_i32_kernel<<<blocks_for(n, 256), 256, 0, st>>>(src, idx, n, out);
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}


void centroid_partial(const float* Xs, int64_t n_s, int d, int d_pad, const int32_t* assign, int32_t B, double* sums,
                      long long* counts, int* err, cudaStream_t st)
{
    check_ids(assign, n_s, B, err, st);
    DevBuf<int32_t> keys_out(n_s, st), idx_in(n_s, st), idx_out(n_s, st);
    DevBuf<int64_t> offsets(static_cast<size_t>(B) + 1, st);
    iota_kernel<<<blocks_for(n_s, 256), 256, 0, st>>>(idx_in.get(), n_s);
    count_launches(1);
    int end_bit = 1;
    while ((1ll << end_bit) < B) ++end_bit;
    size_t tmp = 0;
    GTA_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, tmp, assign, keys_out.get(), idx_in.get(), idx_out.get(),
                                             static_cast<int>(n_s), 0, end_bit, st));
    DevBuf<uint8_t> tbuf(tmp, st);
    GTA_CUDA(cub::DeviceRadixSort::SortPairs(tbuf.get(), tmp, assign, keys_out.get(), idx_in.get(), idx_out.get(),
                                             static_cast<int>(n_s), 0, end_bit, st));
    seg_offsets_kernel<<<blocks_for(B + 1, 256), 256, 0, st>>>(keys_out.get(), n_s, B, offsets.get());
    count_launches(1);
    centroid_partial_kernel<<<B, 128, 0, st>>>(Xs, d, d_pad, idx_out.get(), offsets.get(), sums, counts);
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

void centroid_means(const double* sums, const long long* counts, const float* C_in, int32_t B, int d, float* C_out,
                    cudaStream_t st)
{
    centroid_means_kernel<<<blocks_for(static_cast<int64_t>(B) * d, 256), 256, 0, st>>>(sums, counts, C_in, B, d, C_out);
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

void group_rows(const int32_t* bucket, const int32_t* other, int64_t n, int32_t B, int32_t* order, int64_t* offsets,
                cudaStream_t st)
{
    GTA_REQUIRE(n < (1ll << 31) && static_cast<int64_t>(B) * B < (1ll << 32), kInvalid,
                "group_rows: too many rows or buckets");
    DevBuf<uint32_t> keys_in(n, st), keys_out(n, st);
    DevBuf<int32_t> vals_in(n, st);
    group_keys_kernel<<<blocks_for(n, 256), 256, 0, st>>>(bucket, other, n, B, keys_in.get(), vals_in.get());
    count_launches(1);
    int end_bit = 1;
    while ((1ll << end_bit) < static_cast<int64_t>(B) * B) ++end_bit;
    size_t tmp = 0;
    GTA_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, tmp, keys_in.get(), keys_out.get(), vals_in.get(), order,
                                             static_cast<int>(n), 0, end_bit, st));
    DevBuf<uint8_t> tbuf(tmp, st);
    GTA_CUDA(cub::DeviceRadixSort::SortPairs(tbuf.get(), tmp, keys_in.get(), keys_out.get(), vals_in.get(), order,
                                             static_cast<int>(n), 0, end_bit, st));
    seg_offsets_scaled_kernel<<<blocks_for(B + 1, 256), 256, 0, st>>>(keys_out.get(), n, B, offsets);
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

void sanitize_rows(const int32_t* knn, int64_t n_rows, int64_t row0, int64_t N, int M, uint32_t* out, cudaStream_t st)
{
    ProfScope prof("sanitize", 8.0 * M * static_cast<double>(n_rows), st);
    sanitize_kernel<<<blocks_for(n_rows, 8), 256, 0, st>>>(knn, n_rows, row0, N, M, out);
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

void prune_rows(const uint32_t* g, int64_t N, int M, int K, const int32_t* order, int64_t row0, int64_t n_rows,
                uint32_t* out, int* err, cudaStream_t st)
{
    GTA_REQUIRE(M >= 2 && M <= kMaxM && K >= 1 && K <= M, kInvalid, "prune: need 1 <= K <= M <= 128");
    GTA_REQUIRE(row0 >= 0 && n_rows >= 0 && row0 + n_rows <= N, kInvalid, "prune: row range outside the graph");
    ProfScope prof("prune", (4.0 * M * (M + 1) + 4.0 * K) * static_cast<double>(n_rows), st);
    const size_t smem = prune_smem_bytes(M);
    GTA_CUDA(cudaFuncSetAttribute(prune_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    prune_kernel<<<blocks_for(n_rows, kPruneWarps), kPruneWarps * 32, smem, st>>>(g, N, M, K, order, row0, n_rows, out,
                                                                                    err);
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

void reverse_merge_rows(const uint32_t* pruned, int64_t N, int K, int64_t row0, int64_t n_rows, uint32_t* out,
                        int* err, cudaStream_t st)
{
    GTA_REQUIRE(K >= 1 && K <= kMaxM && row0 >= 0 && n_rows >= 1 && row0 + n_rows <= N, kInvalid,
                "reverse: bad row range or K");
    ProfScope prof("reverse", 32.0 * K * static_cast<double>(n_rows), st);
    reverse_merge_ws(pruned, N, K, row0, n_rows, out, err, st);
}

void sort_rows_l2(const float* X, int d, int d_pad, const int32_t* knn, int64_t N, int M, int32_t* out, cudaStream_t st)
{
    GTA_REQUIRE(M >= 1 && M <= kMaxM, kInvalid, "sort_rows: M must be in [1, 128]");
    sort_rows_kernel<<<blocks_for(N, 4), 128, 0, st>>>(X, d, d_pad, knn, N, M, out);
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

void max_sqrt(const float* v, int64_t n, float* out, cudaStream_t st)
{
    GTA_CUDA(cudaMemsetAsync(out, 0, sizeof(float), st));
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>(1184, std::max<int64_t>(1, (n + 255) / 256)));
    max_sqrt_kernel<<<grid, 256, 0, st>>>(v, n, reinterpret_cast<unsigned*>(out));
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

void check_device_error(const int* err, cudaStream_t st, const char* what)
{
    int h = 0;
    GTA_CUDA(cudaMemcpyAsync(&h, err, sizeof(int), cudaMemcpyDeviceToHost, st));
    GTA_CUDA(cudaStreamSynchronize(st));
    if (h != 0) {
        static const char* names[] = {"ok", "TMA tile wait timed out", "pipeline stage wait timed out",
                                      "accumulator wait timed out", "teardown wait timed out", "id out of range",
                                      "unsupported shape", "grid barrier wait timed out",
                                      "search capacity exceeded (visited set or candidates; lower ef)"};
        const char* n = (h >= 0 && h <= 8) ? names[h] : "unknown device error";
        throw Error(h == kDevBadIndex ? kData : (h == kDevOverflow ? kNoMem : kCuda), std::string(what) + ": " + n);
    }
}

}  // namespace gta
