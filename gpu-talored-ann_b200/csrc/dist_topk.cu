// dist_topk.cu -- the distance contraction of the bucketed kNN build on sm_100a.
//
// One CTA = up to 128 A rows (queries) against a contiguous segment of B rows
// (the members of one bucket, or all k-means centroids).  Warp roles:
//   warp 0      TMA producer: 128-row x 128-byte K chunks of B (and of A when
//               A does not stay resident) into a multi-stage smem ring;
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//               (M=128, N=128, fp32 accumulators, two TMEM buffers so the
//               MMA of column tile j+1 overlaps the epilogue of tile j);
//   warps 2..5  epilogue: thread t owns TMEM lane t = A row t; it reads its
//               row's 128 dot products with tcgen05.ld, forms
//               s = ||b||^2 - 2 a.b (the squared distance minus the row
//               constant ||a||^2, the fused ||x||^2+||y||^2-2x.y epilogue),
//               and keeps the row's best entries in a sorted shared-memory
//               list fed through a small unsorted buffer.
// The (rows x segment) score matrix never reaches HBM.
//
// Two CTAs per SM (lists of up to 64 keys): 64-column tiles, two 64-column
// accumulators and the row lists in TMEM (key i of a row in columns
// 128 + 2i / 129 + 2i), a small shared-memory footprint, so that two CTAs --
// two epilogue warps per SM sub-partition -- share each SM and hide each
// other's scan latency.  Longer lists keep one CTA per SM, 128-column tiles
// and the lists in shared memory.
//
// Two modes:
//   exact  (8-bit integer data: kind::i8 MMAs on the u8 rows themselves with
//          int32 accumulation, or kind::f16 with bf16 operands for other 8-bit
//          rows): every product and partial sum is an integer below 2^24, so s
//          is exact; the kernel writes the final top-M (distance, id) lists
//          directly.
//   screen (f32 operands, kind::tf32): s is approximate with a proven error
//          bound; the kernel keeps every column whose approximate s is within
//          the bound of the running M-th, and topk_rerank_kernel recomputes those
//          candidates with the exact fp32 distance and selects the top-M.
//
// Reference behaviour this replaces (paths relative to the reference root):
//   bucketDemo/buildBucket/src/bucket.cu:5471-5484 (cuBLAS dots per bucket) +
//   :4102-4267 block_topK_from_dots_kernel (top-M, self excluded, ascending),
//   :4315-4688 s6 fp16 screen with a strict error bound + exact fp32 rerank,
//   :1230 / :1379-1490 top-2 centroid assignment with exact rerank.
// Ordering: ascending (distance, id); the reference's strict-less insertion
// keeps the earlier candidate on equal distance, which coincides for distinct
// distances (ties within the stated tolerance may order differently).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cfloat>
#include <cmath>
#include <mutex>

#include "common.cuh"
#include "gta_internal.h"
#include "prof.h"

namespace gta {

namespace {

constexpr int kTileM = 128;
constexpr int kTileN = 128;
constexpr uint32_t kTileBytes = 128u * 128u;  // 128 rows x 128 B
constexpr int kThreads = 192;                  // TMA, MMA, 4 epilogue warps
constexpr uint32_t kSmemMax2 = 233472u / 2u - 1024u;  // per CTA when two share an SM
constexpr uint32_t kSmemMax = 232448;         // 227 KB per CTA (opt-in)

struct DistTopkArgs {
    const WorkItem* work;
    const float* a_norm;
    const float* b_norm;
    const int32_t* b_gid;
    const float* b_maxnorm;   // device scalar: max ||b|| (screen margin)
    int32_t k_chunks;
    int32_t m_out;
    int32_t m_sel;
    int32_t L;
    int32_t cap;
    int32_t stages;
    int32_t a_resident;
    int32_t screen;
    float mc1, mc2;           // margin = mc1*|a|*bmax + mc2*(|a|+bmax)^2
    int32_t* out_ids;
    float* out_dists;
    int32_t* cand_cols;       // screen: [a_total x L]
    int32_t* cand_n;          // screen: [a_total], -1 = list overflowed
    unsigned long long* stats;// optional: [passes, flush events, rows]
    int* err;
    uint32_t list_off, buf_off, pn_off, bar_off;
    uint32_t scr_off;           // two-CTA variant: per-lane score scratch
    const float* seed;          // two-CTA exact variant: per-row starting thresholds (see DistTopkProblem)
    int64_t seed_stride;
    const int32_t* partner;
};

constexpr int kBuf = 32;                  // per-row staging buffer (entries)
constexpr uint64_t kEmptyKey = ~0ull;     // list sentinel (its high half decodes to NaN, never a real key)

__device__ __forceinline__ void cmp_swap(uint64_t& a, uint64_t& b)
{
    const uint64_t lo = a < b ? a : b, hi = a < b ? b : a;
    a = lo;
    b = hi;
}

// One bitonic stage of stride S over 32 register keys; the direction of each
// pair comes from the runtime block size (static indices, compact code).
template <int S>
__device__ __forceinline__ void bitonic_stage(uint64_t (&k)[kBuf], int size)
{
#pragma unroll
    for (int i = 0; i < kBuf; ++i) {
        if ((i & S) == 0) {
            const bool up = (i & size) == 0;
            const uint64_t a = k[i], b = k[i + S];
            const bool sw = (a > b) == up;
            k[i] = sw ? b : a;
            k[i + S] = sw ? a : b;
        }
    }
}

// Bitonic sort of 32 keys held in registers, ascending.  The block-size loop
// runs at run time so each stride's stage is emitted once (the flush is the
// largest code on the epilogue path and competes for the instruction cache).
__device__ __forceinline__ void sort32(uint64_t (&k)[kBuf])
{
#pragma unroll 1
    for (int size = 2; size <= kBuf; size <<= 1) {
        if (size > 16) bitonic_stage<16>(k, size);
        if (size > 8) bitonic_stage<8>(k, size);
        if (size > 4) bitonic_stage<4>(k, size);
        if (size > 2) bitonic_stage<2>(k, size);
        bitonic_stage<1>(k, size);
    }
}

// Bitonic merge (half-cleaners with strides 16..1) of 32 keys in registers.
__device__ __forceinline__ void merge32(uint64_t (&k)[kBuf])
{
#pragma unroll
    for (int stride = kBuf / 2; stride > 0; stride >>= 1) {
#pragma unroll
        for (int i = 0; i < kBuf; ++i)
            if ((i & stride) == 0) cmp_swap(k[i], k[i + stride]);
    }
}

// Merge the 32 sorted keys into the row's sorted list of kL keys (shared
// memory, row stride 128), keeping the kL smallest: elementwise minimum with
// the reversed buffer gives a bitonic sequence holding the kL smallest keys,
// and the bitonic half-cleaner cascade sorts it.  Strides of 32 and more run
// on shared memory; each 32-key block then finishes in registers.
template <int kL>
__device__ __forceinline__ void merge_into_list(uint64_t* list, uint64_t (&k)[kBuf])
{
#pragma unroll
    for (int i = 0; i < kBuf; ++i) {
        const uint64_t a = list[(kL - kBuf + i) * 128];
        const uint64_t b = k[kBuf - 1 - i];
        list[(kL - kBuf + i) * 128] = a < b ? a : b;
    }
#pragma unroll
    for (int stride = kL / 2; stride >= kBuf; stride >>= 1) {
#pragma unroll
        for (int i = 0; i < kL; ++i) {
            if ((i & stride) == 0) {
                const uint64_t a = list[i * 128], b = list[(i + stride) * 128];
                if (b < a) {
                    list[i * 128] = b;
                    list[(i + stride) * 128] = a;
                }
            }
        }
    }
#pragma unroll
    for (int blk = 0; blk < kL; blk += kBuf) {
#pragma unroll
        for (int i = 0; i < kBuf; ++i) k[i] = list[(blk + i) * 128];
        merge32(k);
#pragma unroll
        for (int i = 0; i < kBuf; ++i) list[(blk + i) * 128] = k[i];
    }
}

// Flush the row's staging buffer (nb entries, unsorted) into its list.  One
// out-of-line copy (it is large and runs rarely); never called while a
// tcgen05.ld of the caller is still in flight.
template <int kL>
__device__ __noinline__ void flush_row(uint64_t* list, uint64_t* buf, int nb)
{
    uint64_t k[kBuf];
#pragma unroll
    for (int i = 0; i < kBuf; ++i) k[i] = (i < nb) ? buf[i * 128] : kEmptyKey;
    sort32(k);
    merge_into_list<kL>(list, k);
}

// ---- row lists in TMEM (paired epilogue): key i of the row in columns 2i (low
// word) and 2i+1 (high word) of the list's column range.
__device__ __forceinline__ void keys_load32(uint32_t taddr, uint64_t (&k)[32])
{
    uint32_t a[32], b[32];
    tmem_ld_32x32b_x32(taddr, a);
    tmem_ld_32x32b_x32(taddr + 32u, b);
    tmem_ld_wait_regs2x32(a, b);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        k[i] = (static_cast<uint64_t>(a[2 * i + 1]) << 32) | a[2 * i];
        k[16 + i] = (static_cast<uint64_t>(b[2 * i + 1]) << 32) | b[2 * i];
    }
}

__device__ __forceinline__ void keys_store32(uint32_t taddr, const uint64_t (&k)[32])
{
    uint32_t a[32], b[32];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        a[2 * i] = static_cast<uint32_t>(k[i]);
        a[2 * i + 1] = static_cast<uint32_t>(k[i] >> 32);
        b[2 * i] = static_cast<uint32_t>(k[16 + i]);
        b[2 * i + 1] = static_cast<uint32_t>(k[16 + i] >> 32);
    }
    tmem_st_32x32b_x32(taddr, a);
    tmem_st_32x32b_x32(taddr + 32u, b);
}

__device__ __forceinline__ void keys_load16(uint32_t taddr, uint64_t (&k)[16])
{
    uint32_t a[32];
    tmem_ld_32x32b_x32(taddr, a);
    tmem_ld_wait_regs32(a);
#pragma unroll
    for (int i = 0; i < 16; ++i) k[i] = (static_cast<uint64_t>(a[2 * i + 1]) << 32) | a[2 * i];
}

__device__ __forceinline__ void keys_store16(uint32_t taddr, const uint64_t (&k)[16])
{
    uint32_t a[32];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        a[2 * i] = static_cast<uint32_t>(k[i]);
        a[2 * i + 1] = static_cast<uint32_t>(k[i] >> 32);
    }
    tmem_st_32x32b_x32(taddr, a);
}

__device__ __forceinline__ void keys_load8(uint32_t taddr, uint64_t (&k)[8])
{
    uint32_t a[16];
    tmem_ld_32x32b_x16(taddr, a);
    tmem_ld_wait_regs(a);
#pragma unroll
    for (int i = 0; i < 8; ++i) k[i] = (static_cast<uint64_t>(a[2 * i + 1]) << 32) | a[2 * i];
}

__device__ __forceinline__ void keys_store8(uint32_t taddr, const uint64_t (&k)[8])
{
    uint32_t a[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        a[2 * i] = static_cast<uint32_t>(k[i]);
        a[2 * i + 1] = static_cast<uint32_t>(k[i] >> 32);
    }
    tmem_st_32x32b_x16(taddr, a);
}

__device__ __forceinline__ uint64_t min_key(uint64_t a, uint64_t b) { return a < b ? a : b; }
__device__ __forceinline__ float key_dist(uint64_t key) { return key2f(static_cast<uint32_t>(key >> 32)); }

struct ListTail {
    uint64_t last;  // the list's kL-th key
    uint64_t msel;  // its m_sel-th key (screen mode)
};

// Flush the row's staging buffer into its TMEM list of kL (32 or 64) keys,
// keeping the kL smallest (same network as merge_into_list, in registers).
template <int kL, bool kScreen>
__device__ __noinline__ ListTail flush_tmem(uint32_t tl, const uint64_t* buf, int nb, int m_sel)
{
    uint64_t k[kBuf];
#pragma unroll
    for (int i = 0; i < kBuf; ++i) k[i] = (i < nb) ? buf[i * 128] : kEmptyKey;
    sort32(k);
    ListTail t{kEmptyKey, kEmptyKey};
    if constexpr (kL == 32) {
        uint64_t l[32];
        keys_load32(tl, l);
#pragma unroll
        for (int i = 0; i < 32; ++i) l[i] = min_key(l[i], k[31 - i]);
        merge32(l);
        keys_store32(tl, l);
        t.last = l[31];
    } else {
        // 64 keys in eight 8-key blocks of TMEM (16 columns each), a block or a block pair at a time,
        // so that at most the 32 buffer keys and 16 list keys are held at once
#pragma unroll
        for (int j = 0; j < 4; ++j) {  // keys 32 + 8j .. against buffer keys 31 - 8j ..
            uint64_t a[8];
            keys_load8(tl + 64u + 16u * j, a);
#pragma unroll
            for (int i = 0; i < 8; ++i) a[i] = min_key(a[i], k[31 - 8 * j - i]);
            keys_store8(tl + 64u + 16u * j, a);
        }
        tmem_st_wait();
#pragma unroll 1
        for (int j = 0; j < 4; ++j) {  // stride-32 half-cleaner: (8j.., 32 + 8j..)
            uint64_t a[8], b[8];
            keys_load8(tl + 16u * j, a);
            keys_load8(tl + 64u + 16u * j, b);
#pragma unroll
            for (int i = 0; i < 8; ++i) cmp_swap(a[i], b[i]);
            keys_store8(tl + 16u * j, a);
            keys_store8(tl + 64u + 16u * j, b);
        }
        tmem_st_wait();
        // strides 16..1 inside each 32-key half (one copy of the network)
        uint64_t l[32];
#pragma unroll 1
        for (int hh = 0; hh < 2; ++hh) {
            keys_load32(tl + 64u * hh, l);
            merge32(l);
            keys_store32(tl + 64u * hh, l);
        }
        t.last = l[31];
    }
    tmem_st_wait();
    // the m_sel-th key read back from TMEM (a runtime index into a register array would go to local memory)
    if constexpr (kScreen) t.msel = tmem_ld_key(tl + 2u * static_cast<uint32_t>(m_sel - 1));
    return t;
}

// Write a row's final TMEM list (kL keys, ascending): the top-m_out (distance,
// id) pairs, or in screen mode the candidate columns within the margin of the
// m_sel-th (-1 when entries beyond the list may qualify: exact rescan).
// Warp-collective (TMEM loads); lanes without a row write nothing.
template <int kL, bool kScreen>
__device__ __noinline__ void list_out(uint32_t tl, bool row_ok, int64_t arow, float anorm, float margin, int m_out,
                                      int m_sel, int32_t* out_ids, float* out_dists, int32_t* cand_cols, int32_t* cand_n)
{
    uint64_t msel = kEmptyKey;
    if constexpr (kScreen) msel = tmem_ld_key(tl + 2u * static_cast<uint32_t>(m_sel - 1));
    const float bound = (msel != kEmptyKey) ? key_dist(msel) + margin : INFINITY;
    bool overflow = false;
    if constexpr (kScreen) {
        const uint64_t top = tmem_ld_key(tl + 2u * static_cast<uint32_t>(kL - 1));
        overflow = top != kEmptyKey && key_dist(top) <= bound;
        if (row_ok && overflow) cand_n[arow] = -1;  // entries beyond the list may be within the bound
    }
    int nc = 0;
#pragma unroll 1
    for (int blk = 0; blk < kL; blk += 32) {
        uint64_t c[32];
        keys_load32(tl + 2u * static_cast<uint32_t>(blk), c);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const uint64_t key = c[j];
            if constexpr (!kScreen) {
                if (row_ok && blk + j < m_out) {
                    const bool vld = key != kEmptyKey;
                    out_ids[arow * m_out + blk + j] = vld ? static_cast<int32_t>(static_cast<uint32_t>(key)) : -1;
                    out_dists[arow * m_out + blk + j] = vld ? key_dist(key) + anorm : INFINITY;
                }
            } else {
                const bool in = key != kEmptyKey && key_dist(key) <= bound;
                if (row_ok && !overflow && in) cand_cols[arow * kL + blk + j] = static_cast<int32_t>(static_cast<uint32_t>(key));
                nc += in ? 1 : 0;
            }
        }
    }
    if constexpr (kScreen) {
        if (row_ok && !overflow) cand_n[arow] = nc;
    }
}

// v[e] for a runtime e in [0, 16) through a 4-level select tree (static register indices).
__device__ __forceinline__ uint32_t pick16(const uint32_t (&v)[16], int e)
{
    uint32_t l1[8], l2[4], l3[2];
#pragma unroll
    for (int i = 0; i < 8; ++i) l1[i] = (e & 1) ? v[2 * i + 1] : v[2 * i];
#pragma unroll
    for (int i = 0; i < 4; ++i) l2[i] = (e & 2) ? l1[2 * i + 1] : l1[2 * i];
#pragma unroll
    for (int i = 0; i < 2; ++i) l3[i] = (e & 4) ? l2[2 * i + 1] : l2[2 * i];
    return (e & 8) ? l3[1] : l3[0];
}


// Admission threshold of a row: the kL-th key (every finite value passes while
// the list is not full); screen mode also caps it at the m_sel-th + margin.
template <int kL>
__device__ __forceinline__ float row_thr(const uint64_t* list, int m_sel, int screen, float margin)
{
    const uint64_t top = list[(kL - 1) * 128];
    float t = (top == kEmptyKey) ? FLT_MAX : key_dist(top);
    if (screen) {
        const uint64_t mk = list[(m_sel - 1) * 128];
        if (mk != kEmptyKey) t = fminf(t, key_dist(mk) + margin);
    }
    return t;
}

// Column tiles are visited from the tile holding the rows themselves outward
// (t0, t0+1, t0-1, t0+2, ...): with bucket members grouped by locality the
// nearest candidates come first and the row thresholds tighten early.
__device__ __forceinline__ int tile_at(int k, int t0, int n_ct)
{
    if (k == 0) return t0;
    const int right = n_ct - 1 - t0, left = t0, m = min(right, left);
    if (k <= 2 * m) {
        const int j = (k + 1) >> 1;
        return (k & 1) ? t0 + j : t0 - j;
    }
    const int rem = k - 2 * m;
    return right > left ? t0 + m + rem : t0 - m - rem;
}

__device__ __forceinline__ bool mbar_wait_drain(uint32_t bar, uint32_t parity, int* err)
{
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > kWaitBudgetCycles) {
            if (err) atomicCAS(err, 0, kDevTimeoutDrain);
            return false;
        }
    }
    return true;
}

// kV = 1: one CTA per SM, 128-column tiles, row lists in shared memory.
// kV = 2: two CTAs per SM, 64-column tiles, row lists (at most 64 keys) in TMEM.
// kU8: unsigned 8-bit operand rows (the dataset's own bytes) on kind::i8 MMAs: half the MMA
//      instructions and operand bytes of bf16.  The accumulators start at 0x4B000000, so each
//      int32 result reads as the float 2^23 + x.y (exact for 0 <= x.y < 2^23); the scan
//      screens with fl(s - 2^24) against fl(thr - 2^24) (rounding is monotone: no admitted
//      column is missed) and every admitted column's exact score is recomputed and rechecked.
constexpr uint32_t kMagicU8 = 0x4B000000u;  // the float 2^23
template <bool kTF32, int kL, int kV, bool kU8 = false>
__global__ void __launch_bounds__(kThreads, kV)
    dist_topk_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const DistTopkArgs p)
{
    static_assert(kV == 1 || (kV == 2 && kL <= 64), "TMEM row lists hold at most 64 keys");
    static_assert(!kU8 || (kV == 2 && !kTF32), "8-bit operands take the two-CTA exact variant");
    constexpr uint32_t kTmemCols = 256u;
    constexpr int kTN = kV == 1 ? 128 : 64;                            // column tile
    constexpr uint32_t kBChunk = static_cast<uint32_t>(kTN) * 128u;   // bytes of one B K-chunk
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const uint32_t base = smem_u32(smem_raw);
    uint8_t* gbase = smem_raw;
    // the 128-byte-swizzled TMA / UMMA tiles need a 1024-byte aligned base
    if (base & 1023u) {
        if (threadIdx.x == 0) atomicCAS(p.err, 0, kDevBadShape);
        return;
    }

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const WorkItem w = p.work[blockIdx.x];
    const int n_ct = (w.b_rows + kTN - 1) / kTN;
    const int t0 = (w.self_col0 >= 0) ? min(n_ct - 1, w.self_col0 / kTN) : 0;
    const int S = p.stages;
    const uint32_t stage_bytes = p.a_resident ? kBChunk : kBChunk + kTileBytes;
    const uint32_t a_bytes = p.a_resident ? static_cast<uint32_t>(p.k_chunks) * kTileBytes : 0u;
    const uint32_t stage0 = base + a_bytes;
    constexpr int kElemsPerChunk = kU8 ? 128 : (kTF32 ? 32 : 64);

    uint64_t* list = reinterpret_cast<uint64_t*>(gbase + p.list_off);
    uint64_t* buf = reinterpret_cast<uint64_t*>(gbase + p.buf_off);
    float* pn_s = reinterpret_cast<float*>(gbase + p.pn_off);
    uint32_t* id_s = reinterpret_cast<uint32_t*>(gbase + p.pn_off + 4u * 128u * 4u);
    const uint32_t bar0 = base + p.bar_off;
    const uint32_t a_full = bar0 + 8u * (2 * S);
    const uint32_t mma_done = bar0 + 8u * (2 * S + 5);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + p.bar_off + 8u * (2 * S + 6));
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
#define FULL_BAR(s) (bar0 + 8u * (s))
#define EMPTY_BAR(s) (bar0 + 8u * (S + (s)))
#define ACC_FULL(b) (bar0 + 8u * (2 * S + 1 + (b)))
#define ACC_EMPTY(b) (bar0 + 8u * (2 * S + 3 + (b)))

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) { mbar_init(FULL_BAR(s), 1); mbar_init(EMPTY_BAR(s), 1); }
        mbar_init(a_full, 1);
        for (int b = 0; b < 2; ++b) { mbar_init(ACC_FULL(b), 1); mbar_init(ACC_EMPTY(b), 4); }
        mbar_init(mma_done, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    if constexpr (kU8) {
        // both accumulator stages start at the offset (each epilogue warp arms its own lanes)
        if (warp >= 2) {
            uint32_t mg[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) mg[i] = kMagicU8;
            const uint32_t lb = tmem_base + (static_cast<uint32_t>((warp & 3) * 32) << 16);
#pragma unroll
            for (int c = 0; c < 2 * kTN; c += 32) tmem_st_32x32b_x32(lb + static_cast<uint32_t>(c), mg);
            tmem_st_wait();
        }
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
    }

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            tma_prefetch_desc(&tmA);
            tma_prefetch_desc(&tmB);
            if (p.a_resident) {
                mbar_arrive_expect_tx(a_full, a_bytes);
                for (int kc = 0; kc < p.k_chunks; ++kc)
                    tma_load_2d(base + kc * kTileBytes, &tmA, a_full, kc * kElemsPerChunk, w.a_row0);
            }
            int it = 0;
            bool ok = true;
            for (int k = 0; k < n_ct && ok; ++k) {
                const int ct = tile_at(k, t0, n_ct);
                for (int kc = 0; kc < p.k_chunks; ++kc) {
                    const int s = it % S;
                    const uint32_t ph = static_cast<uint32_t>(it / S) & 1u;
                    if (!mbar_wait_backoff(EMPTY_BAR(s), ph ^ 1u, abort_flag, p.err, kDevTimeoutEmpty)) { ok = false; break; }
                    const uint32_t dst = stage0 + static_cast<uint32_t>(s) * stage_bytes;
                    mbar_arrive_expect_tx(FULL_BAR(s), stage_bytes);
                    tma_load_2d(dst, &tmB, FULL_BAR(s), kc * kElemsPerChunk, w.b_row0 + ct * kTN);
                    if (!p.a_resident)
                        tma_load_2d(dst + kBChunk, &tmA, FULL_BAR(s), kc * kElemsPerChunk, w.a_row0);
                    ++it;
                }
            }
            // every issued copy must land before the CTA can exit
            if (p.a_resident) mbar_wait_drain(a_full, 0, p.err);
            for (int j = max(0, it - S); j < it; ++j)
                mbar_wait_drain(FULL_BAR(j % S), static_cast<uint32_t>(j / S) & 1u, p.err);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t idesc = kU8 ? make_idesc_u8(kTileM, kTN) : make_idesc(kTF32 ? 2u : 1u, kTileM, kTN);
            bool ok = true;
            long long mma_wait_acc = 0, mma_wait_full = 0;
            if (p.a_resident) ok = mbar_wait_backoff(a_full, 0, abort_flag, p.err, kDevTimeoutFull);
            int it = 0;
            for (int k = 0; k < n_ct && ok; ++k) {
                const int b = k & 1;
                const uint32_t use = static_cast<uint32_t>(k >> 1);
                const long long m0 = p.stats ? clock64() : 0;
                if (!mbar_wait_backoff(ACC_EMPTY(b), (use & 1u) ^ 1u, abort_flag, p.err, kDevTimeoutAcc)) { ok = false; break; }
                if (p.stats) mma_wait_acc += clock64() - m0;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(b * kTN);
                for (int kc = 0; kc < p.k_chunks; ++kc) {
                    const int s = it % S;
                    const uint32_t ph = static_cast<uint32_t>(it / S) & 1u;
                    const long long m1 = p.stats ? clock64() : 0;
                    if (!mbar_wait_backoff(FULL_BAR(s), ph, abort_flag, p.err, kDevTimeoutFull)) { ok = false; break; }
                    if (p.stats) mma_wait_full += clock64() - m1;
                    tc_fence_after();
                    const uint32_t sb = stage0 + static_cast<uint32_t>(s) * stage_bytes;
                    const uint32_t sa = p.a_resident ? base + static_cast<uint32_t>(kc) * kTileBytes : sb + kBChunk;
                    const uint64_t adesc = smem_desc_sw128(sa);
                    const uint64_t bdesc = smem_desc_sw128(sb);
#pragma unroll
                    for (int k = 0; k < 4; ++k) {  // 4 x 32 B of K per 128-byte chunk
                        if constexpr (kU8) umma_u8(d_tmem, adesc + 2ull * k, bdesc + 2ull * k, idesc);
                        else umma<kTF32>(d_tmem, adesc + 2ull * k, bdesc + 2ull * k, idesc, (kc | k) != 0 ? 1u : 0u);
                    }
                    umma_commit(EMPTY_BAR(s));
                    ++it;
                }
                if (!ok) break;
                umma_commit(ACC_FULL(b));
            }
            umma_commit(mma_done);
            mbar_wait_drain(mma_done, 0, p.err);
            if (p.stats) {
                atomicAdd(&p.stats[6], static_cast<unsigned long long>(mma_wait_acc));
                atomicAdd(&p.stats[7], static_cast<unsigned long long>(mma_wait_full));
            }
        }
    } else if constexpr (kV == 1) {
        // ------------------------------------------------------------ epilogue
        const int q = warp & 3;
        const int r = q * 32 + lane;
        const bool row_ok = r < w.a_rows;
        const bool has_self = w.self_col0 >= 0;   // the tile's rows are also the segment's columns t0*128 + r
        const int64_t arow = static_cast<int64_t>(w.a_row0) + r;
        const float anorm = row_ok ? p.a_norm[arow] : 0.0f;
        float margin = 0.0f;
        if (p.screen) {
            const float an = sqrtf(fmaxf(anorm, 0.0f)), bm = *p.b_maxnorm;
            margin = p.mc1 * an * bm + p.mc2 * (an + bm) * (an + bm);
        }
        uint64_t* my_list = list + r;
        uint64_t* my_buf = buf + r;
#pragma unroll 4
        for (int i = 0; i < kL; ++i) my_list[i * 128] = kEmptyKey;
        float thr = row_ok ? FLT_MAX : -FLT_MAX;
        int nb = 0, n_pass = 0, n_flush = 0;
        bool ok = true;
        const bool st_on = p.stats != nullptr;
        long long cyc_wait = 0, cyc_flush = 0;
        const long long cyc0 = st_on ? clock64() : 0;
        // this warp's copy of the current tile's column norms / ids; lane l stages columns 4l..4l+3,
        // and the values of the next tile are loaded into registers while this one is scanned
        float* pnw = pn_s + q * 128;
        uint32_t* idw = id_s + q * 128;
        float pf_n[4];
        uint32_t pf_i[4];
        auto prefetch_cols = [&](int kk) {
            const int ctn = tile_at(kk, t0, n_ct);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int col = ctn * kTileN + lane * 4 + j;
                const bool cok = col < w.b_rows;
                const int64_t brow = static_cast<int64_t>(w.b_row0) + col;
                pf_n[j] = cok ? p.b_norm[brow] : INFINITY;
                pf_i[j] = (!p.screen && cok && p.b_gid) ? static_cast<uint32_t>(p.b_gid[brow]) : static_cast<uint32_t>(col);
            }
        };
        prefetch_cols(0);
        for (int k = 0; k < n_ct; ++k) {
            const int ct = tile_at(k, t0, n_ct);
            const int b = k & 1;
            const uint32_t use = static_cast<uint32_t>(k >> 1);
            __syncwarp();
            reinterpret_cast<float4*>(pnw)[lane] = make_float4(pf_n[0], pf_n[1], pf_n[2], pf_n[3]);
            reinterpret_cast<uint4*>(idw)[lane] = make_uint4(pf_i[0], pf_i[1], pf_i[2], pf_i[3]);
            __syncwarp();
            if (k + 1 < n_ct) prefetch_cols(k + 1);
            const long long w0 = st_on ? clock64() : 0;
            if (!mbar_wait_warp(ACC_FULL(b), use & 1u, abort_flag, p.err, kDevTimeoutAcc)) { ok = false; break; }
            if (st_on) cyc_wait += clock64() - w0;
            tc_fence_after();
            const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(b * kTileN);
            uint32_t vn[16];
            __syncwarp();
            tmem_ld_32x32b_x16(tbase, vn);
#pragma unroll 1
            for (int c = 0; c < 8; ++c) {  // 8 slices of 16 columns; slice c+1 loads while c is scanned
                uint32_t v[16];
                tmem_ld_wait_regs(vn);
#pragma unroll
                for (int e = 0; e < 16; ++e) v[e] = vn[e];
                if (c + 1 < 8) {
                    __syncwarp();
                    tmem_ld_32x32b_x16(tbase + static_cast<uint32_t>((c + 1) * 16), vn);
                }
                // the row's own column sits at element lane % 16 of slice 2q + lane / 16 of the diagonal tile
                const int self_e = (has_self && k == 0 && c == 2 * q + (lane >> 4)) ? (lane & 15) : -1;
                const uint32_t c0 = static_cast<uint32_t>(ct * kTileN + c * 16);
                const float4* pn4 = reinterpret_cast<const float4*>(pnw + c * 16);
                // branch-free scan: pass mask first, then predicated appends at popcount offsets
                float sv[16];
                uint32_t mask = 0;
#pragma unroll
                for (int e4 = 0; e4 < 4; ++e4) {
                    const float4 n4 = pn4[e4];
                    const float nv[4] = {n4.x, n4.y, n4.z, n4.w};
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int e = e4 * 4 + u;
                        sv[e] = fmaf(-2.0f, __uint_as_float(v[e]), nv[u]);
                        mask |= (sv[e] <= thr) ? (1u << e) : 0u;
                    }
                }
                if (self_e >= 0) mask &= ~(1u << self_e);
                // appends: one warp-uniform iteration per pass of the busiest lane
                const int npass = __popc(mask);
                const int rounds = __reduce_max_sync(0xffffffffu, static_cast<unsigned>(npass));
                if (rounds > 0) {
                    uint32_t kv[16], idv[16];
#pragma unroll
                    for (int e = 0; e < 16; ++e) kv[e] = f2key(sv[e]);
                    if (!p.screen) {
                        const uint4* id4 = reinterpret_cast<const uint4*>(idw + c * 16);
#pragma unroll
                        for (int e4 = 0; e4 < 4; ++e4) {
                            const uint4 x = id4[e4];
                            idv[e4 * 4 + 0] = x.x; idv[e4 * 4 + 1] = x.y; idv[e4 * 4 + 2] = x.z; idv[e4 * 4 + 3] = x.w;
                        }
                    } else {
#pragma unroll
                        for (int e = 0; e < 16; ++e) idv[e] = c0 + e;  // screen mode keys carry the column
                    }
                    uint32_t m = mask;
                    for (int i = 0; i < rounds; ++i) {
                        const int e = __ffs(m) - 1;
                        if (e >= 0) {
                            my_buf[(nb + i) * 128] = (static_cast<uint64_t>(pick16(kv, e)) << 32) | pick16(idv, e);
                            m &= m - 1u;
                        }
                    }
                    nb += npass;
                }
                // warp-wide flush: when any lane may overflow its buffer in the next
                // 16 columns, every lane merges its own buffer
                if (__any_sync(0xffffffffu, nb > kBuf - 16)) {
                    if (c + 1 < 8) tmem_ld_wait_regs(vn);  // no TMEM load in flight across the call
                    const long long f0 = st_on ? clock64() : 0;
                    n_pass += nb;
                    ++n_flush;
                    flush_row<kL>(my_list, my_buf, nb);
                    nb = 0;
                    thr = row_ok ? row_thr<kL>(my_list, p.m_sel, p.screen, margin) : -FLT_MAX;
                    if (st_on) cyc_flush += clock64() - f0;
                }
                __syncwarp();
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(ACC_EMPTY(b));
        }
        if (ok) {
            if (__any_sync(0xffffffffu, nb > 0)) {
                n_pass += nb;
                ++n_flush;
                flush_row<kL>(my_list, my_buf, nb);
                nb = 0;
            }
            if (st_on) {
                if (row_ok) atomicAdd(&p.stats[0], static_cast<unsigned long long>(n_pass));
                if (row_ok) atomicAdd(&p.stats[2], 1ull);
                if (lane == 0) {
                    atomicAdd(&p.stats[1], static_cast<unsigned long long>(n_flush));
                    atomicAdd(&p.stats[3], static_cast<unsigned long long>(cyc_wait));
                    atomicAdd(&p.stats[4], static_cast<unsigned long long>(cyc_flush));
                    atomicAdd(&p.stats[5], static_cast<unsigned long long>(clock64() - cyc0));
                }
            }
        }
        if (ok && row_ok) {
            if (!p.screen) {
                for (int j = 0; j < p.m_out; ++j) {
                    const uint64_t key = my_list[j * 128];
                    const bool v = key != kEmptyKey;
                    p.out_ids[arow * p.m_out + j] = v ? static_cast<int32_t>(static_cast<uint32_t>(key)) : -1;
                    p.out_dists[arow * p.m_out + j] = v ? key_dist(key) + anorm : INFINITY;
                }
            } else {
                const uint64_t mk = my_list[(p.m_sel - 1) * 128];
                const float bound = (mk != kEmptyKey) ? key_dist(mk) + margin : INFINITY;
                const uint64_t top = my_list[(kL - 1) * 128];
                if (top != kEmptyKey && key_dist(top) <= bound) {
                    p.cand_n[arow] = -1;  // entries beyond the list may be within the bound: rescan exactly
                } else {
                    int j = 0;
                    for (int i = 0; i < kL; ++i) {
                        const uint64_t key = my_list[i * 128];
                        if (key == kEmptyKey || key_dist(key) > bound) break;
                        p.cand_cols[arow * kL + j] = static_cast<int32_t>(static_cast<uint32_t>(key));
                        ++j;
                    }
                    p.cand_n[arow] = j;
                }
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue, lists in TMEM
        const int q = warp & 3;  // TMEM lane quarter (a warp reaches lanes 32 * (warp % 4) ..)
        const int r = q * 32 + lane;
        const bool row_ok = r < w.a_rows;
        const bool has_self = w.self_col0 >= 0;
        const int64_t arow = static_cast<int64_t>(w.a_row0) + r;
        const float anorm = row_ok ? p.a_norm[arow] : 0.0f;
        float margin = 0.0f;
        if (kTF32) {
            const float an = sqrtf(fmaxf(anorm, 0.0f)), bm = *p.b_maxnorm;
            margin = p.mc1 * an * bm + p.mc2 * (an + bm) * (an + bm);
        }
        const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
        const uint32_t tl = lane_base + 2u * static_cast<uint32_t>(kTN);  // after the two accumulators
        uint64_t* my_buf = buf + r;
        // per warp: 16 rows of 32 floats (score e of lane l at [e][l]): conflict-free for any e per lane
        float* scr = reinterpret_cast<float*>(gbase + p.scr_off) + q * 512 + lane;
        {
            uint32_t e[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) e[i] = 0xffffffffu;
#pragma unroll
            for (int c = 0; c < 2 * kL; c += 32) tmem_st_32x32b_x32(tl + static_cast<uint32_t>(c), e);
            tmem_st_wait();
        }
        // seeded rows: a known bound on the merged list (exact scores, so seed - ||a||^2 is exact)
        const bool seeded = !kTF32 && p.seed != nullptr;
        float seed_thr = FLT_MAX;
        int32_t skip_partner = -1;
        if (seeded && row_ok) {
            seed_thr = fminf(p.seed[static_cast<int64_t>(p.b_gid[arow]) * p.seed_stride] - anorm, FLT_MAX) + 0.0f;
            skip_partner = p.partner[arow];
        }
        float thr = row_ok ? seed_thr : -FLT_MAX;
        int nb = 0, n_pass = 0, n_flush = 0;
        bool ok = true;
        const bool st_on = p.stats != nullptr;
        long long cyc_wait = 0, cyc_flush = 0;
        const long long cyc0 = st_on ? clock64() : 0;
        // this warp's copy of the current tile's column norms / ids (lane l: columns 2l, 2l+1)
        float* pnw = pn_s + q * 64;
        uint32_t* idw = reinterpret_cast<uint32_t*>(pn_s + 4 * 64) + q * 64;
        float pf_n[2];
        uint32_t pf_i[2];
        auto prefetch_cols = [&](int kk) {
            const int ctn = tile_at(kk, t0, n_ct);
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int col = ctn * kTN + lane * 2 + j;
                const bool cok = col < w.b_rows;
                const int64_t brow = static_cast<int64_t>(w.b_row0) + col;
                pf_n[j] = cok ? p.b_norm[brow] : INFINITY;
                pf_i[j] = (!kTF32 && cok && p.b_gid) ? static_cast<uint32_t>(p.b_gid[brow]) : static_cast<uint32_t>(col);
            }
        };
        // the row's own column: tile t0 + r / 64, slice (r % 64) / 16, element r % 16
        // the row's own column self_col0 + r: its tile, 16-column slice and element
        const int self_col = w.self_col0 + r;
        const int self_ct = has_self ? (self_col / kTN) : -1;
        const int self_c = (self_col % kTN) >> 4;
        const int self_el = self_col & 15;
        prefetch_cols(0);
        for (int k = 0; k < n_ct; ++k) {
            const int ct = tile_at(k, t0, n_ct);
            const int b = k & 1;
            const uint32_t use = static_cast<uint32_t>(k >> 1);
            __syncwarp();
            reinterpret_cast<float2*>(pnw)[lane] = make_float2(pf_n[0], pf_n[1]);
            reinterpret_cast<uint2*>(idw)[lane] = make_uint2(pf_i[0], pf_i[1]);
            __syncwarp();
            if (k + 1 < n_ct) prefetch_cols(k + 1);
            const long long w0 = st_on ? clock64() : 0;
            if (!mbar_wait_warp(ACC_FULL(b), use & 1u, abort_flag, p.err, kDevTimeoutAcc)) { ok = false; break; }
            if (st_on) cyc_wait += clock64() - w0;
            tc_fence_after();
            const uint32_t tbase = lane_base + static_cast<uint32_t>(b * kTN);
            // slices of 16 columns in two register sets: slice c + 1 loads into the other set
            // while c is scanned (no register copies; the slice loop is unrolled)
            uint32_t va[16], vb[16];
            // One slice of 16 columns: scores s = |y|^2 - 2 x.y by packed f32x2 fma, the pass test
            // s <= thr as the sign of thr - s (an IEEE difference is +0 exactly when the two are
            // equal and never takes the wrong sign; thr is never -0), one funnel shift per score
            // to collect the signs: bit 15 - e of `fail` is set where score e lies above thr.
            auto scan_slice = [&](int c, const uint32_t (&v)[16], uint32_t (&nxt)[16], bool nxt_in_flight) {
                const int self_e = (ct == self_ct && c == self_c) ? self_el : -1;
                const uint32_t c0 = static_cast<uint32_t>(ct * kTN + c * 16);
                const ulonglong2* pn2 = reinterpret_cast<const ulonglong2*>(pnw + c * 16);
                // 8-bit operands: v reads as 2^23 + x.y, so the fma below gives fl(s - 2^24)
                const float thr_s = kU8 ? thr - 16777216.0f : thr;
                const unsigned long long thr2 = f2_pack(thr_s, thr_s), m2 = f2_pack(-2.0f, -2.0f);
                // the exact score of element e of this slice from the scratch copy
                auto exact_score = [&](int e) {
                    return kU8 ? fmaf(-2.0f, scr[e * 32] - 8388608.0f, pnw[c * 16 + e]) : scr[e * 32];
                };
                unsigned long long s2[8];
                // four independent 4-bit groups (short dependency chains), then one combine
                uint32_t f4[4];
#pragma unroll
                for (int e4 = 0; e4 < 4; ++e4) {
                    const ulonglong2 n4 = pn2[e4];  // column norms 4 e4 .. 4 e4 + 3, two packed pairs
                    s2[2 * e4] = f2_fma(m2, f2_pack(__uint_as_float(v[4 * e4]), __uint_as_float(v[4 * e4 + 1])), n4.x);
                    s2[2 * e4 + 1] =
                        f2_fma(m2, f2_pack(__uint_as_float(v[4 * e4 + 2]), __uint_as_float(v[4 * e4 + 3])), n4.y);
                    uint32_t g = 0;
#pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        const unsigned long long dd = f2_sub(thr2, s2[2 * e4 + j]);
                        g = __funnelshift_l(static_cast<uint32_t>(dd), g, 1);
                        g = __funnelshift_l(static_cast<uint32_t>(dd >> 32), g, 1);
                    }
                    f4[e4] = g;
                }
                const uint32_t fail = (f4[0] << 12) | (f4[1] << 8) | (f4[2] << 4) | f4[3];
                uint32_t m = ~fail & 0xffffu;  // passes: bit 15 - e for score e
                if (self_e >= 0) m &= ~(1u << (15 - self_e));
                if (__any_sync(0xffffffffu, m != 0u)) {
                    // scores (8-bit operands: the raw 2^23 + x.y) to this lane's scratch, read back by the appends
                    if constexpr (kU8) {
#pragma unroll
                        for (int e = 0; e < 16; ++e) scr[e * 32] = __uint_as_float(v[e]);
                    } else {
#pragma unroll
                        for (int e2 = 0; e2 < 8; ++e2) {
                            float lo, hi;
                            f2_unpack(s2[e2], lo, hi);
                            scr[(2 * e2) * 32] = lo;
                            scr[(2 * e2 + 1) * 32] = hi;
                        }
                    }
                    const int npass = __popc(m);
                    // flush only when a lane's buffer cannot take this slice's passes
                    if (__any_sync(0xffffffffu, nb + npass > kBuf)) {
                        if (nxt_in_flight) tmem_ld_wait_regs(nxt);  // no TMEM load in flight across the call
                        const long long f0 = st_on ? clock64() : 0;
                        n_pass += nb;
                        ++n_flush;
                        const ListTail lt = flush_tmem<kL, kTF32>(tl, my_buf, nb, p.m_sel);
                        nb = 0;
                        if (row_ok) {
                            thr = (lt.last == kEmptyKey) ? FLT_MAX : key_dist(lt.last);
                            if (kTF32 && lt.msel != kEmptyKey) thr = fminf(thr, key_dist(lt.msel) + margin);
                            thr = fminf(thr, seed_thr) + 0.0f;  // -0 -> +0 for the sign test
                        }
                        // this slice's passes against the new threshold
                        m = 0u;
#pragma unroll
                        for (int e = 0; e < 16; ++e) m |= (exact_score(e) <= thr) ? (1u << (15 - e)) : 0u;
                        if (self_e >= 0) m &= ~(1u << (15 - self_e));
                        if (st_on) cyc_flush += clock64() - f0;
                    }
                    int i = nb;
                    while (m != 0u) {  // this lane's passes
                        const int e = 15 - (__ffs(m) - 1);
                        m &= m - 1u;
                        const float se = exact_score(e);
                        if (kU8 && !(se <= thr)) continue;  // admitted by the rounded screen only
                        // seeded rows skip the points of their other bucket (already in that list)
                        if (seeded && p.partner[static_cast<int64_t>(w.b_row0) + c0 + e] == skip_partner) continue;
                        const uint32_t id = kTF32 ? c0 + static_cast<uint32_t>(e) : idw[c * 16 + e];
                        my_buf[i * 128] = (static_cast<uint64_t>(f2key(se)) << 32) | id;
                        ++i;
                    }
                    nb = i;
                }
                __syncwarp();
            };
            constexpr int kSlices = kTN / 16;
            // the stage goes back to the MMA as soon as its last slice is in registers (before
            // that slice is scanned); 8-bit operands first re-arm it with the offset
            auto release_stage = [&]() {
                if constexpr (kU8) {
                    uint32_t mg[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) mg[i] = kMagicU8;
                    __syncwarp();
                    tmem_st_32x32b_x32(tbase, mg);
                    tmem_st_32x32b_x32(tbase + 32u, mg);
                    tmem_st_wait();
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(ACC_EMPTY(b));
            };
            __syncwarp();
            tmem_ld_32x32b_x16(tbase, va);
#pragma unroll
            for (int c = 0; c < kSlices; ++c) {
                const bool more = c + 1 < kSlices;
                if ((c & 1) == 0) {
                    tmem_ld_wait_regs(va);
                    if (more) {
                        __syncwarp();
                        tmem_ld_32x32b_x16(tbase + static_cast<uint32_t>((c + 1) * 16), vb);
                    } else {
                        release_stage();
                    }
                    scan_slice(c, va, vb, more);
                } else {
                    tmem_ld_wait_regs(vb);
                    if (more) {
                        __syncwarp();
                        tmem_ld_32x32b_x16(tbase + static_cast<uint32_t>((c + 1) * 16), va);
                    } else {
                        release_stage();
                    }
                    scan_slice(c, vb, va, more);
                }
            }
        }
        if (ok && __any_sync(0xffffffffu, nb > 0)) {
            n_pass += nb;
            ++n_flush;
            flush_tmem<kL, kTF32>(tl, my_buf, nb, p.m_sel);
            nb = 0;
        }
        if (ok && st_on) {
            if (row_ok) atomicAdd(&p.stats[0], static_cast<unsigned long long>(n_pass));
            if (row_ok) atomicAdd(&p.stats[2], 1ull);
            if (lane == 0) {
                atomicAdd(&p.stats[1], static_cast<unsigned long long>(n_flush));
                atomicAdd(&p.stats[3], static_cast<unsigned long long>(cyc_wait));
                atomicAdd(&p.stats[4], static_cast<unsigned long long>(cyc_flush));
                atomicAdd(&p.stats[5], static_cast<unsigned long long>(clock64() - cyc0));
            }
        }
        if (ok)  // warp-uniform: the TMEM loads inside are warp-collective
            list_out<kL, kTF32>(tl, row_ok, arow, anorm, margin, p.m_out, p.m_sel, p.out_ids, p.out_dists, p.cand_cols,
                                p.cand_n);
    }
#undef FULL_BAR
#undef EMPTY_BAR
#undef ACC_FULL
#undef ACC_EMPTY
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

// --------------------------------------------------------------------------
// exact rerank: one warp per A row, candidates -> exact fp32 distances ->
// bitonic sort of (distance, id) keys -> top-M.  Rows whose screen list
// overflowed rescan their whole segment exactly.
// --------------------------------------------------------------------------
struct RerankArgs {
    const WorkItem* work;
    const void* A;
    const void* B;       // rows read for the exact distances (pitch b_pitch)
    int elem;
    int d, d_pad;        // d_pad: the pitch of A
    int b_pitch;
    const int32_t* b_gid;
    const int32_t* cand_cols;
    const int32_t* cand_n;
    int L;
    int m_out;
    int32_t* out_ids;
    float* out_dists;
};

constexpr int kSortMax = 512;

template <typename T>
__device__ __forceinline__ float exact_dist_row(const float* __restrict__ a, const T* __restrict__ b, int d)
{
    float acc = 0.0f;
    for (int i = 0; i < d; ++i) {
        const float t = a[i] - to_f32(b[i]);
        acc = fmaf(t, t, acc);
    }
    return acc;
}

__device__ __forceinline__ void warp_bitonic_sort(uint64_t* keys, int n, int lane)
{
    for (int k = 2; k <= n; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int t = lane; t < (n >> 1); t += 32) {
                const int i = 2 * j * (t / j) + (t % j);
                const int l = i + j;
                const bool up = (i & k) == 0;
                const uint64_t x = keys[i], y = keys[l];
                if ((x > y) == up) { keys[i] = y; keys[l] = x; }
            }
            __syncwarp();
        }
    }
}

template <typename T>
__global__ void __launch_bounds__(128) topk_rerank_kernel(const RerankArgs p)
{
    extern __shared__ uint8_t sm[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t* keys = reinterpret_cast<uint64_t*>(sm) + warp * kSortMax;
    float* arow_s = reinterpret_cast<float*>(sm + 4 * kSortMax * sizeof(uint64_t)) + warp * p.d_pad;
    const WorkItem w = p.work[blockIdx.x];
    const T* A = static_cast<const T*>(p.A);
    const T* B = static_cast<const T*>(p.B);
    for (int r = warp; r < w.a_rows; r += 4) {
        const int64_t arow = static_cast<int64_t>(w.a_row0) + r;
        for (int i = lane; i < p.d; i += 32) arow_s[i] = to_f32(A[arow * p.d_pad + i]);
        __syncwarp();
        const int n = p.cand_n[arow];
        const int self = (w.self_col0 >= 0) ? w.self_col0 + r : -1;
        if (n >= 0) {
            int np2 = 1;
            while (np2 < n) np2 <<= 1;
            for (int j = lane; j < np2; j += 32) {
                uint64_t key = ~0ull;
                if (j < n) {
                    const int c = p.cand_cols[arow * p.L + j];
                    const int64_t brow = static_cast<int64_t>(w.b_row0) + c;
                    const float dd = exact_dist_row(arow_s, B + brow * p.b_pitch, p.d);
                    const uint32_t id = p.b_gid ? static_cast<uint32_t>(p.b_gid[brow]) : static_cast<uint32_t>(c);
                    key = (static_cast<uint64_t>(f2key(dd)) << 32) | id;
                }
                keys[j] = key;
            }
            __syncwarp();
            warp_bitonic_sort(keys, np2, lane);
            for (int j = lane; j < p.m_out; j += 32) {
                const uint64_t key = j < np2 ? keys[j] : ~0ull;
                const bool v = key != ~0ull;
                p.out_ids[arow * p.m_out + j] = v ? static_cast<int32_t>(static_cast<uint32_t>(key)) : -1;
                p.out_dists[arow * p.m_out + j] = v ? key2f(static_cast<uint32_t>(key >> 32)) : INFINITY;
            }
        } else {
            // full exact rescan of the segment: keys[0..256) = best so far, [256..512) = next chunk
            for (int j = lane; j < kSortMax; j += 32) keys[j] = ~0ull;
            __syncwarp();
            for (int c0 = 0; c0 < w.b_rows; c0 += kSortMax / 2) {
                for (int j = lane; j < kSortMax / 2; j += 32) {
                    const int c = c0 + j;
                    uint64_t key = ~0ull;
                    if (c < w.b_rows && c != self) {
                        const int64_t brow = static_cast<int64_t>(w.b_row0) + c;
                        const float dd = exact_dist_row(arow_s, B + brow * p.b_pitch, p.d);
                        const uint32_t id = p.b_gid ? static_cast<uint32_t>(p.b_gid[brow]) : static_cast<uint32_t>(c);
                        key = (static_cast<uint64_t>(f2key(dd)) << 32) | id;
                    }
                    keys[kSortMax / 2 + j] = key;
                }
                __syncwarp();
                warp_bitonic_sort(keys, kSortMax, lane);
            }
            for (int j = lane; j < p.m_out; j += 32) {
                const uint64_t key = keys[j];
                const bool v = key != ~0ull;
                p.out_ids[arow * p.m_out + j] = v ? static_cast<int32_t>(static_cast<uint32_t>(key)) : -1;
                p.out_dists[arow * p.m_out + j] = v ? key2f(static_cast<uint32_t>(key >> 32)) : INFINITY;
            }
        }
        __syncwarp();
    }
}

// --------------------------------------------------------------------------
// host side
// --------------------------------------------------------------------------
struct Plan {
    int stages = 0, L = 0, a_res = 0, variant = 1;
    uint32_t list_off = 0, buf_off = 0, pn_off = 0, bar_off = 0, scr_off = 0, total = 0;
};

// Row list length: a power of two (the merge network) and at least the
// 32-entry buffer; screen lists keep 16+ entries of headroom beyond M for the
// margin candidates when that fits.  Lists of up to 64 keys take the two-CTA
// variant (64-column tiles, lists in TMEM) when its shared memory fits half an
// SM; otherwise one CTA per SM with 128-column tiles and shared-memory lists.
bool make_plan(int k_chunks, int m, bool screen, Plan& pl)
{
    int L = 32;
    while (L < (screen ? m + 16 : m)) L <<= 1;
    struct Cfg { int a_res, S; };
    const Cfg cfgs1[] = {{1, 4}, {1, 3}, {0, 4}, {0, 3}, {1, 2}, {0, 2}, {1, 1}, {0, 1}};
    const Cfg cfgs2[] = {{1, 4}, {1, 3}, {0, 4}, {0, 3}, {1, 2}, {0, 2}};
    for (; L >= 32 && L >= m; L >>= 1) {
        if (L <= 64) {
            for (const Cfg& c : cfgs2) {
                const uint32_t stage_bytes = (c.a_res ? 0u : kTileBytes) + 64u * 128u;
                uint32_t off = (c.a_res ? static_cast<uint32_t>(k_chunks) * kTileBytes : 0u) + c.S * stage_bytes;
                Plan t;
                t.stages = c.S; t.L = L; t.a_res = c.a_res; t.variant = 2;
                t.buf_off = off; off += static_cast<uint32_t>(kBuf) * 128u * 8u;
                t.pn_off = off; off += 4u * 64u * 4u * 2u;   // per epilogue warp: the tile's norms, then ids
                t.scr_off = off; off += 4u * 32u * 16u * 4u; // per lane: 16 scores
                t.bar_off = off; off += 8u * (2u * c.S + 6u) + 16u;
                t.total = off;
                if (t.total <= kSmemMax2) { pl = t; return true; }
            }
        }
        for (const Cfg& c : cfgs1) {
            const uint32_t stage_bytes = c.a_res ? kTileBytes : 2u * kTileBytes;
            uint32_t off = (c.a_res ? static_cast<uint32_t>(k_chunks) * kTileBytes : 0u) + c.S * stage_bytes;
            Plan t;
            t.stages = c.S; t.L = L; t.a_res = c.a_res; t.variant = 1;
            t.list_off = off; off += static_cast<uint32_t>(L) * 128u * 8u;
            t.buf_off = off; off += static_cast<uint32_t>(kBuf) * 128u * 8u;
            t.pn_off = off; off += 4u * 128u * 4u * 2u;  // per epilogue warp: column norms, then column ids
            t.bar_off = off; off += 8u * (2u * c.S + 6u) + 16u;
            t.total = off;
            if (t.total <= kSmemMax) { pl = t; return true; }
        }
    }
    return false;
}

template <bool kTF32, int kL, int kV, bool kU8 = false>
void launch_dist_topk(const CUtensorMap& tmA, const CUtensorMap& tmB, const DistTopkArgs& a, int n_work,
                      uint32_t smem, cudaStream_t st)
{
    auto fn = dist_topk_kernel<kTF32, kL, kV, kU8>;
    GTA_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    GTA_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
    fn<<<n_work, kThreads, smem, st>>>(tmA, tmB, a);
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

template <bool kTF32>
void launch_dist_topk_L(int L, int variant, const CUtensorMap& tmA, const CUtensorMap& tmB, const DistTopkArgs& a,
                        int n_work, uint32_t smem, cudaStream_t st)
{
    if (variant == 2) {
        switch (L) {
            case 32: launch_dist_topk<kTF32, 32, 2>(tmA, tmB, a, n_work, smem, st); return;
            case 64: launch_dist_topk<kTF32, 64, 2>(tmA, tmB, a, n_work, smem, st); return;
            default: break;
        }
    } else {
        switch (L) {
            case 32: launch_dist_topk<kTF32, 32, 1>(tmA, tmB, a, n_work, smem, st); return;
            case 64: launch_dist_topk<kTF32, 64, 1>(tmA, tmB, a, n_work, smem, st); return;
            case 128: launch_dist_topk<kTF32, 128, 1>(tmA, tmB, a, n_work, smem, st); return;
            default: break;
        }
    }
    throw Error(kInvalid, "dist_topk: unsupported list length");
}

using EncodeFn = PFN_cuTensorMapEncodeTiled_v12000;

EncodeFn get_encode()
{
    static EncodeFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeFn>(ptr);
    });
    GTA_REQUIRE(fn != nullptr, kCuda, "cuTensorMapEncodeTiled is not available from the driver");
    return fn;
}

CUtensorMap make_tmap(const void* base, int elem, int64_t rows, int d_pad, int box_rows = 128)
{
    CUtensorMap m;
    const int esz = elem_bytes(elem);
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(d_pad), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(d_pad) * esz};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / esz), static_cast<cuuint32_t>(box_rows)};
    cuuint32_t estr[2] = {1u, 1u};
    const CUtensorMapDataType ty = elem == kElemU8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                   : elem == kElemBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                       : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    const CUresult r = get_encode()(&m, ty,
                                    2, const_cast<void*>(base), dims, strides, box, estr,
                                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    GTA_REQUIRE(r == CUDA_SUCCESS, kCuda, "cuTensorMapEncodeTiled failed (" + std::to_string(static_cast<int>(r)) + ")");
    return m;
}

}  // namespace

bool dist_topk_seedable(int elem, int d_pad, int m_out)
{
    if (elem == kElemF32 || m_out < 1 || m_out > 64) return false;
    Plan pl;
    return make_plan(d_pad * elem_bytes(elem) / 128, m_out, false, pl) && pl.variant == 2;
}

bool dist_topk_u8_fits(int d_pad, int m_out)
{
    Plan pl;
    return m_out >= 1 && m_out <= 64 && d_pad % 128 == 0 && make_plan(d_pad / 128, m_out, false, pl) && pl.variant == 2;
}

void dist_topk(const DistTopkProblem& pr, cudaStream_t st)
{
    if (pr.n_work == 0) return;
    GTA_REQUIRE(pr.A && pr.B && pr.a_norm && pr.b_norm && pr.work && pr.out_ids && pr.out_dists, kInvalid,
                "dist_topk: null operand");
    const int esz = elem_bytes(pr.elem);
    GTA_REQUIRE((pr.d_pad * esz) % 128 == 0 && pr.d <= pr.d_pad, kInvalid, "dist_topk: rows must be 128-byte multiples");
    GTA_REQUIRE((reinterpret_cast<uintptr_t>(pr.A) & 15) == 0 && (reinterpret_cast<uintptr_t>(pr.B) & 15) == 0,
                kInvalid, "dist_topk: operands must be 16-byte aligned");
    GTA_REQUIRE(pr.m_out >= 1 && pr.m_out <= 256, kInvalid, "dist_topk: list length must be in [1, 256]");
    const bool screen = pr.elem == kElemF32;
    const int k_chunks = pr.d_pad * esz / 128;
    const int m_sel = pr.m_out;  // the row itself is masked in the kernel, not carried in its list
    Plan pl;
    GTA_REQUIRE(pr.m_out <= 128 && make_plan(k_chunks, m_sel, screen, pl), kInvalid,
                "dist_topk: list length too large for shared memory");
    GTA_REQUIRE(!screen || pl.L <= kSortMax, kInvalid, "dist_topk: candidate list too long");

    const CUtensorMap tmA = make_tmap(pr.A, pr.elem, pr.a_total, pr.d_pad);
    const CUtensorMap tmB = make_tmap(pr.B, pr.elem, pr.b_total, pr.d_pad, pl.variant == 2 ? 64 : 128);

    DevBuf<int32_t> cand_cols, cand_n;
    DevBuf<float> bmax;
    if (screen) {
        cand_cols = DevBuf<int32_t>(static_cast<size_t>(pr.a_total) * pl.L, st);
        cand_n = DevBuf<int32_t>(static_cast<size_t>(pr.a_total), st);
        bmax = DevBuf<float>(1, st);
        max_sqrt(pr.b_norm, pr.b_total, bmax.get(), st);
    }
    DistTopkArgs a{};
    a.work = pr.work; a.a_norm = pr.a_norm; a.b_norm = pr.b_norm; a.b_gid = pr.b_gid;
    a.b_maxnorm = screen ? bmax.get() : nullptr;
    a.k_chunks = k_chunks; a.m_out = pr.m_out; a.m_sel = m_sel; a.L = pl.L; a.cap = kBuf;
    a.stages = pl.stages; a.a_resident = pl.a_res; a.screen = screen ? 1 : 0;
    // tf32 screen error bound (operand truncation 2^-10 each, fp32 accumulation with 2 ulp per add,
    // fp32 norms and the fused multiply-add), with a 1.25 safety factor.
    const double d = pr.d;
    const double kacc = pr.screen_k > 0 ? pr.screen_k : pr.d;
    a.mc1 = static_cast<float>(1.25 * 4.0 * (pr.screen_trunc + kacc * std::ldexp(1.0, -22)));
    a.mc2 = static_cast<float>(1.25 * 3.0 * (d + 2.0) * std::ldexp(1.0, -24));
    a.out_ids = pr.out_ids; a.out_dists = pr.out_dists;
    a.cand_cols = cand_cols.get(); a.cand_n = cand_n.get();
    a.err = pr.err;
    a.list_off = pl.list_off; a.buf_off = pl.buf_off; a.pn_off = pl.pn_off; a.bar_off = pl.bar_off;
    a.scr_off = pl.scr_off;
    if (pr.seed) {
        GTA_REQUIRE(!screen && pl.variant == 2 && pr.partner && pr.b_gid, kInvalid,
                    "dist_topk: seeded rows need exact data, lists of at most 64 and partner / id arrays");
        a.seed = pr.seed; a.seed_stride = pr.seed_stride; a.partner = pr.partner;
    }

    {
        ProfScope prof(pr.prof_name, pr.flops, st);
        a.stats = prof.counters(8);
        if (pr.elem == kElemU8) {
            GTA_REQUIRE(pl.variant == 2 && (pl.L == 32 || pl.L == 64), kInvalid,
                        "dist_topk: 8-bit operands need lists of at most 64 in the two-CTA variant");
            if (pl.L == 32) launch_dist_topk<false, 32, 2, true>(tmA, tmB, a, pr.n_work, pl.total, st);
            else launch_dist_topk<false, 64, 2, true>(tmA, tmB, a, pr.n_work, pl.total, st);
        } else if (screen) {
            launch_dist_topk_L<true>(pl.L, pl.variant, tmA, tmB, a, pr.n_work, pl.total, st);
        } else {
            launch_dist_topk_L<false>(pl.L, pl.variant, tmA, tmB, a, pr.n_work, pl.total, st);
        }
    }

    if (screen) {
        RerankArgs r{};
        r.work = pr.work; r.A = pr.A; r.elem = pr.elem; r.d = pr.d; r.d_pad = pr.d_pad;
        r.B = pr.b_exact ? pr.b_exact : pr.B;
        r.b_pitch = pr.b_exact ? pr.b_exact_pitch : pr.d_pad;
        r.b_gid = pr.b_gid; r.cand_cols = cand_cols.get(); r.cand_n = cand_n.get(); r.L = pl.L; r.m_out = pr.m_out;
        r.out_ids = pr.out_ids; r.out_dists = pr.out_dists;
        const size_t smem = 4 * kSortMax * sizeof(uint64_t) + 4 * static_cast<size_t>(pr.d_pad) * sizeof(float);
        GTA_REQUIRE(smem <= kSmemMax, kInvalid, "rerank: dimension too large");
        GTA_CUDA(cudaFuncSetAttribute(topk_rerank_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(smem)));
        ProfScope prof("rerank", 0.0, st);
        topk_rerank_kernel<float><<<pr.n_work, 128, smem, st>>>(r);
        count_launches(1);
        GTA_CUDA(cudaGetLastError());
    }
}

}  // namespace gta
