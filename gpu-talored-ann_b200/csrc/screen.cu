// screen.cu -- the float-row distance screen of the bucketed kNN build on sm_100a.
//
// For float rows the exact distance of the build is the ascending-dimension fp32 fmaf chain
// (the reference's exact rerank, bucketDemo/buildBucket/src/bucket.cu:4350-4363 s6_dot_rows),
// which no tensor-core contraction reproduces.  The build screens on the tensor cores and
// recomputes the survivors exactly, as the reference's s6 path does (bucket.cu:4458
// s6_scan_kernel: fp16 screen with a strict error bound; :4604 s6_rerank_kernel: exact
// rerank):
//
//   screen_kernel   per A row, the kL smallest approximate distances (kL = 128 or 256 > M),
//                   keeping every B column within a proven margin of the row's M-th;
//   rerank_kernel   exact distances of the first M keys, whose largest (E) bounds the row's
//                   exact M-th; then of the keys whose approximate distance may lie within E
//                   plus the one-sided error bound; the top-M.  Only when even the list's last
//                   key may lie within that bound (columns beyond the list may qualify) is the
//                   row's whole segment rescanned exactly (rescan_kernel).
//
// Operands: each row x is scaled by a power of two S (exact; S = 2^floor(log2(2^15 / max ||x||)),
// so every coordinate stays below 2^15) and split into fp16 parts hi = rn(S x) and
// lo = rn(S x - hi).  The split screen's kind::f16 MMAs form hi.hi + hi.lo + lo.hi (the dropped
// lo.lo and the rounding of lo are below 3 * 2^-22 of |x||y|); the one-part screen forms hi.hi
// alone (rounding 2^-10 per element, a wider margin, a third of the MMAs).  Products of fp16
// values are exact in fp32, so the error left is the parts' rounding and the fp32
// accumulation, both bounded in the margin.  screen_knn picks the mode per wave (long rows
// start one-part, a wave with many rescans hands the rest to the split screen).
//
// Long segments run as column chunks sized for the L2, in waves; a pilot wave seeds their rows
// with an exact bound on the M-th distance, and each wave's lists tighten it (see screen_knn).
//
// CTA = 128 A rows against one bucket segment, one CTA per SM:
//   warp 0      TMA producer: per K chunk of 64 fp16 (32 with the correction accumulator), the
//               A and B parts into a 4-6 stage ring;
//   warp 1      TMEM allocator (all 512 columns) + single-thread tcgen05.mma issuer into two
//               128-column accumulators (column tile j+1 overlaps the epilogue of tile j);
//   warps 2..5  epilogue: thread t owns TMEM lane t = A row t.  Scores of 16 columns at a time
//               (tcgen05.ld), approximate distance S^2 (||b||^2 - 2 a.b + ||a||^2) by packed
//               f32x2 arithmetic, the admission test by sign bits, admitted columns staged in
//               shared memory and merged (bitonic) into the row's sorted list of kL 32-bit keys
//               kept in TMEM columns 256.. (key = distance code << col_bits | column).
// The 16-bit distance code covers the 31 binades below 4 (S max ||x||)^2 (no scaled distance is
// larger) with 11 mantissa bits: the distance's float bits above that base, rounded UP to a
// multiple of 2^12; everything below the base codes as 0 and the top code (0xFFFE) decodes as
// +inf (0xFFFF is the sentinel's).
// decode(code) >= the distance > decode(code - 1), and the admission threshold and the
// rerank's bound are taken from decoded codes, so every test errs toward admitting.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "gta.h"
#include "gta_internal.h"
#include "prof.h"

namespace gta {

namespace {

constexpr int kSThreads = 192;
constexpr int kSTile = 128;                    // A rows per CTA and B columns per tile
constexpr uint32_t kSChunk = 128u * 128u;      // one 128-row x 128-byte part chunk (64 fp16)
constexpr int kSBuf = 32;                      // per-row staging buffer (keys)
constexpr uint32_t kSEmpty = 0xFFFFFFFFu;      // list sentinel (above every real key)
constexpr uint32_t kSListCol = 256u;           // first TMEM column of the row lists
constexpr uint32_t kSSmemMax = 232448u;        // 227 KB per CTA

struct ScreenArgs {
    const WorkItem* work;
    const float* norm;         // exact ||x||^2 of the pool rows (A and B are the same pool)
    const float* maxnorm;      // device scalar: max ||x|| over the pool
    int32_t k_chunks;          // 128-byte chunks per part (d16 / 64)
    int32_t part_stride;       // fp16 elements from a row's hi part to its lo part
    int32_t m_sel;             // the list position that sets the bound (M)
    int32_t stages;
    int32_t col_bits;          // 16 or 17
    float mc1, mc2;            // margin = mc1 |a| bmax + mc2 (|a| + bmax)^2 (unscaled)
    const float* seed;         // [seeded rows] a known bound on the row's exact M-th (unscaled); item
                               // rows with pad2 >= 0 read seed[pad2 + r]
    int32_t* cand_cols;        // [item rows x L] the row's list: keys (code << col_bits | column), ascending
    int32_t* cand_n;           // [item rows] keys in the row's list
    unsigned long long* stats; // optional: the library's eight profile counters
    int* err;
    uint32_t buf_off, pn_off, bar_off;
    uint32_t stg_off;          // kCorr: the drained tile (128 columns x 128 rows of fp32)
};

// the largest real code (decodes as +inf); code 0xFFFF only appears in the sentinel key
constexpr uint32_t kCodeTop = 0xFFFEu;

// The float bits every distance code counts from: 31 binades below 4 (S bmax)^2.
__device__ __forceinline__ uint32_t code_base(float sc, float bm)
{
    const float top = 4.0f * (sc * bm) * (sc * bm);
    const uint32_t tb = __float_as_uint(top) + (1u << 23);  // one binade of headroom for rounding
    return tb > (31u << 23) ? tb - (31u << 23) : 0u;
}
__device__ __forceinline__ uint32_t dist_code(float dist, uint32_t base)
{
    const uint32_t bits = __float_as_uint(fmaxf(dist, 0.0f));
    if (bits <= base) return 0u;
    const uint32_t c = (bits - base + 4095u) >> 12;
    return c < kCodeTop ? c : kCodeTop;
}
__device__ __forceinline__ float code_value(uint32_t code, uint32_t base)
{
    return code >= kCodeTop ? INFINITY : __uint_as_float(base + (code << 12));
}

// The power-of-two scale of the operands (the same in the conversion and the epilogue).
__device__ __forceinline__ float screen_scale(float maxnorm)
{
    if (!(maxnorm > 0.0f) || !(maxnorm < FLT_MAX)) return 1.0f;
    const int e = static_cast<int>(floorf(log2f(32768.0f / maxnorm)));
    return exp2f(static_cast<float>(max(-60, min(60, e))));
}

__device__ __forceinline__ uint32_t tmem_ld1(uint32_t taddr)
{
    uint32_t v;
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];\n\t"
                 "tcgen05.wait::ld.sync.aligned;"
                 : "=r"(v)
                 : "r"(taddr)
                 : "memory");
    return v;
}

__device__ __forceinline__ void cswap(uint32_t& a, uint32_t& b)
{
    const uint32_t lo = min(a, b), hi = max(a, b);
    a = lo;
    b = hi;
}

// bitonic half-cleaners of strides 16..1 over 32 register keys (a bitonic block -> ascending)
__device__ __forceinline__ void merge32u(uint32_t (&k)[32])
{
#pragma unroll
    for (int s = 16; s > 0; s >>= 1)
#pragma unroll
        for (int i = 0; i < 32; ++i)
            if ((i & s) == 0) cswap(k[i], k[i + s]);
}

// full bitonic sort of 32 register keys, ascending
__device__ __forceinline__ void sort32u(uint32_t (&k)[32])
{
#pragma unroll
    for (int size = 2; size <= 32; size <<= 1)
#pragma unroll
        for (int s = size >> 1; s > 0; s >>= 1)
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if ((i & s) == 0) {
                    const bool up = (i & size) == 0;
                    uint32_t& a = k[i];
                    uint32_t& b = k[i + s];
                    const uint32_t lo = min(a, b), hi = max(a, b);
                    a = up ? lo : hi;
                    b = up ? hi : lo;
                }
}

// Merge a row's staged keys (nb of them, unsorted, buf[i * 128]) into its ascending TMEM list
// of kL keys, keeping the kL smallest: the list with its last 32 keys replaced by the
// element-wise minimum against the reversed sorted buffer is bitonic and holds them; the
// half-cleaner cascade sorts it.  A pair of blocks that both still hold the untouched sorted
// list needs no exchange, so each half-cleaner pass visits one block pair per sub-array.
// Warp-collective (TMEM loads / stores); never called with a TMEM load of the caller in flight.
template <int kL>
__device__ __noinline__ void flush_list(uint32_t tl, const uint32_t* buf, int nb)
{
    uint32_t k[32], a[32], b[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) k[i] = (i < nb) ? buf[i * 128] : kSEmpty;
    sort32u(k);
    tmem_ld_32x32b_x32(tl + static_cast<uint32_t>(kL - 32), a);
    tmem_ld_wait_regs32(a);
#pragma unroll
    for (int i = 0; i < 32; ++i) a[i] = min(a[i], k[31 - i]);
    tmem_st_32x32b_x32(tl + static_cast<uint32_t>(kL - 32), a);
    tmem_st_wait();
#pragma unroll 1
    for (int s = kL / 2; s >= 32; s >>= 1) {
#pragma unroll 1
        for (int base = 0; base < kL; base += 2 * s) {
            const uint32_t lo_blk = tl + static_cast<uint32_t>(base + s - 32);
            const uint32_t hi_blk = tl + static_cast<uint32_t>(base + 2 * s - 32);
            tmem_ld_32x32b_x32(lo_blk, a);
            tmem_ld_32x32b_x32(hi_blk, b);
            tmem_ld_wait_regs2x32(a, b);
#pragma unroll
            for (int i = 0; i < 32; ++i) cswap(a[i], b[i]);
            tmem_st_32x32b_x32(lo_blk, a);
            tmem_st_32x32b_x32(hi_blk, b);
            tmem_st_wait();
        }
    }
#pragma unroll 1
    for (int blk = 0; blk < kL; blk += 32) {
        tmem_ld_32x32b_x32(tl + static_cast<uint32_t>(blk), a);
        tmem_ld_wait_regs32(a);
        merge32u(a);
        tmem_st_32x32b_x32(tl + static_cast<uint32_t>(blk), a);
    }
    tmem_st_wait();
}

// Column tiles of an item: the rows' own tile first (the nearest candidates: its threshold
// tightens early), then every other tile in ascending order -- the CTAs of one bucket, which run
// side by side, then read the same B tiles at about the same time and share them in L2.
__device__ __forceinline__ int tile_order(int k, int t0, int n_ct)
{
    (void)n_ct;
    if (k == 0) return t0;
    return k <= t0 ? k - 1 : k;
}

__device__ __forceinline__ bool drain_wait(uint32_t bar, uint32_t parity, int* err)
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

__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b)
{
    unsigned long long r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

// Shared-memory matrix descriptor of a K-major tile of 64-byte rows with the 64-byte swizzle
// written by TMA (8-row atoms, 512 B apart).
__device__ __forceinline__ uint64_t smem_desc_sw64(uint32_t saddr)
{
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);   // start address
    d |= static_cast<uint64_t>(1u) << 16;                  // leading byte offset (unused for swizzled K-major)
    d |= static_cast<uint64_t>(512u >> 4) << 32;           // stride byte offset: 8 rows x 64 B
    d |= static_cast<uint64_t>(1u) << 46;                  // descriptor version (sm_100)
    d |= static_cast<uint64_t>(4u) << 61;                  // layout: 64-byte swizzle
    return d;
}

// Wait for this thread's outstanding tcgen05.ld into two 16-register arrays (in/out operands keep
// every use of them below the wait).
__device__ __forceinline__ void tmem_ld_wait_2x16(uint32_t (&a)[16], uint32_t (&b)[16])
{
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]), "+r"(a[6]), "+r"(a[7]),
                   "+r"(a[8]), "+r"(a[9]), "+r"(a[10]), "+r"(a[11]), "+r"(a[12]), "+r"(a[13]), "+r"(a[14]), "+r"(a[15]),
                   "+r"(b[0]), "+r"(b[1]), "+r"(b[2]), "+r"(b[3]), "+r"(b[4]), "+r"(b[5]), "+r"(b[6]), "+r"(b[7]),
                   "+r"(b[8]), "+r"(b[9]), "+r"(b[10]), "+r"(b[11]), "+r"(b[12]), "+r"(b[13]), "+r"(b[14]), "+r"(b[15])
                 :
                 : "memory");
}

// kCorr (two operand parts, long rows): the small products hi.lo + lo.hi accumulate in their own
// TMEM accumulator (columns 128..255) and only hi.hi in the main one (columns 0..127), so the
// main accumulator's rounding grows with d products instead of 3 d; the epilogue adds the two.
// Both halves of one tile's accumulator pair fill the 256 columns, so the tile is not double
// buffered (the MMA of the next tile waits until the epilogue holds the last slice in registers).
template <int kL, bool kSplit, bool kCorr>
__global__ void __launch_bounds__(kSThreads, 1) screen_kernel(const __grid_constant__ CUtensorMap tm, const ScreenArgs p)
{
    static_assert(!kCorr || kSplit, "the correction accumulator holds the lo products");
    constexpr int kParts = kSplit ? 2 : 1;
    // operand chunks of 64 fp16 (128-byte swizzle) or, kCorr, 32 fp16 (64-byte swizzle: smaller
    // stages leave room for the drained tile)
    constexpr int kChunkElems = kCorr ? 32 : 64;
    constexpr uint32_t kPartChunk = 128u * static_cast<uint32_t>(kChunkElems) * 2u;
    constexpr uint32_t kStageBytes = 2u * kParts * kPartChunk;  // A parts then B parts
    constexpr uint32_t kTmemCols = 512u;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const uint32_t base = smem_u32(smem_raw);
    if (base & 1023u) {  // the 128-byte-swizzled TMA / UMMA tiles need a 1024-byte aligned base
        if (threadIdx.x == 0) atomicCAS(p.err, 0, kDevBadShape);
        return;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const WorkItem w = p.work[blockIdx.x];
    const int n_ct = (w.b_rows + kSTile - 1) / kSTile;
    // the column tile of the rows themselves first (clamped into the item's columns)
    const int t0 = (w.has_self & 1) ? max(0, min(n_ct - 1, w.self_col0 / kSTile)) : 0;
    const int S = p.stages;
    uint32_t* buf = reinterpret_cast<uint32_t*>(smem_raw + p.buf_off);
    float* pn_s = reinterpret_cast<float*>(smem_raw + p.pn_off);
    const uint32_t bar0 = base + p.bar_off;
    const uint32_t mma_done = bar0 + 8u * (2 * S + 4);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem_raw + p.bar_off + 8u * (2 * S + 5));
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
#define S_FULL(s) (bar0 + 8u * (s))
#define S_EMPTY(s) (bar0 + 8u * (S + (s)))
#define S_ACC_FULL(b) (bar0 + 8u * (2 * S + (b)))
#define S_ACC_EMPTY(b) (bar0 + 8u * (2 * S + 2 + (b)))

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(S_FULL(s), 1);
            mbar_init(S_EMPTY(s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(S_ACC_FULL(b), 1);
            mbar_init(S_ACC_EMPTY(b), 4);
        }
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

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            tma_prefetch_desc(&tm);
            int it = 0;
            bool ok = true;
            for (int k = 0; k < n_ct && ok; ++k) {
                const int ct = tile_order(k, t0, n_ct);
                for (int kc = 0; kc < p.k_chunks; ++kc) {
                    const int s = it % S;
                    const uint32_t ph = static_cast<uint32_t>(it / S) & 1u;
                    if (!mbar_wait_backoff(S_EMPTY(s), ph ^ 1u, abort_flag, p.err, kDevTimeoutEmpty)) {
                        ok = false;
                        break;
                    }
                    const uint32_t dst = base + static_cast<uint32_t>(s) * kStageBytes;
                    mbar_arrive_expect_tx(S_FULL(s), kStageBytes);
#pragma unroll
                    for (int q = 0; q < kParts; ++q) {
                        const int x = q * p.part_stride + kc * kChunkElems;
                        tma_load_2d(dst + static_cast<uint32_t>(q) * kPartChunk, &tm, S_FULL(s), x, w.a_row0);
                        tma_load_2d(dst + static_cast<uint32_t>(kParts + q) * kPartChunk, &tm, S_FULL(s), x,
                                    w.b_row0 + ct * kSTile);
                    }
                    ++it;
                }
            }
            // every issued copy lands before the CTA can exit
            for (int j = max(0, it - S); j < it; ++j) drain_wait(S_FULL(j % S), static_cast<uint32_t>(j / S) & 1u, p.err);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t idesc = make_idesc(0u, kSTile, kSTile);  // fp16 x fp16 -> fp32
            auto mma = [&](uint32_t d, uint64_t a, uint64_t b, uint32_t acc) { umma<false>(d, a, b, idesc, acc); };
            bool ok = true;
            long long wait_acc = 0, wait_full = 0;
            int it = 0;
            for (int k = 0; k < n_ct && ok; ++k) {
                const int b = kCorr ? 0 : (k & 1);
                const uint32_t use = static_cast<uint32_t>(kCorr ? k : (k >> 1));
                const long long m0 = p.stats ? clock64() : 0;
                if (!mbar_wait_backoff(S_ACC_EMPTY(b), (use & 1u) ^ 1u, abort_flag, p.err, kDevTimeoutAcc)) break;
                if (p.stats) wait_acc += clock64() - m0;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(b * kSTile);
                for (int kc = 0; kc < p.k_chunks; ++kc) {
                    const int s = it % S;
                    const uint32_t ph = static_cast<uint32_t>(it / S) & 1u;
                    const long long m1 = p.stats ? clock64() : 0;
                    if (!mbar_wait_backoff(S_FULL(s), ph, abort_flag, p.err, kDevTimeoutFull)) {
                        ok = false;
                        break;
                    }
                    if (p.stats) wait_full += clock64() - m1;
                    tc_fence_after();
                    const uint32_t sa = base + static_cast<uint32_t>(s) * kStageBytes;
                    auto desc = [](uint32_t addr) { return kCorr ? smem_desc_sw64(addr) : smem_desc_sw128(addr); };
                    const uint64_t ah = desc(sa), bh = desc(sa + kParts * kPartChunk);
#pragma unroll
                    for (int kk = 0; kk < kChunkElems / 16; ++kk) {  // 16 fp16 of K per MMA
                        mma(d_tmem, ah + 2ull * kk, bh + 2ull * kk, (kc | kk) != 0 ? 1u : 0u);
                        if constexpr (kSplit) {
                            const uint64_t al = desc(sa + kPartChunk), bl = desc(sa + 3u * kPartChunk);
                            const uint32_t c_tmem = kCorr ? tmem_base + static_cast<uint32_t>(kSTile) : d_tmem;
                            mma(c_tmem, ah + 2ull * kk, bl + 2ull * kk, (!kCorr || (kc | kk) != 0) ? 1u : 0u);
                            mma(c_tmem, al + 2ull * kk, bh + 2ull * kk, 1u);
                        }
                    }
                    umma_commit(S_EMPTY(s));
                    ++it;
                }
                if (!ok) break;
                umma_commit(S_ACC_FULL(b));
            }
            umma_commit(mma_done);
            drain_wait(mma_done, 0, p.err);
            if (p.stats) {
                atomicAdd(&p.stats[6], static_cast<unsigned long long>(wait_acc));
                atomicAdd(&p.stats[7], static_cast<unsigned long long>(wait_full));
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue
        const int q = warp & 3;  // TMEM lane quarter of this warp
        const int r = q * 32 + lane;
        const bool row_ok = r < w.a_rows;
        const int64_t arow = static_cast<int64_t>(w.a_row0) + r;
        const float bm = *p.maxnorm;
        const float sc = screen_scale(bm);
        const float s2 = sc * sc;
        const float anorm = row_ok ? p.norm[arow] : 0.0f;
        const float an_s = s2 * anorm;
        const float an = sqrtf(fmaxf(anorm, 0.0f));
        const float margin = s2 * (p.mc1 * an * bm + p.mc2 * (an + bm) * (an + bm));
        const uint32_t code_b = code_base(sc, bm);
        const uint32_t col_mask = (1u << p.col_bits) - 1u;
        const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
        const uint32_t tl = lane_base + kSListCol;
        uint32_t* my_buf = buf + r;
        {
            uint32_t e[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) e[i] = kSEmpty;
#pragma unroll
            for (int c = 0; c < kL; c += 32) tmem_st_32x32b_x32(tl + static_cast<uint32_t>(c), e);
            tmem_st_wait();
        }
        // admission threshold on the approximate (scaled) distance; rows past the tile admit nothing
        float thr = row_ok ? FLT_MAX : -FLT_MAX;
        // a seeded row needs only the columns whose exact distance may lie within the seed: their
        // approximate distance is at most the seed plus the one-sided error (half the margin)
        float seed_thr = FLT_MAX;
        if (row_ok && w.pad2 >= 0) {
            const float sd = p.seed[static_cast<int64_t>(w.pad2) + r];
            if (sd < FLT_MAX) seed_thr = fmaf(s2, sd, 0.5f * margin);
            thr = seed_thr;
        }
        auto decode = [&](uint32_t code) { return code_value(code, code_b); };
        auto refresh_thr = [&]() {
            const uint32_t kl = tmem_ld1(tl + static_cast<uint32_t>(kL - 1));
            const uint32_t km = tmem_ld1(tl + static_cast<uint32_t>(p.m_sel - 1));
            float t = kl == kSEmpty ? FLT_MAX : decode(kl >> p.col_bits);
            if (km != kSEmpty) t = fminf(t, decode(km >> p.col_bits) + margin);
            if (row_ok) thr = fminf(t, seed_thr);
        };
        int nb = 0, n_pass = 0, n_flush = 0;
        bool ok = true;
        const bool st_on = p.stats != nullptr;
        long long cyc_wait = 0, cyc_flush = 0;
        const long long cyc0 = st_on ? clock64() : 0;
        // this warp's copy of the tile's scaled column norms (lane l stages columns 4l .. 4l + 3)
        float* pnw = pn_s + q * kSTile;
        float pf[4];
        auto prefetch_cols = [&](int kk) {
            const int ctn = tile_order(kk, t0, n_ct);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int col = ctn * kSTile + lane * 4 + j;
                pf[j] = col < w.b_rows ? s2 * p.norm[static_cast<int64_t>(w.b_row0) + col] : INFINITY;
            }
        };
        // the row's own column, when it lies in this item's columns
        const int self_col =
            ((w.has_self & 1) && w.self_col0 + r >= 0 && w.self_col0 + r < w.b_rows) ? w.self_col0 + r : -1;
        const int64_t irow = static_cast<int64_t>(w.item_row0) + r;
        const int self_ct = self_col >= 0 ? self_col / kSTile : -1;
        const int self_c = (self_col % kSTile) >> 4;
        const int self_el = self_col & 15;
        const unsigned long long an2 = f2_pack(an_s, an_s), m2 = f2_pack(-2.0f, -2.0f);
        prefetch_cols(0);
        for (int k = 0; k < n_ct && ok; ++k) {
            const int ct = tile_order(k, t0, n_ct);
            const int b = kCorr ? 0 : (k & 1);
            const uint32_t use = static_cast<uint32_t>(kCorr ? k : (k >> 1));
            __syncwarp();
            reinterpret_cast<float4*>(pnw)[lane] = make_float4(pf[0], pf[1], pf[2], pf[3]);
            __syncwarp();
            if (k + 1 < n_ct) prefetch_cols(k + 1);
            const long long w0 = st_on ? clock64() : 0;
            if (!mbar_wait_warp(S_ACC_FULL(b), use & 1u, abort_flag, p.err, kDevTimeoutAcc)) {
                ok = false;
                break;
            }
            if (st_on) cyc_wait += clock64() - w0;
            tc_fence_after();
            const uint32_t tbase = lane_base + static_cast<uint32_t>(b * kSTile);
            const uint32_t corr_base = lane_base + static_cast<uint32_t>(kSTile);  // kCorr: the correction accumulator
            uint32_t va[16], vb[16], ca[16], cb[16];
            // load slice c (and, kCorr, its corrections); wait for it (and add the corrections)
            auto ld_slice = [&](int c, uint32_t (&m)[16], uint32_t (&cr)[16]) {
                tmem_ld_32x32b_x16(tbase + static_cast<uint32_t>(c * 16), m);
                if constexpr (kCorr) tmem_ld_32x32b_x16(corr_base + static_cast<uint32_t>(c * 16), cr);
            };
            auto wait_slice = [&](uint32_t (&m)[16], uint32_t (&cr)[16]) {
                if constexpr (kCorr) {
                    tmem_ld_wait_2x16(m, cr);
#pragma unroll
                    for (int e = 0; e < 16; ++e) m[e] = __float_as_uint(__uint_as_float(m[e]) + __uint_as_float(cr[e]));
                } else {
                    tmem_ld_wait_regs(m);
                }
            };
            // one slice of 16 columns: approximate distances by packed f32x2 arithmetic, the
            // admission test dist <= thr as the sign of thr - dist (an IEEE difference is +0 exactly
            // on equality and never takes the wrong sign), then this lane's admitted columns
            auto scan_slice = [&](int c, const uint32_t (&v)[16], uint32_t (&nxt)[16], uint32_t (&nxtc)[16],
                                  bool nxt_in_flight) {
                const int self_e = (ct == self_ct && c == self_c) ? self_el : -1;
                const uint32_t c0 = static_cast<uint32_t>(ct * kSTile + c * 16);
                const ulonglong2* pn2 = reinterpret_cast<const ulonglong2*>(pnw + c * 16);
                float dist[16];
                uint32_t m = 0;
                {
                    const unsigned long long thr2 = f2_pack(thr, thr);
#pragma unroll
                    for (int e4 = 0; e4 < 4; ++e4) {
                        const ulonglong2 n4 = pn2[e4];
                        const unsigned long long sa = f2_fma(m2, f2_pack(__uint_as_float(v[4 * e4]), __uint_as_float(v[4 * e4 + 1])), n4.x);
                        const unsigned long long sb = f2_fma(m2, f2_pack(__uint_as_float(v[4 * e4 + 2]), __uint_as_float(v[4 * e4 + 3])), n4.y);
                        const unsigned long long da = f2_add(sa, an2), db = f2_add(sb, an2);
                        f2_unpack(da, dist[4 * e4], dist[4 * e4 + 1]);
                        f2_unpack(db, dist[4 * e4 + 2], dist[4 * e4 + 3]);
                        const unsigned long long ga = f2_sub(thr2, da), gb = f2_sub(thr2, db);
                        uint32_t g = 0;
                        g = __funnelshift_l(static_cast<uint32_t>(ga), g, 1);
                        g = __funnelshift_l(static_cast<uint32_t>(ga >> 32), g, 1);
                        g = __funnelshift_l(static_cast<uint32_t>(gb), g, 1);
                        g = __funnelshift_l(static_cast<uint32_t>(gb >> 32), g, 1);
                        m |= (~g & 0xFu) << (12 - 4 * e4);  // bit 15 - e: column e admitted
                    }
                }
                if (self_e >= 0) m &= ~(1u << (15 - self_e));
                if (__any_sync(0xffffffffu, m != 0u)) {
                    const int npass = __popc(m);
                    if (__any_sync(0xffffffffu, nb + npass > kSBuf)) {
                        if (nxt_in_flight) {  // no TMEM load in flight across the call
                            if constexpr (kCorr) tmem_ld_wait_2x16(nxt, nxtc);
                            else tmem_ld_wait_regs(nxt);
                        }
                        const long long f0 = st_on ? clock64() : 0;
                        n_pass += nb;
                        ++n_flush;
                        flush_list<kL>(tl, my_buf, nb);
                        nb = 0;
                        refresh_thr();
                        m = 0u;  // this slice again, against the new threshold
#pragma unroll
                        for (int e = 0; e < 16; ++e) m |= (dist[e] <= thr) ? (1u << (15 - e)) : 0u;
                        if (self_e >= 0) m &= ~(1u << (15 - self_e));
                        if (st_on) cyc_flush += clock64() - f0;
                    }
                    int i = nb;
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        if (m & (1u << (15 - e))) {
                            const uint32_t code = dist_code(dist[e], code_b);
                            my_buf[i * 128] = (code << p.col_bits) | ((c0 + static_cast<uint32_t>(e)) & col_mask);
                            ++i;
                        }
                    }
                    nb = i;
                }
                __syncwarp();
            };
            // the accumulator goes back to the MMA as soon as its last slice is in registers
            auto release_acc = [&]() {
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(S_ACC_EMPTY(b));
            };
            __syncwarp();
            ld_slice(0, va, ca);
            if constexpr (kCorr) {
                // the single accumulator pair goes back to the MMA as soon as the whole tile (main
                // plus corrections) sits in shared memory; the scan then reads it from there
                float* stg = reinterpret_cast<float*>(smem_raw + p.stg_off) + r;
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const bool more = c + 1 < 8;
                    uint32_t (&cur)[16] = (c & 1) == 0 ? va : vb;
                    uint32_t (&curc)[16] = (c & 1) == 0 ? ca : cb;
                    uint32_t (&nxt)[16] = (c & 1) == 0 ? vb : va;
                    uint32_t (&nxtc)[16] = (c & 1) == 0 ? cb : ca;
                    wait_slice(cur, curc);
                    if (more) {
                        __syncwarp();
                        ld_slice(c + 1, nxt, nxtc);
                    }
#pragma unroll
                    for (int e = 0; e < 16; ++e) stg[(c * 16 + e) * 128] = __uint_as_float(cur[e]);
                }
                release_acc();
#pragma unroll 1
                for (int c = 0; c < 8; ++c) {
#pragma unroll
                    for (int e = 0; e < 16; ++e) va[e] = __float_as_uint(stg[(c * 16 + e) * 128]);
                    scan_slice(c, va, vb, cb, false);
                }
            } else {
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const bool more = c + 1 < 8;
                    if ((c & 1) == 0) {
                        wait_slice(va, ca);
                        if (more) {
                            __syncwarp();
                            ld_slice(c + 1, vb, cb);
                        } else {
                            release_acc();
                        }
                        scan_slice(c, va, vb, cb, more);
                    } else {
                        wait_slice(vb, cb);
                        if (more) {
                            __syncwarp();
                            ld_slice(c + 1, va, ca);
                        } else {
                            release_acc();
                        }
                        scan_slice(c, vb, va, ca, more);
                    }
                }
            }
        }
        if (ok && __any_sync(0xffffffffu, nb > 0)) {
            n_pass += nb;
            ++n_flush;
            flush_list<kL>(tl, my_buf, nb);
            nb = 0;
        }
        if (ok) {
            // the row's list (ascending keys, sentinels last) for the rerank, which decides from
            // exact distances which keys it needs and whether columns beyond the list may qualify
            int nv = 0;
#pragma unroll 1
            for (int blk = 0; blk < kL; blk += 32) {
                uint32_t c[32];
                tmem_ld_32x32b_x32(tl + static_cast<uint32_t>(blk), c);
                tmem_ld_wait_regs32(c);
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    if (row_ok && c[j] != kSEmpty) p.cand_cols[irow * kL + blk + j] = static_cast<int32_t>(c[j]);
                    nv += c[j] != kSEmpty ? 1 : 0;
                }
            }
            if (row_ok) p.cand_n[irow] = nv;
            if (st_on) {
                if (row_ok) {
                    atomicAdd(&p.stats[0], static_cast<unsigned long long>(n_pass));
                    atomicAdd(&p.stats[2], 1ull);
                }
                if (lane == 0) {
                    atomicAdd(&p.stats[1], static_cast<unsigned long long>(n_flush));
                    atomicAdd(&p.stats[3], static_cast<unsigned long long>(cyc_wait));
                    atomicAdd(&p.stats[4], static_cast<unsigned long long>(cyc_flush));
                    atomicAdd(&p.stats[5], static_cast<unsigned long long>(clock64() - cyc0));
                }
            }
        }
    }
#undef S_FULL
#undef S_EMPTY
#undef S_ACC_FULL
#undef S_ACC_EMPTY
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

__global__ void fill_inf_kernel(float* __restrict__ p, int64_t n)
{
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) p[i] = INFINITY;
}

// ---- operand rows: scaled fp16 parts ---------------------------------------------------
// One warp per pool row (f32, pitch dp): out row j holds its hi part (d16 fp16, zero past d) and,
// with two parts, its lo part after d16 elements.
__global__ void split_rows_kernel(const float* __restrict__ pool, int dp, int d, int64_t n,
                                  const float* __restrict__ maxnorm, __half* __restrict__ out, int d16, int parts)
{
    const int lane = threadIdx.x & 31;
    const int64_t j = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (j >= n) return;
    const float sc = screen_scale(*maxnorm);
    const float* x = pool + j * dp;
    __half* o = out + j * static_cast<int64_t>(parts) * d16;
    for (int i = lane; i < d16; i += 32) {
        const float v = i < d ? x[i] * sc : 0.0f;
        const __half h = __float2half_rn(v);
        o[i] = h;
        if (parts == 2) o[d16 + i] = __float2half_rn(v - __half2float(h));
    }
}

// ---- exact rerank ------------------------------------------------------------------------
// The exact distances run on a bucket-contiguous f32 copy of the pool rows (pitch dp, a
// multiple of 32, zero past d: the extra terms add +0 to the chain and change nothing; rows
// 128-byte aligned).  A warp evaluates 32 candidates at a time, one per lane: 32-dimension
// chunks of the 32 candidate rows are staged in shared memory by cp.async (each 128-byte row
// segment one transaction; two chunks in flight), and every lane reads its own row from there
// (16-byte loads, rows 36 floats apart: conflict-free) and continues its ascending fmaf chain
// against the query row (shared memory, broadcast reads).
constexpr int kRrWarps = 4;
constexpr int kRrKeys = 512;
constexpr int kRrRows = 8;          // A rows per rerank work item (few rows in flight per bucket)
constexpr int kChainStride = 36;    // floats between staged rows
constexpr int kChainStage = 32 * kChainStride;          // floats of one staged chunk
constexpr int kChainBufBytes = 2 * kChainStage * 4;     // per warp: two chunks

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// exact fp32 chain (ascending dimensions) of the query row q_s (shared memory, dp floats) against
// pool row `brow` of this lane (-1: none, the result is ignored); warp-collective, buf: this
// warp's kChainBufBytes of shared memory
__device__ __forceinline__ float warp_chain(const float* __restrict__ q_s, const float* __restrict__ pool, int dp,
                                            int64_t brow, float* __restrict__ buf, int lane)
{
    // per chunk this lane copies 16 bytes of rows 4 i + lane / 8 (i = 0..7), piece lane % 8
    const float* src[8];
    uint32_t nbytes[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int64_t br = __shfl_sync(0xffffffffu, brow, 4 * i + (lane >> 3));
        src[i] = pool + (br >= 0 ? br : 0) * static_cast<int64_t>(dp) + (lane & 7) * 4;
        nbytes[i] = br >= 0 ? 16u : 0u;  // no candidate: zeros
    }
    const uint32_t dst0 = smem_u32(buf) + static_cast<uint32_t>(((lane >> 3) * kChainStride + (lane & 7) * 4) * 4);
    auto issue = [&](int c) {
        const uint32_t d = dst0 + static_cast<uint32_t>((c & 1) * kChainStage * 4);
#pragma unroll
        for (int i = 0; i < 8; ++i)
            cp_async16(d + static_cast<uint32_t>(i * 4 * kChainStride * 4), src[i] + c * 32, nbytes[i]);
        cp_async_commit();
    };
    const int nc = dp >> 5;
    issue(0);
    if (nc > 1) issue(1);
    float acc = 0.0f;
    for (int c = 0; c < nc; ++c) {
        if (c + 1 < nc) cp_async_wait<1>();
        else cp_async_wait<0>();
        __syncwarp();
        const float4* mine = reinterpret_cast<const float4*>(buf + (c & 1) * kChainStage + lane * kChainStride);
        const float4* q4 = reinterpret_cast<const float4*>(q_s + c * 32);
#pragma unroll
        for (int b = 0; b < 8; ++b) {
            const float4 x = mine[b];
            const float4 q = q4[b];
            float t = q.x - x.x;
            acc = fmaf(t, t, acc);
            t = q.y - x.y;
            acc = fmaf(t, t, acc);
            t = q.z - x.z;
            acc = fmaf(t, t, acc);
            t = q.w - x.w;
            acc = fmaf(t, t, acc);
        }
        __syncwarp();
        if (c + 2 < nc) issue(c + 2);
    }
    return acc;
}

__device__ __forceinline__ void rr_sort(uint64_t* keys, int n, int lane)
{
    for (int k = 2; k <= n; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            const int lj = __ffs(j) - 1;
            for (int t = lane; t < (n >> 1); t += 32) {
                const int i = ((t >> lj) << (lj + 1)) + (t & (j - 1));
                const int l = i + j;
                const bool up = (i & k) == 0;
                const uint64_t x = keys[i], y = keys[l];
                if ((x > y) == up) {
                    keys[i] = y;
                    keys[l] = x;
                }
            }
            __syncwarp();
        }
    }
}

struct RerankX {
    const WorkItem* work;      // groups of up to kRrRows A rows (self_col0: the first row's column)
    const float* pool;         // f32 pool rows, pitch dp
    int dp;
    const int32_t* gid;        // pool row -> output id
    const int32_t* cand_cols;  // the screen's row lists (keys), by pool row
    const int32_t* cand_n;
    const float* norm;         // exact ||x||^2 of the pool rows
    const float* maxnorm;      // device scalar: max ||x|| (the screen's scale and margin)
    float mc1, mc2;            // the screen's margin coefficients (two-sided)
    int col_bits;
    int L;
    int m_out;
    int32_t* out_ids;           // [n_rows x m_out]: item rows below n_rows (the pool row itself)
    float* out_dists;
    int32_t* ext_ids;           // [item rows - n_rows x m_out]: the column chunks of long segments
    float* ext_dists;
    int64_t n_rows;
    unsigned long long* stats;  // optional: [exact candidates, rows rescanned, rows]
    const float* seed;          // as ScreenArgs::seed (work items with pad2 >= 0)
    float* seed_out;            // the same array: pilot items write their rows' bounds into it
    int2* rescan;               // [item rows] (item row, work item) of the rows whose columns are rescanned
    unsigned* n_rescan;         // device counter of those rows
};

// The row's top-m_out (keys ascending, n_sorted of them in keys[]).  compact (a chunk k > 0
// list, read only by merge_step_kernel): the valid entries and, when there are fewer than m_out,
// one id -1 after them; the rest of the row keeps stale entries.
__device__ __forceinline__ void write_list(const RerankX& p, int64_t irow, const uint64_t* keys, int n_sorted, int lane,
                                           bool compact = false)
{
    int32_t* oi = irow < p.n_rows ? p.out_ids + irow * p.m_out : p.ext_ids + (irow - p.n_rows) * p.m_out;
    float* od = irow < p.n_rows ? p.out_dists + irow * p.m_out : p.ext_dists + (irow - p.n_rows) * p.m_out;
    int n_w = p.m_out;
    if (compact) {
        int nv = 0;  // valid keys (sorted first)
        for (int j0 = 0; j0 < n_sorted && j0 < p.m_out; j0 += 32) {
            const int j = j0 + lane;
            nv += __popc(__ballot_sync(0xffffffffu, j < n_sorted && j < p.m_out && keys[j] != ~0ull));
        }
        n_w = nv < p.m_out ? nv + 1 : p.m_out;
    }
    for (int j = lane; j < n_w; j += 32) {
        const uint64_t key = j < n_sorted ? keys[j] : ~0ull;
        const bool v = key != ~0ull;
        oi[j] = v ? static_cast<int32_t>(static_cast<uint32_t>(key)) : -1;
        od[j] = v ? key2f(static_cast<uint32_t>(key >> 32)) : INFINITY;
    }
}

__global__ void __launch_bounds__(kRrWarps * 32) rerank_kernel(const RerankX p)
{
    extern __shared__ uint8_t sm[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t* keys = reinterpret_cast<uint64_t*>(sm) + warp * kRrKeys;
    float* cbuf = reinterpret_cast<float*>(sm + kRrWarps * kRrKeys * sizeof(uint64_t) + warp * kChainBufBytes);
    float* q_s = reinterpret_cast<float*>(sm + kRrWarps * (kRrKeys * sizeof(uint64_t) + kChainBufBytes)) + warp * p.dp;
    const WorkItem w = p.work[blockIdx.x];
    const float bm = *p.maxnorm;
    const float sc = screen_scale(bm);
    const float inv_s2 = 1.0f / (sc * sc);   // a power of two: exact
    const uint32_t code_b = code_base(sc, bm);
    const uint32_t col_mask = (1u << p.col_bits) - 1u;
    // lower bound of a key's approximate distance (unscaled): decode(code - 1) < approx
    auto approx_lo = [&](uint32_t key) {
        const uint32_t code = key >> p.col_bits;
        return code == 0u ? -INFINITY : code_value(code - 1u, code_b) * inv_s2;
    };
    // has_self bit 1: a chunk k > 0 list, written compactly (merge_step_kernel reads it); bit 2: a
    // pilot item, which only bounds its rows' M-th distance (seed_out[pad2 + r])
    const bool compact = (w.has_self & 2) != 0;
    const bool pilot = (w.has_self & 4) != 0;
    for (int r = warp; r < w.a_rows; r += kRrWarps) {
        const int64_t arow = static_cast<int64_t>(w.a_row0) + r;
        const int64_t irow = static_cast<int64_t>(w.item_row0) + r;
        const int nv = p.cand_n[irow];
        if (nv == 0) {  // nothing admitted: an empty list
            if (!pilot) {
                if (p.stats && lane == 0) atomicAdd(&p.stats[2], 1ull);
                write_list(p, irow, keys, 0, lane, compact);
            }
            __syncwarp();
            continue;
        }
        const uint32_t* kl = reinterpret_cast<const uint32_t*>(p.cand_cols) + irow * p.L;
        const int n1 = nv < p.m_out ? nv : p.m_out;
        if (pilot) {
            // The row's exact M-th distance over the whole bucket is at most the largest exact
            // distance of any m_out distinct columns of it.  A listed column's exact distance is at
            // most its approximate one plus the screen's one-sided error (the bound of step 2
            // below), and its code's value is at least the approximate distance, so the window's
            // first m_out keys give the bound without exact chains (rounded up throughout).
            if (n1 == p.m_out) {
                float mx = -INFINITY;
                for (int j = lane; j < n1; j += 32)
                    mx = fmaxf(mx, __fmul_ru(code_value(kl[j] >> p.col_bits, code_b), inv_s2));
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                const float an = sqrtf(fmaxf(p.norm[arow], 0.0f));
                const float err = 0.5f * (p.mc1 * an * bm + p.mc2 * (an + bm) * (an + bm));
                if (lane == 0) p.seed_out[static_cast<int64_t>(w.pad2) + r] = __fadd_ru(mx, err);
            }
            __syncwarp();
            continue;
        }
        for (int i = lane; i < p.dp; i += 32) q_s[i] = p.pool[arow * p.dp + i];
        __syncwarp();
        // exact keys of list positions [j_lo, j_hi) into keys[j]; returns the largest distance
        auto exact_range = [&](int j_lo, int j_hi) {
            float mx = -INFINITY;
            for (int j0 = j_lo; j0 < j_hi; j0 += 32) {
                const int j = j0 + lane;
                const int c = j < j_hi ? static_cast<int>(kl[j] & col_mask) : -1;
                const int64_t brow = c >= 0 ? static_cast<int64_t>(w.b_row0) + c : -1;
                const float dd = warp_chain(q_s, p.pool, p.dp, brow, cbuf, lane);
                if (c >= 0) {
                    keys[j] = (static_cast<uint64_t>(f2key(dd)) << 32) | static_cast<uint32_t>(p.gid[brow]);
                    mx = fmaxf(mx, dd);
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            return mx;
        };
        // 1. the first M keys: their largest exact distance bounds the row's exact M-th
        const float e_m = exact_range(0, n1);
        int n_tot = n1;
        bool rescan = false;
        if (nv > n1) {
            // 2. the keys whose approximate distance may lie within e_m (or the row's seed, when
            //    smaller: both bound its exact M-th) plus the one-sided error
            const float an = sqrtf(fmaxf(p.norm[arow], 0.0f));
            const float sd = w.pad2 >= 0 ? p.seed[static_cast<int64_t>(w.pad2) + r] : INFINITY;
            const float bound = fminf(e_m, sd) + 0.5f * (p.mc1 * an * bm + p.mc2 * (an + bm) * (an + bm));
            int n2 = nv - n1;
            for (int j0 = n1; j0 < nv; j0 += 32) {
                const int j = j0 + lane;
                const unsigned fail = __ballot_sync(0xffffffffu, j < nv && !(approx_lo(kl[j]) <= bound));
                if (fail) {
                    n2 = j0 + __ffs(fail) - 1 - n1;
                    break;
                }
            }
            exact_range(n1, n1 + n2);
            n_tot = n1 + n2;
            // 3. every key of a full list passed: columns beyond the list may lie within the bound
            rescan = nv == p.L && n_tot == p.L;
        }
        if (p.stats && lane == 0) {
            atomicAdd(&p.stats[0], static_cast<unsigned long long>(n_tot));
            atomicAdd(&p.stats[1], rescan ? 1ull : 0ull);
            atomicAdd(&p.stats[2], 1ull);
        }
        if (rescan) {
            // the whole segment, exactly, by rescan_kernel (a CTA per row, the columns split over its warps)
            if (lane == 0) {
                const unsigned slot = atomicAdd(p.n_rescan, 1u);
                p.rescan[slot] = make_int2(static_cast<int>(irow), static_cast<int>(blockIdx.x));
            }
            __syncwarp();
            continue;
        }
        int np2 = 1;
        while (np2 < n_tot) np2 <<= 1;
        for (int j = n_tot + lane; j < np2; j += 32) keys[j] = ~0ull;
        __syncwarp();
        rr_sort(keys, np2, lane);
        write_list(p, irow, keys, np2, lane, compact);
        __syncwarp();
    }
}

// Exact top-m_out of whole segments for the rows the rerank could not settle from its list:
// persistent CTAs walk the rescan list; per row, each of the kRsWarps warps keeps the 256 best
// (distance, id) keys of its share of the columns (a bitonic sort of 512 keys per 256 columns),
// then warp 0 merges the warps' lists.  A wave usually rescans fewer rows than there are CTAs,
// so its time is one row's scan (C3: 3.7 ms per wave for a 32 768-column chunk with 8 warps):
// 16 warps per CTA (one CTA per SM) halve it where their shared memory fits, 8 (two per SM)
// serve longer rows.  With fewer rows than CTAs a row's columns are also cut into `slices`
// ranges (multiples of 256 columns), one per CTA, each writing its best m_out keys to `partial`
// for rescan_merge_kernel.  The list depends on neither split.
template <int kRsWarps>
__global__ void __launch_bounds__(kRsWarps * 32) rescan_kernel(const RerankX p, int slices, uint64_t* partial)
{
    extern __shared__ uint8_t sm[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t* all = reinterpret_cast<uint64_t*>(sm);
    uint64_t* keys = all + warp * kRrKeys;
    float* cbuf = reinterpret_cast<float*>(sm + kRsWarps * kRrKeys * sizeof(uint64_t) + warp * kChainBufBytes);
    float* q_s = reinterpret_cast<float*>(sm + kRsWarps * (kRrKeys * sizeof(uint64_t) + kChainBufBytes));
    const uint64_t n = *p.n_rescan;
    const uint64_t units = n * static_cast<uint64_t>(slices);
    for (uint64_t u = blockIdx.x; u < units; u += gridDim.x) {
        const uint64_t i = u / static_cast<uint64_t>(slices);
        const int sl = static_cast<int>(u - i * static_cast<uint64_t>(slices));
        const int2 e = p.rescan[i];
        const int64_t irow = e.x;
        const WorkItem w = p.work[e.y];
        const int r = static_cast<int>(irow - w.item_row0);
        const int64_t arow = static_cast<int64_t>(w.a_row0) + r;
        const int self = (w.has_self & 1) ? w.self_col0 + r : -1;  // outside [0, b_rows): no column is skipped
        // this unit's columns [c_lo, c_hi) of the row's b_rows
        const int span = ((w.b_rows + slices - 1) / slices + 255) / 256 * 256;
        const int c_lo = sl * span;
        const int c_hi = c_lo + span < w.b_rows ? c_lo + span : w.b_rows;
        __syncthreads();
        for (int j = threadIdx.x; j < p.dp; j += blockDim.x) q_s[j] = p.pool[arow * p.dp + j];
        for (int j = lane; j < kRrKeys; j += 32) keys[j] = ~0ull;
        __syncthreads();
        // this warp's columns: chunks of 256 starting at c_lo + 256 * warp, strided by the CTA
        for (int c0 = c_lo + 256 * warp; c0 < c_hi; c0 += 256 * kRsWarps) {
            for (int j = 0; j < kRrKeys / 2; j += 32) {
                const int c = c0 + j + lane;
                const bool ok = c < c_hi && c != self;
                const int64_t brow = ok ? static_cast<int64_t>(w.b_row0) + c : -1;
                const float dd = warp_chain(q_s, p.pool, p.dp, brow, cbuf, lane);
                keys[kRrKeys / 2 + j + lane] =
                    ok ? (static_cast<uint64_t>(f2key(dd)) << 32) | static_cast<uint32_t>(p.gid[brow]) : ~0ull;
            }
            __syncwarp();
            rr_sort(keys, kRrKeys, lane);
        }
        __syncthreads();
        if (warp == 0) {
            // the warps' best m_out each (their lists are sorted) -> the row's best m_out
            for (int q = 1; q < kRsWarps; ++q) {
                const uint64_t* other = all + q * kRrKeys;
                for (int j = lane; j < kRrKeys / 2; j += 32) keys[kRrKeys / 2 + j] = j < p.m_out ? other[j] : ~0ull;
                __syncwarp();
                rr_sort(keys, kRrKeys, lane);
            }
            if (slices == 1) {
                write_list(p, irow, keys, kRrKeys / 2, lane);
            } else {
                uint64_t* dst = partial + (i * static_cast<uint64_t>(slices) + static_cast<uint64_t>(sl)) * p.m_out;
                for (int j = lane; j < p.m_out; j += 32) dst[j] = keys[j];
            }
        }
    }
}

// The rows rescanned in slices: one warp per row merges its slices' best m_out keys (each
// slice's list sorted; the row's list kept in the first half of the buffer as in the CTA merge
// above) and writes the row's list.
__global__ void __launch_bounds__(kRrWarps * 32)
    rescan_merge_kernel(const RerankX p, int slices, const uint64_t* __restrict__ partial)
{
    __shared__ uint64_t s_keys[kRrWarps][kRrKeys];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint64_t n = *p.n_rescan;
    const uint64_t i = static_cast<uint64_t>(blockIdx.x) * kRrWarps + warp;
    if (i >= n) return;
    uint64_t* keys = s_keys[warp];
    const uint64_t* src = partial + i * static_cast<uint64_t>(slices) * p.m_out;
    for (int j = lane; j < kRrKeys; j += 32) keys[j] = j < p.m_out ? src[j] : ~0ull;
    for (int sl = 1; sl < slices; ++sl) {
        __syncwarp();
        for (int j = lane; j < kRrKeys / 2; j += 32)
            keys[kRrKeys / 2 + j] = j < p.m_out ? src[static_cast<int64_t>(sl) * p.m_out + j] : ~0ull;
        __syncwarp();
        rr_sort(keys, kRrKeys, lane);
    }
    __syncwarp();
    write_list(p, p.rescan[i].x, keys, kRrKeys / 2, lane);
}

// Rows of segments that run as column chunks, one chunk per wave: the row's running list (the
// exact top-m_out of the chunks so far, in its chunk-0 extension row) and its seed (the running
// list's m_out-th distance, a bound on the row's exact M-th that the next chunk's screen and
// rerank use).  lo, nb: the first pool row with a list and the count of such rows (a row range of
// the segment, whose columns are all its rows).  Two extension slots per row: chunk 0's list (then
// the running list) at base_ext + i, the current chunk k > 0 at base_ext + nb + i (reused by every
// wave: a wave's lists are merged before the next wave's rerank writes).
struct ChunkSeg {
    int64_t lo, nb, base_ext, row_prefix;  // base_ext: extension row of (chunk 0, row 0)
    int32_t nch, pad;
};

// k = 0: seeds tightened by the chunk-0 lists; k > 0: chunk k merged into the running list (by
// (distance, id)), then the seed (nothing to do for an empty chunk list); k < 0: the running
// lists written to the rows' outputs.
// One warp per row of the chunked segments.
__global__ void __launch_bounds__(kRrWarps * 32)
    merge_step_kernel(const ChunkSeg* __restrict__ segs, int n_segs, int64_t n_rows_total, int k,
                      int32_t* __restrict__ ext_ids, float* __restrict__ ext_dists, int m_out, float* __restrict__ seeds,
                      int32_t* __restrict__ out_ids, float* __restrict__ out_dists)
{
    __shared__ uint64_t s_keys[kRrWarps][kRrKeys];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t j = static_cast<int64_t>(blockIdx.x) * kRrWarps + warp;
    if (j >= n_rows_total) return;
    int lo = 0, hi = n_segs - 1;  // the segment holding row j: last with row_prefix <= j
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (segs[mid].row_prefix <= j) lo = mid;
        else hi = mid - 1;
    }
    const ChunkSeg sg = segs[lo];
    const int64_t i = j - sg.row_prefix;
    const int64_t run = sg.base_ext + i;
    if (k < 0) {
        const int64_t prow = sg.lo + i;
        for (int t = lane; t < m_out; t += 32) {
            out_ids[prow * m_out + t] = ext_ids[run * m_out + t];
            out_dists[prow * m_out + t] = ext_dists[run * m_out + t];
        }
        return;
    }
    if (k >= sg.nch) return;
    if (k > 0) {
        const int64_t er = sg.base_ext + sg.nb + i;
        // a chunk list with no entry (every column beyond the seed) leaves the running list and
        // its seed as they are
        if (ext_ids[er * m_out] < 0) return;
        uint64_t* keys = s_keys[warp];
        // the chunk list is compact: its entries end at the first id -1 (or at m_out)
        int n_new = m_out;
        for (int t0 = 0; t0 < m_out; t0 += 32) {
            const unsigned neg = __ballot_sync(0xffffffffu, t0 + lane < m_out && ext_ids[er * m_out + t0 + lane] < 0);
            if (neg) {
                n_new = t0 + __ffs(neg) - 1;
                break;
            }
        }
        auto key_of = [&](int64_t row, int t) {
            const int32_t id = (row == er && t >= n_new) ? -1 : ext_ids[row * m_out + t];
            return id < 0 ? ~0ull
                          : (static_cast<uint64_t>(f2key(ext_dists[row * m_out + t])) << 32) | static_cast<uint32_t>(id);
        };
        // both lists ascending by (distance, id), disjoint (chunks split the columns): the running
        // list then the chunk's reversed form one bitonic sequence of 2P keys; half-cleaners sort it
        int P = 32;
        while (P < m_out) P <<= 1;
        for (int t = lane; t < P; t += 32) {
            keys[t] = t < m_out ? key_of(run, t) : ~0ull;
            keys[2 * P - 1 - t] = t < m_out ? key_of(er, t) : ~0ull;
        }
        __syncwarp();
        for (int j = P; j > 0; j >>= 1) {
            const int lj = __ffs(j) - 1;
            for (int t = lane; t < P; t += 32) {
                const int a = ((t >> lj) << (lj + 1)) + (t & (j - 1));
                const uint64_t x = keys[a], y = keys[a + j];
                if (x > y) {
                    keys[a] = y;
                    keys[a + j] = x;
                }
            }
            __syncwarp();
        }
        for (int t = lane; t < m_out; t += 32) {
            const uint64_t key = keys[t];
            const bool v = key != ~0ull;
            ext_ids[run * m_out + t] = v ? static_cast<int32_t>(static_cast<uint32_t>(key)) : -1;
            ext_dists[run * m_out + t] = v ? key2f(static_cast<uint32_t>(key >> 32)) : INFINITY;
        }
        __syncwarp();
    }
    if (lane == 0) {  // the running list's m_out-th distance tightens the row's seed (the pilot's bound)
        const bool full = ext_ids[run * m_out + m_out - 1] >= 0;
        if (full) seeds[j] = fminf(seeds[j], ext_dists[run * m_out + m_out - 1]);
    }
}

struct ScreenPlan {
    int stages = 0;
    uint32_t buf_off = 0, pn_off = 0, stg_off = 0, bar_off = 0, total = 0;
};

bool screen_plan(bool split, bool corr, ScreenPlan& pl)
{
    // operand chunk: 64 fp16 per row (corr: 32) of each part of A and B
    const uint32_t stage_bytes = 2u * (split ? 2u : 1u) * (corr ? kSChunk / 2u : kSChunk);
    for (int S = 6; S >= 2; --S) {
        ScreenPlan t;
        t.stages = S;
        uint32_t off = static_cast<uint32_t>(S) * stage_bytes;
        t.buf_off = off;
        off += static_cast<uint32_t>(kSBuf) * 128u * 4u;
        t.pn_off = off;
        off += 4u * kSTile * 4u;
        t.stg_off = off;
        if (corr) off += 128u * 128u * 4u;
        t.bar_off = off;
        off += 8u * (2u * S + 5u) + 16u;
        t.total = off;
        if (t.total <= kSSmemMax) {
            pl = t;
            return true;
        }
    }
    return false;
}

using EncodeFnS = PFN_cuTensorMapEncodeTiled_v12000;

EncodeFnS screen_encode()
{
    static EncodeFnS fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeFnS>(ptr);
    });
    GTA_REQUIRE(fn != nullptr, kCuda, "cuTensorMapEncodeTiled is not available from the driver");
    return fn;
}

template <int kL, bool kSplit, bool kCorr = false>
void launch_screen(const CUtensorMap& tm, const ScreenArgs& a, int n_work, uint32_t smem, cudaStream_t st)
{
    auto fn = screen_kernel<kL, kSplit, kCorr>;
    GTA_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    fn<<<n_work, kSThreads, smem, st>>>(tm, a);
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

}  // namespace

int screen_list_len(int m) { return m <= 64 ? 128 : 256; }

void screen_knn(const ScreenProblem& pr, cudaStream_t st)
{
    if (pr.seg_lo.empty()) return;
    GTA_REQUIRE(pr.X && pr.ids && pr.gid && pr.out_ids && pr.out_dists && pr.seg_lo.size() == pr.seg_n.size(), kInvalid,
                "screen: null operand");
    GTA_REQUIRE(pr.dtype == GTA_F32 || pr.dtype == GTA_U8 || pr.dtype == GTA_I8, kInvalid, "screen: bad dtype");
    GTA_REQUIRE(pr.d >= 1 && pr.m_out >= 1 && pr.m_out <= 128, kInvalid, "screen: unsupported shape");
    GTA_REQUIRE(pr.parts == 1 || pr.parts == 2, kInvalid, "screen: one or two operand parts");
    // Work: one item per 128 rows of a segment.  A segment longer than kChunk runs as column
    // chunks of kChunk in waves: wave 0 holds every short segment and the chunk 0 of the long
    // ones; wave k > 0 holds chunk k, its rows seeded with the m-th distance of their running list
    // (the exact top-m of chunks 0 .. k-1).  A chunked row has two list rows past the pool rows
    // (extension rows): its running list and the current chunk's.
    // kChunk: the CTAs of a wave re-read their own A tiles and the chunk's B tiles from L2 once per
    // column tile, so a chunk is sized for both to stay in L2 (the A tiles of one CTA per SM plus
    // the chunk's columns within 90% of it; a power of two, 4096 .. 65536 columns).
    // (the operand bytes a row tile reads: one fp16 part when the screen starts with one part)
    const int64_t row_bytes = static_cast<int64_t>(pr.parts == 1 || pr.d >= 256 ? 1 : pr.parts) * ((pr.d + 63) / 64 * 64) * 2;
    int64_t kChunk = 1 << 16;
    {
        int dev = 0, l2 = 0, n_sm = 0;
        GTA_CUDA(cudaGetDevice(&dev));
        GTA_CUDA(cudaDeviceGetAttribute(&l2, cudaDevAttrL2CacheSize, dev));
        GTA_CUDA(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev));
        const int64_t room = static_cast<int64_t>(0.9 * l2) - static_cast<int64_t>(n_sm) * kSTile * row_bytes;
        while (kChunk > 4096 && kChunk * row_bytes > room) kChunk >>= 1;
    }
    std::vector<std::vector<WorkItem>> waves(1);
    std::vector<ChunkSeg> chunked;
    std::vector<WorkItem> pilot;  // seeds of the chunked rows (one item per row tile)
    constexpr int64_t kPilot = 4096;
    int64_t ext_rows = 0, chunked_rows = 0;
    GTA_REQUIRE((pr.seg_r0.empty() && pr.seg_r1.empty()) ||
                    (pr.seg_r0.size() == pr.seg_lo.size() && pr.seg_r1.size() == pr.seg_lo.size()),
                kInvalid, "screen: row ranges need one entry per segment");
    for (size_t sgi = 0; sgi < pr.seg_lo.size(); ++sgi) {
        const int64_t lo = pr.seg_lo[sgi], nb = pr.seg_n[sgi];
        GTA_REQUIRE(lo >= 0 && nb >= 1 && lo + nb <= pr.n_rows, kInvalid, "screen: bad segment");
        // the segment's rows that get lists: [r0, r1) of its nb (every row is a column)
        const int64_t r0 = pr.seg_r0.empty() ? 0 : pr.seg_r0[sgi];
        const int64_t r1 = pr.seg_r1.empty() ? nb : pr.seg_r1[sgi];
        GTA_REQUIRE(0 <= r0 && r0 <= r1 && r1 <= nb, kInvalid, "screen: bad row range");
        if (r0 == r1) continue;
        const int64_t nr = r1 - r0;
        const int nch = static_cast<int>((nb + kChunk - 1) / kChunk);
        if (nch == 1) {
            for (int64_t t = r0; t < r1; t += 128)
                waves[0].push_back(WorkItem{static_cast<int32_t>(lo + t), static_cast<int32_t>(std::min<int64_t>(128, r1 - t)),
                                            static_cast<int32_t>(lo), static_cast<int32_t>(nb), static_cast<int32_t>(t),
                                            static_cast<int32_t>(lo + t), 1, -1});
            continue;
        }
        const int64_t base = pr.n_rows + ext_rows;
        chunked.push_back(ChunkSeg{lo + r0, nr, ext_rows, chunked_rows, nch, 0});
        if (static_cast<int>(waves.size()) < nch) waves.resize(static_cast<size_t>(nch));
        // the pilot: each row tile against a window of kPilot columns around its own tile (rows
        // of a bucket are grouped by their other bucket, so the window holds points of the same
        // region); the exact M-th distance over its first M candidates seeds every chunk
        const int64_t W = std::min<int64_t>(kPilot, nb);
        for (int64_t t = r0; t < r1; t += 128) {
            const int64_t ws = std::max<int64_t>(0, std::min<int64_t>(t + 64 - W / 2, nb - W));
            pilot.push_back(WorkItem{static_cast<int32_t>(lo + t), static_cast<int32_t>(std::min<int64_t>(128, r1 - t)),
                                     static_cast<int32_t>(lo + ws), static_cast<int32_t>(W),
                                     static_cast<int32_t>(t - ws), static_cast<int32_t>(base + nr + (t - r0)), 1,
                                     static_cast<int32_t>(chunked_rows + (t - r0))});
        }
        for (int k = 0; k < nch; ++k) {
            const int64_t c0 = k * kChunk, cn = std::min<int64_t>(kChunk, nb - c0);
            for (int64_t t = r0; t < r1; t += 128)
                waves[static_cast<size_t>(k)].push_back(
                    WorkItem{static_cast<int32_t>(lo + t), static_cast<int32_t>(std::min<int64_t>(128, r1 - t)),
                             static_cast<int32_t>(lo + c0), static_cast<int32_t>(cn), static_cast<int32_t>(t - c0),
                             static_cast<int32_t>(base + (k == 0 ? 0 : nr) + (t - r0)), k == 0 ? 1 : 3,
                             static_cast<int32_t>(chunked_rows + (t - r0))});
        }
        ext_rows += 2 * nr;
        chunked_rows += nr;
    }
    // per wave: the chunk whose lists its merge step takes (-1: none), and whether it runs the
    // split screen whatever the current mode
    std::vector<int> wave_chunk(waves.size());
    for (size_t k = 0; k < waves.size(); ++k) wave_chunk[k] = static_cast<int>(k);
    std::vector<char> wave_split(waves.size(), 0);
    // The rows of segments shorter than a chunk have no seed: under the one-part margin their full
    // lists admit many columns and often a rescan (C3: 81 ms of rerank and 96 ms of rescans for
    // 6 597 row tiles), against about 10 exact keys per row and no rescan under the split margin.
    // So they run as a wave of their own on the split screen (as the pilot does), before chunk 0
    // of the long segments; GTA_SCREEN_UNSEEDED_SPLIT=0 keeps them in wave 0 on the current mode.
    static const bool unseeded_split = [] {
        const char* e = std::getenv("GTA_SCREEN_UNSEEDED_SPLIT");
        return e == nullptr || e[0] != '0';
    }();
    if (unseeded_split && pr.parts == 2 && pr.d >= 256) {
        std::vector<WorkItem> unseeded, seeded;
        for (const WorkItem& it : waves[0]) (it.pad2 < 0 ? unseeded : seeded).push_back(it);
        if (!unseeded.empty()) {
            waves[0] = std::move(seeded);
            waves.insert(waves.begin(), std::move(unseeded));
            wave_chunk.insert(wave_chunk.begin(), -1);
            wave_split.insert(wave_split.begin(), 1);
        }
    }
    const int64_t item_rows = pr.n_rows + ext_rows;
    GTA_REQUIRE(item_rows < (1ll << 31), kInvalid, "screen: too many list rows");
    const int L = screen_list_len(pr.m_out);
    const int d16 = (pr.d + 63) / 64 * 64;
    // the pool's rows as f32 (bucket-contiguous, pitch dp, zero past d) with their exact squared
    // norms, the scale's source (max ||x||) and the scaled fp16 operand rows
    const int dp = (pr.d + 31) / 32 * 32;
    DevBuf<float> fpool(static_cast<size_t>(pr.n_rows) * dp, st), norm(static_cast<size_t>(pr.n_rows), st);
    DevBuf<float> bmax(1, st);
    DevBuf<__half> rows(static_cast<size_t>(pr.n_rows) * pr.parts * d16, st);
    {
        const double in_bytes = static_cast<double>(pr.n_rows) * pr.d * (pr.dtype == GTA_F32 ? 4.0 : 1.0);
        ProfScope prof("screen_rows", in_bytes + static_cast<double>(pr.n_rows) * (8.0 * dp + 2.0 * pr.parts * d16), st);
        convert_rows(pr.X, pr.dtype, pr.d, pr.ids, pr.n_rows, fpool.get(), kElemF32, dp, norm.get(), st);
        max_sqrt(norm.get(), pr.n_rows, bmax.get(), st);
        const int wpb = 8;
        split_rows_kernel<<<static_cast<unsigned>((pr.n_rows + wpb - 1) / wpb), wpb * 32, 0, st>>>(
            fpool.get(), dp, pr.d, pr.n_rows, bmax.get(), rows.get(), d16, pr.parts);
        count_launches(1);
        GTA_CUDA(cudaGetLastError());
    }
    // Screen modes (each with its kernel, shared-memory plan, tensor map and error bound):
    //  * split: hi.hi + hi.lo + lo.hi (the lo products in their own accumulator for d >= 256);
    //  * one part: hi.hi only, on the hi half of the same rows -- a margin about 2^12 times wider
    //    (2^-10 of |a| bmax per element) but a third of the tensor work and half the operand
    //    bytes.  Long rows (d >= 256) start with it: their neighbour distances are large against
    //    the margin (C3, 1M x 960: 1.78 s per build against 3.16 s split).  A wave that sends more
    //    than 5% of its rows to a rescan (too many columns within the wider margin) hands the
    //    remaining waves to the split screen; the seeds carry over (they are exact bounds).
    // error bound of the screened distance (the margin, applied to the M-th key), relative to
    // |a||b| <= |a| bmax:
    //  * operand parts: split 3 * 2^-22 (the dropped lo.lo and the rounding of lo), one part 2^-10;
    //  * fp32 accumulation, 2^-22 per product added to an accumulator: split into one accumulator
    //    3 d products; with the correction accumulator (corr) d products plus the final addition
    //    (the corrections themselves are below 2^-10 of the sum); one part d;
    // and, relative to (|a| + bmax)^2, the fp32 squared norms (each lane of the norm kernel chains
    // 4 ceil(dp / 128) products, then five butterfly additions) and the two fused operations of
    // the score; a 1.25 safety factor on both
    struct Mode {
        bool split = false, corr = false;
        ScreenPlan pl;
        CUtensorMap tm;
        int k_chunks = 0;
        float mc1 = 0.f, mc2 = 0.f;
    };
    auto make_mode = [&](bool split) {
        Mode m;
        m.split = split;
        m.corr = split && pr.d >= 256;
        GTA_REQUIRE(screen_plan(m.split, m.corr, m.pl), kInvalid, "screen: shared memory plan failed");
        cuuint64_t dims[2] = {static_cast<cuuint64_t>(pr.parts) * d16, static_cast<cuuint64_t>(pr.n_rows)};
        cuuint64_t strides[1] = {static_cast<cuuint64_t>(pr.parts) * d16 * 2u};
        cuuint32_t box[2] = {m.corr ? 32u : 64u, 128u};
        cuuint32_t estr[2] = {1u, 1u};
        const CUresult r = screen_encode()(&m.tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, rows.get(), dims, strides, box,
                                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                           m.corr ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        GTA_REQUIRE(r == CUDA_SUCCESS, kCuda, "cuTensorMapEncodeTiled failed (" + std::to_string(static_cast<int>(r)) + ")");
        m.k_chunks = d16 / (m.corr ? 32 : 64);
        const double dd = pr.d;
        const double part_err = split ? 3.0 * std::ldexp(1.0, -22) : std::ldexp(1.0, -10);
        const double n_prod = split ? (m.corr ? dd + 3.0 : 3.0 * dd) : dd;
        const double k_norm = 4.0 * ((dp + 127) / 128) + 8.0;
        m.mc1 = static_cast<float>(1.25 * 4.0 * (part_err + n_prod * std::ldexp(1.0, -22)));
        m.mc2 = static_cast<float>(1.25 * 3.0 * (k_norm + 4.0) * std::ldexp(1.0, -24));
        return m;
    };
    Mode modes[2];
    int n_modes = 0, cur = 0;
    if (pr.parts == 1 || pr.d >= 256) modes[n_modes++] = make_mode(false);
    const int split_mode = pr.parts == 2 ? n_modes : -1;
    if (pr.parts == 2) modes[n_modes++] = make_mode(true);
    DevBuf<int32_t> cand_cols(static_cast<size_t>(item_rows) * L, st), cand_n(static_cast<size_t>(item_rows), st);
    DevBuf<int32_t> ext_ids(static_cast<size_t>(ext_rows) * pr.m_out, st);
    DevBuf<float> ext_dists(static_cast<size_t>(ext_rows) * pr.m_out, st);
    DevBuf<float> seeds(static_cast<size_t>(chunked_rows), st);
    DevBuf<int2> rescan(static_cast<size_t>(item_rows), st);
    DevBuf<unsigned> n_rescan(1, st);
    DevBuf<ChunkSeg> segs(chunked.size(), st);
    if (!chunked.empty())
        GTA_CUDA(cudaMemcpyAsync(segs.get(), chunked.data(), sizeof(ChunkSeg) * chunked.size(), cudaMemcpyHostToDevice, st));
    ScreenArgs a{};
    a.norm = norm.get();
    a.maxnorm = bmax.get();
    a.part_stride = d16;
    a.m_sel = pr.m_out;
    a.col_bits = 16;  // columns of an item: at most kChunk
    a.seed = seeds.get();
    a.cand_cols = cand_cols.get();
    a.cand_n = cand_n.get();
    a.err = pr.err;
    RerankX r{};
    r.pool = fpool.get();
    r.dp = dp;
    r.gid = pr.gid;
    r.cand_cols = cand_cols.get();
    r.cand_n = cand_n.get();
    r.norm = norm.get();
    r.maxnorm = bmax.get();
    r.col_bits = a.col_bits;
    r.L = L;
    r.m_out = pr.m_out;
    r.out_ids = pr.out_ids;
    r.out_dists = pr.out_dists;
    r.ext_ids = ext_ids.get();
    r.ext_dists = ext_dists.get();
    r.n_rows = pr.n_rows;
    r.seed = seeds.get();
    r.rescan = rescan.get();
    r.n_rescan = n_rescan.get();
    const size_t smem_rr = kRrWarps * (kRrKeys * sizeof(uint64_t) + kChainBufBytes + static_cast<size_t>(dp) * 4);
    const size_t smem_rs16 = 16 * (kRrKeys * sizeof(uint64_t) + kChainBufBytes) + static_cast<size_t>(dp) * 4;
    const bool rs16 = smem_rs16 <= kSSmemMax;
    const size_t smem_rs = rs16 ? smem_rs16 : 8 * (kRrKeys * sizeof(uint64_t) + kChainBufBytes) + static_cast<size_t>(dp) * 4;
    GTA_REQUIRE(smem_rr <= kSSmemMax && smem_rs <= kSSmemMax, kInvalid, "rerank: dimension too large");
    GTA_CUDA(cudaFuncSetAttribute(rerank_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem_rr)));
    GTA_CUDA(cudaFuncSetAttribute(rs16 ? rescan_kernel<16> : rescan_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(smem_rs)));
    int dev = 0, n_sm = 0;
    GTA_CUDA(cudaGetDevice(&dev));
    GTA_CUDA(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev));
    const unsigned merge_grid = static_cast<unsigned>((chunked_rows + kRrWarps - 1) / kRrWarps);
    r.seed_out = seeds.get();
    if (chunked_rows > 0) {
        fill_inf_kernel<<<static_cast<unsigned>((chunked_rows + 255) / 256), 256, 0, st>>>(seeds.get(), chunked_rows);
        count_launches(1);
        GTA_CUDA(cudaGetLastError());
    }
    // wave -1: the pilot (unseeded screen of the windows, then the bound of each row)
    for (size_t k = 0; k < waves.size() + (pilot.empty() ? 0 : 1); ++k) {
        const bool is_pilot = !pilot.empty() && k == 0;
        const size_t wk = pilot.empty() ? k : k - 1;
        const std::vector<WorkItem>& items = is_pilot ? pilot : waves[wk];
        if (items.empty()) continue;
        const bool force_split = is_pilot ? true : wave_split[wk] != 0;
        double flops = 0.0;  // algorithmic: 2 d per (row, column) pair
        for (const WorkItem& it : items) flops += 2.0 * it.a_rows * static_cast<double>(it.b_rows) * pr.d;
        // the screen's items (the pilot's unseeded: its rerank groups carry the seed slots)
        std::vector<WorkItem> launch(items);
        if (is_pilot)
            for (WorkItem& it : launch) it.pad2 = -1;
        DevBuf<WorkItem> work(launch.size(), st);
        // pageable sources: each copy is staged before cudaMemcpyAsync returns
        GTA_CUDA(cudaMemcpyAsync(work.get(), launch.data(), sizeof(WorkItem) * launch.size(), cudaMemcpyHostToDevice, st));
        a.work = work.get();
        // unseeded rows (the pilot's, the short segments') admit many more keys under the one-part
        // margin (slow list merges, more exact keys, rescans): they run the split screen
        const Mode& md = modes[force_split && split_mode >= 0 ? split_mode : cur];
        a.k_chunks = md.k_chunks;
        a.stages = md.pl.stages;
        a.buf_off = md.pl.buf_off;
        a.pn_off = md.pl.pn_off;
        a.bar_off = md.pl.bar_off;
        a.stg_off = md.pl.stg_off;
        a.mc1 = r.mc1 = md.mc1;
        a.mc2 = r.mc2 = md.mc2;
        {
            // split waves are named apart (three issued products per element against one)
            const std::string pname = std::string(is_pilot ? "screen_pilot" : pr.prof_name) + (md.split ? "_split" : "");
            ProfScope prof(pname.c_str(), flops, st);
            a.stats = prof.counters(8);
            const int n_work = static_cast<int>(launch.size());
            const uint32_t smem = md.pl.total;
            if (L == 128) {
                if (md.corr) launch_screen<128, true, true>(md.tm, a, n_work, smem, st);
                else if (md.split) launch_screen<128, true>(md.tm, a, n_work, smem, st);
                else launch_screen<128, false>(md.tm, a, n_work, smem, st);
            } else {
                if (md.corr) launch_screen<256, true, true>(md.tm, a, n_work, smem, st);
                else if (md.split) launch_screen<256, true>(md.tm, a, n_work, smem, st);
                else launch_screen<256, false>(md.tm, a, n_work, smem, st);
            }
        }
        // the rerank's work: groups of kRrRows rows of the same items, in the same (bucket) order
        std::vector<WorkItem> groups;
        groups.reserve(items.size() * (128 / kRrRows));
        for (const WorkItem& it : items)
            for (int g = 0; g < it.a_rows; g += kRrRows)
                groups.push_back(WorkItem{it.a_row0 + g, std::min(kRrRows, it.a_rows - g), it.b_row0, it.b_rows,
                                          it.self_col0 + g, it.item_row0 + g, it.has_self | (is_pilot ? 4 : 0),
                                          it.pad2 >= 0 ? it.pad2 + g : -1});
        DevBuf<WorkItem> gwork(groups.size(), st);
        GTA_CUDA(cudaMemcpyAsync(gwork.get(), groups.data(), sizeof(WorkItem) * groups.size(), cudaMemcpyHostToDevice, st));
        r.work = gwork.get();
        GTA_CUDA(cudaMemsetAsync(n_rescan.get(), 0, sizeof(unsigned), st));
        {
            ProfScope prof(is_pilot ? "rerank_pilot" : "rerank", 0.0, st);
            r.stats = prof.counters(8);
            rerank_kernel<<<static_cast<unsigned>(groups.size()), kRrWarps * 32, smem_rr, st>>>(r);
            count_launches(1);
            GTA_CUDA(cudaGetLastError());
        }
        if (is_pilot) continue;  // the pilot writes no lists: nothing to rescan or merge
        // the rows the rerank left to a whole-segment rescan (the launch shape depends on their count)
        unsigned n_rs = 0;
        GTA_CUDA(cudaMemcpyAsync(&n_rs, n_rescan.get(), sizeof(unsigned), cudaMemcpyDeviceToHost, st));
        GTA_CUDA(cudaStreamSynchronize(st));
        if (n_rs > 0) {
            // persistent CTAs over the device-side list; fewer rows than CTAs: each row's columns
            // in slices over several CTAs, then a merge of the slices' lists
            ProfScope prof("rescan", 0.0, st);
            const int ctas = std::max(1, n_sm) * (rs16 ? 1 : 2);
            const int slices = n_rs >= static_cast<unsigned>(ctas) ? 1 : std::min(16, ctas / static_cast<int>(n_rs));
            DevBuf<uint64_t> partial(slices > 1 ? static_cast<size_t>(n_rs) * slices * pr.m_out : 0, st);
            if (rs16)
                rescan_kernel<16><<<static_cast<unsigned>(ctas), 16 * 32, smem_rs, st>>>(r, slices, partial.get());
            else
                rescan_kernel<8><<<static_cast<unsigned>(ctas), 8 * 32, smem_rs, st>>>(r, slices, partial.get());
            count_launches(1);
            GTA_CUDA(cudaGetLastError());
            if (slices > 1) {
                rescan_merge_kernel<<<(n_rs + kRrWarps - 1) / kRrWarps, kRrWarps * 32, 0, st>>>(r, slices, partial.get());
                count_launches(1);
                GTA_CUDA(cudaGetLastError());
            }
        }
        if (split_mode >= 0 && cur != split_mode && !wave_split[wk] && wk + 1 < waves.size()) {
            // too many rescans under the one-part margin: the remaining waves screen split
            int64_t wave_rows = 0;
            for (const WorkItem& it : items) wave_rows += it.a_rows;
            if (static_cast<double>(n_rs) > 0.05 * static_cast<double>(wave_rows)) cur = split_mode;
        }
        if (!chunked.empty() && wave_chunk[wk] >= 0) {
            // chunk k into the running lists (k = 0: the seeds of chunk 0's lists)
            ProfScope prof("merge_chunks", 24.0 * pr.m_out * static_cast<double>(chunked_rows), st);
            merge_step_kernel<<<merge_grid, kRrWarps * 32, 0, st>>>(segs.get(), static_cast<int>(chunked.size()),
                                                                    chunked_rows, wave_chunk[wk], ext_ids.get(),
                                                                    ext_dists.get(), pr.m_out, seeds.get(), pr.out_ids,
                                                                    pr.out_dists);
            count_launches(1);
            GTA_CUDA(cudaGetLastError());
        }
    }
    if (!chunked.empty()) {
        ProfScope prof("merge_chunks", 16.0 * pr.m_out * static_cast<double>(chunked_rows), st);
        merge_step_kernel<<<merge_grid, kRrWarps * 32, 0, st>>>(segs.get(), static_cast<int>(chunked.size()), chunked_rows,
                                                                -1, ext_ids.get(), ext_dists.get(), pr.m_out, seeds.get(),
                                                                pr.out_ids, pr.out_dists);
        count_launches(1);
        GTA_CUDA(cudaGetLastError());
    }
}

}  // namespace gta
