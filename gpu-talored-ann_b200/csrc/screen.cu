// screen.cu -- the float-row distance screen of the bucketed kNN build on sm_100a.
//
// For float rows the exact distance of the build is the ascending-dimension fp32 fmaf chain
// (the reference's exact rerank, bucketDemo/buildBucket/src/bucket.cu:4350-4363 s6_dot_rows),
// which no tensor-core contraction reproduces.  The build screens on the tensor cores and
// recomputes the survivors exactly, as the reference's s6 path does (bucket.cu:4458
// s6_scan_kernel: fp16 screen with a strict error bound; :4604 s6_rerank_kernel: exact
// rerank):
//
//   screen_kernel   per A row, every B column whose approximate distance lies within a proven
//                   margin of the row's M-th smallest (the candidates);
//   rerank          the candidates' exact distances and the top-M (dist_topk.cu rerank_kernel,
//                   reading the dataset's own rows).
//
// Operands: each row x is scaled by a power of two S (exact; S = 2^floor(log2(2^15 / max ||x||)),
// so every coordinate stays below 2^15) and split into fp16 parts hi = rn(S x) and
// lo = rn(S x - hi).  kind::f16 MMAs form hi.hi + hi.lo + lo.hi (the dropped lo.lo and the
// rounding of lo are below 3 * 2^-22 of |x||y|); with one part only hi.hi.  Products of fp16
// values are exact in fp32, so the error left is the parts' rounding and the fp32
// accumulation, both bounded in the margin.
//
// CTA = 128 A rows against one bucket segment, one CTA per SM:
//   warp 0      TMA producer: per K chunk of 64 fp16, the A and B parts (128 x 128 B each)
//               into a 4-6 stage ring;
//   warp 1      TMEM allocator (all 512 columns) + single-thread tcgen05.mma issuer into two
//               128-column accumulators (column tile j+1 overlaps the epilogue of tile j);
//   warps 2..5  epilogue: thread t owns TMEM lane t = A row t.  Scores of 16 columns at a time
//               (tcgen05.ld), approximate distance S^2 (||b||^2 - 2 a.b + ||a||^2) by packed
//               f32x2 arithmetic, the admission test by sign bits, admitted columns staged in
//               shared memory and merged (bitonic) into the row's sorted list of kL 32-bit keys
//               kept in TMEM columns 256.. (key = distance code << col_bits | column).
// The distance code is the distance's float bits rounded UP to its top 32 - col_bits bits:
// decode(code) >= the distance > decode(code - 1), and the admission threshold and the final
// bound are taken from decoded codes, so every test errs toward admitting.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cfloat>
#include <cmath>
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
    int32_t* cand_cols;        // [a_total x L] segment columns
    int32_t* cand_n;           // [a_total] candidates, -1: rescan the row exactly
    unsigned long long* stats; // optional: the library's eight profile counters
    int* err;
    uint32_t buf_off, pn_off, bar_off;
};

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

__device__ __forceinline__ int tile_order(int k, int t0, int n_ct)
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

template <int kL, bool kSplit>
__global__ void __launch_bounds__(kSThreads, 1) screen_kernel(const __grid_constant__ CUtensorMap tm, const ScreenArgs p)
{
    constexpr int kParts = kSplit ? 2 : 1;
    constexpr uint32_t kStageBytes = 2u * kParts * kSChunk;  // A parts then B parts
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
    const int t0 = (w.self_col0 >= 0) ? min(n_ct - 1, w.self_col0 / kSTile) : 0;
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
                        const int x = q * p.part_stride + kc * 64;
                        tma_load_2d(dst + static_cast<uint32_t>(q) * kSChunk, &tm, S_FULL(s), x, w.a_row0);
                        tma_load_2d(dst + static_cast<uint32_t>(kParts + q) * kSChunk, &tm, S_FULL(s), x,
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
            bool ok = true;
            long long wait_acc = 0, wait_full = 0;
            int it = 0;
            for (int k = 0; k < n_ct && ok; ++k) {
                const int b = k & 1;
                const uint32_t use = static_cast<uint32_t>(k >> 1);
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
                    const uint64_t ah = smem_desc_sw128(sa), bh = smem_desc_sw128(sa + kParts * kSChunk);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {  // 4 x 16 fp16 of K per 128-byte chunk
                        umma<false>(d_tmem, ah + 2ull * kk, bh + 2ull * kk, idesc, (kc | kk) != 0 ? 1u : 0u);
                        if constexpr (kSplit) {
                            const uint64_t al = smem_desc_sw128(sa + kSChunk), bl = smem_desc_sw128(sa + 3u * kSChunk);
                            umma<false>(d_tmem, ah + 2ull * kk, bl + 2ull * kk, idesc, 1u);
                            umma<false>(d_tmem, al + 2ull * kk, bh + 2ull * kk, idesc, 1u);
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
        const int shift = p.col_bits - 1;
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
        auto decode = [&](uint32_t code) { return __uint_as_float(code << shift); };
        auto refresh_thr = [&]() {
            const uint32_t kl = tmem_ld1(tl + static_cast<uint32_t>(kL - 1));
            const uint32_t km = tmem_ld1(tl + static_cast<uint32_t>(p.m_sel - 1));
            float t = kl == kSEmpty ? FLT_MAX : decode(kl >> p.col_bits);
            if (km != kSEmpty) t = fminf(t, decode(km >> p.col_bits) + margin);
            if (row_ok) thr = t;
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
        const int self_col = w.self_col0 >= 0 ? w.self_col0 + r : -1;
        const int self_ct = self_col >= 0 ? self_col / kSTile : -1;
        const int self_c = (self_col % kSTile) >> 4;
        const int self_el = self_col & 15;
        const unsigned long long an2 = f2_pack(an_s, an_s), m2 = f2_pack(-2.0f, -2.0f);
        prefetch_cols(0);
        for (int k = 0; k < n_ct && ok; ++k) {
            const int ct = tile_order(k, t0, n_ct);
            const int b = k & 1;
            const uint32_t use = static_cast<uint32_t>(k >> 1);
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
            uint32_t va[16], vb[16];
            // one slice of 16 columns: approximate distances by packed f32x2 arithmetic, the
            // admission test dist <= thr as the sign of thr - dist (an IEEE difference is +0 exactly
            // on equality and never takes the wrong sign), then this lane's admitted columns
            auto scan_slice = [&](int c, const uint32_t (&v)[16], uint32_t (&nxt)[16], bool nxt_in_flight) {
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
                        if (nxt_in_flight) tmem_ld_wait_regs(nxt);  // no TMEM load in flight across the call
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
                            const uint32_t bits = __float_as_uint(fmaxf(dist[e], 0.0f));
                            const uint32_t code = (bits + ((1u << shift) - 1u)) >> shift;
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
            tmem_ld_32x32b_x16(tbase, va);
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const bool more = c + 1 < 8;
                if ((c & 1) == 0) {
                    tmem_ld_wait_regs(va);
                    if (more) {
                        __syncwarp();
                        tmem_ld_32x32b_x16(tbase + static_cast<uint32_t>((c + 1) * 16), vb);
                    } else {
                        release_acc();
                    }
                    scan_slice(c, va, vb, more);
                } else {
                    tmem_ld_wait_regs(vb);
                    if (more) {
                        __syncwarp();
                        tmem_ld_32x32b_x16(tbase + static_cast<uint32_t>((c + 1) * 16), va);
                    } else {
                        release_acc();
                    }
                    scan_slice(c, vb, va, more);
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
            // candidates: the list's keys whose distance may lie within the bound (sorted: a prefix);
            // overflow when keys beyond the list may as well
            const uint32_t km = tmem_ld1(tl + static_cast<uint32_t>(p.m_sel - 1));
            const float bnd = km == kSEmpty ? INFINITY : decode(km >> p.col_bits) + margin;
            const uint32_t kl = tmem_ld1(tl + static_cast<uint32_t>(kL - 1));
            auto may_pass = [&](uint32_t key) {
                const uint32_t code = key >> p.col_bits;
                return key != kSEmpty && (code == 0u || decode(code - 1u) < bnd);
            };
            const bool overflow = may_pass(kl);
            int nc = 0;
            bool open = true;
#pragma unroll 1
            for (int blk = 0; blk < kL; blk += 32) {
                uint32_t c[32];
                tmem_ld_32x32b_x32(tl + static_cast<uint32_t>(blk), c);
                tmem_ld_wait_regs32(c);
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    open = open && may_pass(c[j]);
                    if (row_ok && !overflow && open) p.cand_cols[arow * kL + blk + j] = static_cast<int32_t>(c[j] & col_mask);
                    nc += open ? 1 : 0;
                }
            }
            if (row_ok) p.cand_n[arow] = overflow ? -1 : nc;
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

// ---- operand rows: scaled fp16 parts ---------------------------------------------------
// One warp per pool row: row j of the pool is dataset row ids[j]; out row j holds its hi part
// (d16 fp16, zero past d) and, with two parts, its lo part after d16 elements.
template <typename T>
__global__ void split_rows_kernel(const T* __restrict__ X, int d, const int32_t* __restrict__ ids, int64_t n,
                                  const float* __restrict__ maxnorm, __half* __restrict__ out, int d16, int parts)
{
    const int lane = threadIdx.x & 31;
    const int64_t j = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (j >= n) return;
    const float sc = screen_scale(*maxnorm);
    const T* x = X + static_cast<int64_t>(ids[j]) * d;
    __half* o = out + j * static_cast<int64_t>(parts) * d16;
    for (int i = lane; i < d16; i += 32) {
        const float v = i < d ? to_f32(x[i]) * sc : 0.0f;
        const __half h = __float2half_rn(v);
        o[i] = h;
        if (parts == 2) o[d16 + i] = __float2half_rn(v - __half2float(h));
    }
}

// ---- exact rerank ------------------------------------------------------------------------
// One warp per A row of a work item: the row's candidates (or, after an overflow, every column
// of its segment but itself) with the exact fp32 chain over the dataset's own rows, as
// (distance, output id) keys; a bitonic sort; the first m_out written.  Two candidates per lane
// at a time (independent chains), rows read four elements per load where aligned.
constexpr int kRrWarps = 4;
constexpr int kRrKeys = 512;

template <typename T>
__device__ __forceinline__ float chain_dist(const float* __restrict__ a, const T* __restrict__ b, int d)
{
    float acc = 0.0f;
    for (int i = 0; i < d; ++i) {
        const float t = a[i] - to_f32(b[i]);
        acc = fmaf(t, t, acc);
    }
    return acc;
}

// two independent chains (same order of operations as chain_dist for each)
__device__ __forceinline__ void chain_dist2_f4(const float* __restrict__ a, const float* __restrict__ b0,
                                               const float* __restrict__ b1, int d, float& o0, float& o1)
{
    float acc0 = 0.0f, acc1 = 0.0f;
    const float4* a4 = reinterpret_cast<const float4*>(a);
    const float4* p0 = reinterpret_cast<const float4*>(b0);
    const float4* p1 = reinterpret_cast<const float4*>(b1);
    for (int i = 0; i < d / 4; ++i) {
        const float4 x = a4[i], u = __ldg(p0 + i), v = __ldg(p1 + i);
        float t;
        t = x.x - u.x; acc0 = fmaf(t, t, acc0);
        t = x.x - v.x; acc1 = fmaf(t, t, acc1);
        t = x.y - u.y; acc0 = fmaf(t, t, acc0);
        t = x.y - v.y; acc1 = fmaf(t, t, acc1);
        t = x.z - u.z; acc0 = fmaf(t, t, acc0);
        t = x.z - v.z; acc1 = fmaf(t, t, acc1);
        t = x.w - u.w; acc0 = fmaf(t, t, acc0);
        t = x.w - v.w; acc1 = fmaf(t, t, acc1);
    }
    o0 = acc0;
    o1 = acc1;
}

__device__ __forceinline__ void rr_sort(uint64_t* keys, int n, int lane)
{
    for (int k = 2; k <= n; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int t = lane; t < (n >> 1); t += 32) {
                const int i = 2 * j * (t / j) + (t % j);
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
    const WorkItem* work;
    const void* X;
    int d;
    int vec4;                  // float rows, d % 4 == 0, 16-byte aligned rows: four-element loads
    const int32_t* ids;        // pool row -> dataset row
    const int32_t* gid;        // pool row -> output id
    const int32_t* cand_cols;
    const int32_t* cand_n;
    int L;
    int m_out;
    int32_t* out_ids;
    float* out_dists;
};

template <typename T>
__global__ void __launch_bounds__(kRrWarps * 32) rerank_x_kernel(const RerankX p)
{
    extern __shared__ uint8_t sm[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t* keys = reinterpret_cast<uint64_t*>(sm) + warp * kRrKeys;
    const int d4 = (p.d + 3) / 4 * 4;
    float* arow_s = reinterpret_cast<float*>(sm + kRrWarps * kRrKeys * sizeof(uint64_t)) + warp * d4;
    const WorkItem w = p.work[blockIdx.x];
    const T* X = static_cast<const T*>(p.X);
    auto brow_ptr = [&](int c) { return X + static_cast<int64_t>(p.ids[static_cast<int64_t>(w.b_row0) + c]) * p.d; };
    auto out_id = [&](int c) { return static_cast<uint32_t>(p.gid[static_cast<int64_t>(w.b_row0) + c]); };
    for (int r = warp; r < w.a_rows; r += kRrWarps) {
        const int64_t arow = static_cast<int64_t>(w.a_row0) + r;
        const T* xa = X + static_cast<int64_t>(p.ids[arow]) * p.d;
        for (int i = lane; i < d4; i += 32) arow_s[i] = i < p.d ? to_f32(xa[i]) : 0.0f;
        __syncwarp();
        const int n = p.cand_n[arow];
        const int self = (w.self_col0 >= 0) ? w.self_col0 + r : -1;
        int n_sorted = 0;
        if (n >= 0) {
            int np2 = 1;
            while (np2 < n) np2 <<= 1;
            const int32_t* cc = p.cand_cols + arow * p.L;
            for (int j0 = 0; j0 < np2; j0 += 64) {
                const int ja = j0 + lane, jb = j0 + 32 + lane;
                const bool va = ja < n, vb = jb < n;
                const int ca = va ? cc[ja] : 0, cb = vb ? cc[jb] : 0;
                float da = 0.0f, db = 0.0f;
                if constexpr (sizeof(T) == 4) {
                    if (p.vec4 && va && vb) {
                        chain_dist2_f4(arow_s, reinterpret_cast<const float*>(brow_ptr(ca)),
                                       reinterpret_cast<const float*>(brow_ptr(cb)), p.d, da, db);
                    } else {
                        if (va) da = chain_dist(arow_s, brow_ptr(ca), p.d);
                        if (vb) db = chain_dist(arow_s, brow_ptr(cb), p.d);
                    }
                } else {
                    if (va) da = chain_dist(arow_s, brow_ptr(ca), p.d);
                    if (vb) db = chain_dist(arow_s, brow_ptr(cb), p.d);
                }
                if (ja < np2) keys[ja] = va ? (static_cast<uint64_t>(f2key(da)) << 32) | out_id(ca) : ~0ull;
                if (jb < np2) keys[jb] = vb ? (static_cast<uint64_t>(f2key(db)) << 32) | out_id(cb) : ~0ull;
            }
            __syncwarp();
            rr_sort(keys, np2, lane);
            n_sorted = np2;
        } else {
            // exact rescan of the whole segment: keys[0, 256) the best so far, [256, 512) the next chunk
            for (int j = lane; j < kRrKeys; j += 32) keys[j] = ~0ull;
            __syncwarp();
            for (int c0 = 0; c0 < w.b_rows; c0 += kRrKeys / 2) {
                for (int j = lane; j < kRrKeys / 2; j += 32) {
                    const int c = c0 + j;
                    uint64_t key = ~0ull;
                    if (c < w.b_rows && c != self)
                        key = (static_cast<uint64_t>(f2key(chain_dist(arow_s, brow_ptr(c), p.d))) << 32) | out_id(c);
                    keys[kRrKeys / 2 + j] = key;
                }
                __syncwarp();
                rr_sort(keys, kRrKeys, lane);
            }
            n_sorted = kRrKeys / 2;
        }
        for (int j = lane; j < p.m_out; j += 32) {
            const uint64_t key = j < n_sorted ? keys[j] : ~0ull;
            const bool v = key != ~0ull;
            p.out_ids[arow * p.m_out + j] = v ? static_cast<int32_t>(static_cast<uint32_t>(key)) : -1;
            p.out_dists[arow * p.m_out + j] = v ? key2f(static_cast<uint32_t>(key >> 32)) : INFINITY;
        }
        __syncwarp();
    }
}

struct ScreenPlan {
    int stages = 0;
    uint32_t buf_off = 0, pn_off = 0, bar_off = 0, total = 0;
};

bool screen_plan(bool split, ScreenPlan& pl)
{
    const uint32_t stage_bytes = 2u * (split ? 2u : 1u) * kSChunk;
    for (int S = 6; S >= 2; --S) {
        ScreenPlan t;
        t.stages = S;
        uint32_t off = static_cast<uint32_t>(S) * stage_bytes;
        t.buf_off = off;
        off += static_cast<uint32_t>(kSBuf) * 128u * 4u;
        t.pn_off = off;
        off += 4u * kSTile * 4u;
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

template <int kL, bool kSplit>
void launch_screen(const CUtensorMap& tm, const ScreenArgs& a, int n_work, uint32_t smem, cudaStream_t st)
{
    auto fn = screen_kernel<kL, kSplit>;
    GTA_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    fn<<<n_work, kSThreads, smem, st>>>(tm, a);
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

}  // namespace

int screen_list_len(int m) { return m <= 64 ? 128 : 256; }

void screen_knn(const ScreenProblem& pr, cudaStream_t st)
{
    if (pr.n_work == 0) return;
    GTA_REQUIRE(pr.X && pr.ids && pr.gid && pr.work && pr.out_ids && pr.out_dists, kInvalid, "screen: null operand");
    GTA_REQUIRE(pr.dtype == GTA_F32 || pr.dtype == GTA_U8 || pr.dtype == GTA_I8, kInvalid, "screen: bad dtype");
    GTA_REQUIRE(pr.d >= 1 && pr.m_out >= 1 && pr.m_out <= 128 && pr.max_cols >= 1 && pr.max_cols <= (1 << 17),
                kInvalid, "screen: unsupported shape");
    GTA_REQUIRE(pr.parts == 1 || pr.parts == 2, kInvalid, "screen: one or two operand parts");
    const bool split = pr.parts == 2;
    const int L = screen_list_len(pr.m_out);
    const int d16 = (pr.d + 63) / 64 * 64;
    ScreenPlan pl;
    GTA_REQUIRE(screen_plan(split, pl), kInvalid, "screen: shared memory plan failed");
    // exact squared norms, the scale's source (max ||x||) and the scaled fp16 operand rows
    DevBuf<float> norm(static_cast<size_t>(pr.n_rows), st), bmax(1, st);
    DevBuf<__half> rows(static_cast<size_t>(pr.n_rows) * pr.parts * d16, st);
    {
        const double in_bytes = static_cast<double>(pr.n_rows) * pr.d * (pr.dtype == GTA_F32 ? 4.0 : 1.0);
        ProfScope prof("screen_rows", 2.0 * in_bytes + static_cast<double>(pr.n_rows) * 2.0 * pr.parts * d16, st);
        convert_rows(pr.X, pr.dtype, pr.d, pr.ids, pr.n_rows, nullptr, kElemF32, pr.d, norm.get(), st);
        max_sqrt(norm.get(), pr.n_rows, bmax.get(), st);
        const int wpb = 8;
        const unsigned grid = static_cast<unsigned>((pr.n_rows + wpb - 1) / wpb);
        if (pr.dtype == GTA_F32)
            split_rows_kernel<float><<<grid, wpb * 32, 0, st>>>(static_cast<const float*>(pr.X), pr.d, pr.ids,
                                                                pr.n_rows, bmax.get(), rows.get(), d16, pr.parts);
        else if (pr.dtype == GTA_U8)
            split_rows_kernel<uint8_t><<<grid, wpb * 32, 0, st>>>(static_cast<const uint8_t*>(pr.X), pr.d, pr.ids,
                                                                  pr.n_rows, bmax.get(), rows.get(), d16, pr.parts);
        else
            split_rows_kernel<int8_t><<<grid, wpb * 32, 0, st>>>(static_cast<const int8_t*>(pr.X), pr.d, pr.ids,
                                                                 pr.n_rows, bmax.get(), rows.get(), d16, pr.parts);
        count_launches(1);
        GTA_CUDA(cudaGetLastError());
    }
    CUtensorMap tm;
    {
        cuuint64_t dims[2] = {static_cast<cuuint64_t>(pr.parts) * d16, static_cast<cuuint64_t>(pr.n_rows)};
        cuuint64_t strides[1] = {static_cast<cuuint64_t>(pr.parts) * d16 * 2u};
        cuuint32_t box[2] = {64u, 128u};
        cuuint32_t estr[2] = {1u, 1u};
        const CUresult r = screen_encode()(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, rows.get(), dims, strides, box, estr,
                                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        GTA_REQUIRE(r == CUDA_SUCCESS, kCuda, "cuTensorMapEncodeTiled failed (" + std::to_string(static_cast<int>(r)) + ")");
    }
    DevBuf<int32_t> cand_cols(static_cast<size_t>(pr.n_rows) * L, st), cand_n(static_cast<size_t>(pr.n_rows), st);
    ScreenArgs a{};
    a.work = pr.work;
    a.norm = norm.get();
    a.maxnorm = bmax.get();
    a.k_chunks = d16 / 64;
    a.part_stride = d16;
    a.m_sel = pr.m_out;
    a.stages = pl.stages;
    a.col_bits = pr.max_cols <= (1 << 16) ? 16 : 17;
    // error bound of the screened distance (the margin, applied to the M-th key): operand parts
    // (split: 3 * 2^-22 of |a||b|, one part: 2^-10), fp32 accumulation of the products (2^-22
    // per product, 3 d products split, d single), fp32 norms and the two fused operations, with
    // a 1.25 safety factor; the bound is on |a.b| <= |a| |b| <= |a| bmax
    const double dd = pr.d;
    const double part_err = split ? 3.0 * std::ldexp(1.0, -22) : std::ldexp(1.0, -10);
    const double n_prod = split ? 3.0 * dd : dd;
    a.mc1 = static_cast<float>(1.25 * 4.0 * (part_err + n_prod * std::ldexp(1.0, -22)));
    a.mc2 = static_cast<float>(1.25 * 3.0 * (dd + 4.0) * std::ldexp(1.0, -24));
    a.cand_cols = cand_cols.get();
    a.cand_n = cand_n.get();
    a.err = pr.err;
    a.buf_off = pl.buf_off;
    a.pn_off = pl.pn_off;
    a.bar_off = pl.bar_off;
    {
        ProfScope prof(pr.prof_name, pr.flops, st);
        a.stats = prof.counters(8);
        if (L == 128) {
            if (split) launch_screen<128, true>(tm, a, pr.n_work, pl.total, st);
            else launch_screen<128, false>(tm, a, pr.n_work, pl.total, st);
        } else {
            if (split) launch_screen<256, true>(tm, a, pr.n_work, pl.total, st);
            else launch_screen<256, false>(tm, a, pr.n_work, pl.total, st);
        }
    }
    RerankX r{};
    r.work = pr.work;
    r.X = pr.X;
    r.d = pr.d;
    r.vec4 = (pr.dtype == GTA_F32 && pr.d % 4 == 0 && (reinterpret_cast<uintptr_t>(pr.X) & 15) == 0) ? 1 : 0;
    r.ids = pr.ids;
    r.gid = pr.gid;
    r.cand_cols = cand_cols.get();
    r.cand_n = cand_n.get();
    r.L = L;
    r.m_out = pr.m_out;
    r.out_ids = pr.out_ids;
    r.out_dists = pr.out_dists;
    const size_t smem = kRrWarps * kRrKeys * sizeof(uint64_t) + kRrWarps * static_cast<size_t>((pr.d + 3) / 4 * 4) * 4;
    GTA_REQUIRE(smem <= kSSmemMax, kInvalid, "rerank: dimension too large");
    ProfScope prof("rerank", 0.0, st);
    if (pr.dtype == GTA_F32) {
        GTA_CUDA(cudaFuncSetAttribute(rerank_x_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
        rerank_x_kernel<float><<<pr.n_work, kRrWarps * 32, smem, st>>>(r);
    } else if (pr.dtype == GTA_U8) {
        GTA_CUDA(cudaFuncSetAttribute(rerank_x_kernel<uint8_t>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
        rerank_x_kernel<uint8_t><<<pr.n_work, kRrWarps * 32, smem, st>>>(r);
    } else {
        GTA_CUDA(cudaFuncSetAttribute(rerank_x_kernel<int8_t>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
        rerank_x_kernel<int8_t><<<pr.n_work, kRrWarps * 32, smem, st>>>(r);
    }
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

}  // namespace gta
