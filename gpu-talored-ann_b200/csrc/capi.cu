// capi.cu -- host orchestration of the bucketed kNN / CAGRA build and the C ABI of libgta.
//
// The pipeline mirrors the reference's bucket2 GPU-resident path
// (bucketDemo/buildBucket/src/bucket.cu:8523 run_pipeline_impl): centroids,
// bucket assignment, per-bucket kNN, merge, then CAGRA optimize.  Every stage
// runs on the GPU; there is no CPU fallback.  Host code only sequences
// launches, builds the per-CTA work list from the bucket sizes, and moves the
// caller's host buffers.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <numeric>
#include <string>
#include <vector>
#include <memory>
#include <unistd.h>

#include "../../include/gta.h"
#include "gta_internal.h"
#include "prof.h"

#include <atomic>
#include <mutex>

namespace gta {

namespace {
std::mutex g_prof_mu;
bool g_prof_on = false;
std::vector<ProfRecord> g_prof;

void prof_clear()
{
    for (auto& r : g_prof) {
        if (r.start) cudaEventDestroy(r.start);
        if (r.stop) cudaEventDestroy(r.stop);
        if (r.counters) cudaFree(r.counters);
    }
    g_prof.clear();
}
}  // namespace

bool prof_enabled() { return g_prof_on; }

// ---------------------------------------------------------------- workspace arenas
namespace {
struct Arena {
    char* base = nullptr;
    size_t cap = 0;   // bytes held
    size_t off = 0;   // bump offset of the running call
    size_t want = 0;  // high-water mark seen (arena size for the next call)
};
std::mutex g_ws_mu;
std::vector<std::pair<std::pair<int, cudaStream_t>, Arena*>> g_arenas;
thread_local Arena* t_arena = nullptr;
thread_local int t_depth = 0;

Arena* arena_for(int dev, cudaStream_t st)
{
    std::lock_guard<std::mutex> g(g_ws_mu);
    for (auto& e : g_arenas)
        if (e.first.first == dev && e.first.second == st) return e.second;
    g_arenas.push_back({{dev, st}, new Arena()});
    return g_arenas.back().second;
}
}  // namespace

WorkspaceScope::WorkspaceScope(cudaStream_t st)
{
    if (t_depth++ > 0) return;  // nested entry points share the outer call's arena
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return;
    Arena* a = arena_for(dev, st);
    if (a->want > a->cap) {
        if (a->base) {
            cudaStreamSynchronize(st);
            cudaFree(a->base);
            a->base = nullptr;
            a->cap = 0;
        }
        void* p = nullptr;
        if (cudaMalloc(&p, a->want) == cudaSuccess) {
            a->base = static_cast<char*>(p);
            a->cap = a->want;
        } else {
            cudaGetLastError();  // fall back to the stream-ordered allocator for this call
        }
    }
    a->off = 0;
    t_arena = a;
    active_ = true;
}

WorkspaceScope::~WorkspaceScope()
{
    --t_depth;
    if (!active_) return;
    t_arena = nullptr;
}

void* workspace_alloc(size_t bytes, cudaStream_t st, bool* from_arena)
{
    const size_t aligned = (bytes + 255) & ~static_cast<size_t>(255);
    Arena* a = t_arena;
    if (a) {
        const size_t end = a->off + aligned;
        if (end > a->want) a->want = end;
        if (a->base && end <= a->cap) {
            void* p = a->base + a->off;
            a->off = end;
            *from_arena = true;
            return p;
        }
        a->off = end;  // account for it so the next call's arena covers this call
    }
    void* p = nullptr;
    GTA_CUDA(cudaMallocAsync(&p, bytes, st));
    *from_arena = false;
    return p;
}
namespace {
std::atomic<long long> g_launches{0};
}
void count_launches(long long n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
void prof_push(ProfRecord&& r)
{
    std::lock_guard<std::mutex> g(g_prof_mu);
    g_prof.push_back(std::move(r));
}

namespace {

thread_local std::string g_err;

template <typename F>
int guard(F&& f)
{
    try {
        f();
        return kOk;
    } catch (const Error& e) {
        g_err = e.what();
        return e.code;
    } catch (const std::bad_alloc&) {
        g_err = "host out of memory";
        return kNoMem;
    } catch (const std::exception& e) {
        g_err = e.what();
        return kInvalid;
    }
}

// Keep memory freed by the stream-ordered allocator cached in the device's default pool, so the
// per-call scratch of repeated builds is not returned to and re-mapped from the driver each time.
void keep_pool_memory()
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return;
    static std::mutex mu;
    static std::vector<int> done;
    std::lock_guard<std::mutex> g(mu);
    for (int x : done) if (x == dev) return;
    cudaMemPool_t pool;
    if (cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess) {
        uint64_t thr = UINT64_MAX;
        cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr);
    }
    done.push_back(dev);
}

inline cudaStream_t S(void* s)
{
    keep_pool_memory();
    return static_cast<cudaStream_t>(s);
}

#define GTA_WORKSPACE(stream) ::gta::WorkspaceScope ws_scope_(S(stream))

// operand rows padded to 128-byte multiples (one TMA / MMA K chunk)
int pad_dim(int d, int elem) { const int q = 128 / elem_bytes(elem); return (d + q - 1) / q * q; }

int elem_size(int dtype) { return dtype == GTA_F32 ? 4 : 1; }

// 8-bit rows are exact in bf16, and with 2*d*max|x|^2 < 2^24 every product,
// partial sum and distance of the fused epilogue is an exact fp32 integer.
bool exact_bf16(int dtype, int d)
{
    if (dtype == GTA_U8) return 2.0 * d * 255.0 * 255.0 < 16777216.0;
    if (dtype == GTA_I8) return 2.0 * d * 128.0 * 128.0 < 16777216.0;
    return false;
}

// Operand type of the bucket kNN: the dataset's own bytes for u8 rows when the 8-bit MMA path
// applies (lists of at most 64), bf16 for other exact 8-bit rows, else f32 (tf32 screen).
int knn_elem(int dtype, int d, int M)
{
    if (!exact_bf16(dtype, d)) return kElemF32;
    if (dtype == GTA_U8 && dist_topk_u8_fits(pad_dim(d, kElemU8), M)) return kElemU8;
    return kElemBF16;
}

void copy_rows_padded(float* dst, int d_pad, const float* src, int d, int64_t n, bool src_dev, cudaStream_t st)
{
    GTA_CUDA(cudaMemsetAsync(dst, 0, sizeof(float) * static_cast<size_t>(n) * d_pad, st));
    GTA_CUDA(cudaMemcpy2DAsync(dst, sizeof(float) * d_pad, src, sizeof(float) * d, sizeof(float) * d, n,
                               src_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, st));
}

void unpad_rows(float* dst, int d, const float* src, int d_pad, int64_t n, bool dst_dev, cudaStream_t st)
{
    GTA_CUDA(cudaMemcpy2DAsync(dst, sizeof(float) * d, src, sizeof(float) * d_pad, sizeof(float) * d, n,
                               dst_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, st));
}

template <typename T>
DevBuf<T> upload(const std::vector<T>& h, cudaStream_t st)
{
    DevBuf<T> d(h.size(), st);
    if (!h.empty()) GTA_CUDA(cudaMemcpyAsync(d.get(), h.data(), sizeof(T) * h.size(), cudaMemcpyHostToDevice, st));
    return d;
}

// ---------------------------------------------------------------- stages

// Top-k nearest rows of C (B x d_pad, norms cn) for rows of Xp (n x d_pad, norms xn).
// int_rows: every value of the rows Xp is an integer exact in tf32 (8-bit data).  The tensor-core
// screen then runs on split operands ([x | x] against [hi | lo] centroids, K = 2d) whose dot products
// are within 2^-20 of exact, so far fewer candidates need the exact rerank.  X2 (optional): the
// [x | x] rows already built (pitch pad_dim(2d)).
void assign_topk_impl(const float* Xp, const float* xn, int64_t n, int d, int d_pad, const float* Cp, const float* cn,
                      int B, int k, int32_t* ids, float* dists, int* err, cudaStream_t st, bool int_rows = false,
                      const float* X2 = nullptr)
{
    GTA_REQUIRE(k >= 1 && k <= B, kInvalid, "assign: need 1 <= k <= B");
    if (assign_exact_applies(B, k)) {  // few centroids: exact chain on the FP32 pipe, no screen
        assign_exact(Xp, GTA_F32, n, d_pad, d, nullptr, Cp, d_pad, B, k, ids, dists, st);
        return;
    }
    DevBuf<float> A2, C2;
    const int pitch2 = pad_dim(2 * d, kElemF32);
    if (int_rows) {
        if (!X2) {
            A2 = DevBuf<float>(static_cast<size_t>(n) * pitch2, st);
            dup_rows(Xp, d, d_pad, n, A2.get(), pitch2, st);
            X2 = A2.get();
        }
        C2 = DevBuf<float>(static_cast<size_t>(B) * pitch2, st);
        split_rows_tf32(Cp, d, d_pad, B, C2.get(), pitch2, st);
    }
    std::vector<WorkItem> wl;
    wl.reserve(static_cast<size_t>((n + 127) / 128));
    for (int64_t r = 0; r < n; r += 128)
        wl.push_back(WorkItem{static_cast<int32_t>(r), static_cast<int32_t>(std::min<int64_t>(128, n - r)), 0, B, -1, 0, 0, 0});
    auto work = upload(wl, st);
    DistTopkProblem pr;
    pr.A = Xp; pr.a_total = n; pr.B = Cp; pr.b_total = B; pr.elem = kElemF32; pr.d = d; pr.d_pad = d_pad;
    pr.a_norm = xn; pr.b_norm = cn; pr.b_gid = nullptr; pr.work = work.get(); pr.n_work = static_cast<int>(wl.size());
    pr.m_out = k; pr.exclude_self = false; pr.out_ids = ids; pr.out_dists = dists; pr.err = err;
    pr.prof_name = "dist_topk_assign";
    pr.flops = 2.0 * static_cast<double>(n) * B * d;
    if (int_rows) {
        pr.A = X2; pr.B = C2.get(); pr.d_pad = pitch2;
        pr.b_exact = Cp; pr.b_exact_pitch = d_pad;
        pr.screen_trunc = 0x1p-19;
        pr.screen_k = 2 * d;
    }
    dist_topk(pr, st);
}

// Top-k of bf16 rows (8-bit data held exactly) against bf16 centroid rows: the tensor-core path
// with exact integer distances, no screen and no rerank.
void assign_topk_bf16(const void* Xb, const float* xn, int64_t n, int d, int d_pad, const void* Cb, const float* cn,
                      int B, int k, int32_t* ids, float* dists, int* err, cudaStream_t st)
{
    GTA_REQUIRE(k >= 1 && k <= B, kInvalid, "assign: need 1 <= k <= B");
    std::vector<WorkItem> wl;
    wl.reserve(static_cast<size_t>((n + 127) / 128));
    for (int64_t r = 0; r < n; r += 128)
        wl.push_back(WorkItem{static_cast<int32_t>(r), static_cast<int32_t>(std::min<int64_t>(128, n - r)), 0, B, -1, 0, 0, 0});
    auto work = upload(wl, st);
    DistTopkProblem pr;
    pr.A = Xb; pr.a_total = n; pr.B = Cb; pr.b_total = B; pr.elem = kElemBF16; pr.d = d; pr.d_pad = d_pad;
    pr.a_norm = xn; pr.b_norm = cn; pr.b_gid = nullptr; pr.work = work.get(); pr.n_work = static_cast<int>(wl.size());
    pr.m_out = k; pr.exclude_self = false; pr.out_ids = ids; pr.out_dists = dists; pr.err = err;
    pr.prof_name = "dist_topk_assign";
    pr.flops = 2.0 * static_cast<double>(n) * B * d;
    dist_topk(pr, st);
}

// The sample's rows in the dataset's own element type (for the exact assignment, which then
// reads 8-bit rows instead of the f32 copy): row_ids[i] is sample row i's row of X.
struct RawRows {
    const void* X = nullptr;
    int dtype = GTA_F32;
    int ldx = 0;
    const int32_t* row_ids = nullptr;
};

void kmeans_fit_impl(const float* Xs, const float* xn, int64_t n_s, int d, int d_pad, float* C, float* cn, int B,
                     int iters, int32_t* assign_out, int* err, cudaStream_t st, bool integer_rows = false,
                     const RawRows& raw = RawRows())
{
    DevBuf<int32_t> ids(static_cast<size_t>(n_s), st);
    DevBuf<float> dd(static_cast<size_t>(n_s), st);
    DevBuf<float> C2(static_cast<size_t>(B) * d_pad, st);
    DevBuf<float> X2;  // [x | x] rows of the split screen, built once for all steps
    if (integer_rows && !assign_exact_applies(B, 1) && iters > 0) {
        const int pitch2 = pad_dim(2 * d, kElemF32);
        X2 = DevBuf<float>(static_cast<size_t>(n_s) * pitch2, st);
        dup_rows(Xs, d, d_pad, n_s, X2.get(), pitch2, st);
    }
    for (int it = 0; it < iters; ++it) {
        if (raw.X && assign_exact_applies(B, 1))
            assign_exact(raw.X, raw.dtype, n_s, raw.ldx, d, raw.row_ids, C, d_pad, B, 1, ids.get(), dd.get(), st);
        else
            assign_topk_impl(Xs, xn, n_s, d, d_pad, C, cn, B, 1, ids.get(), dd.get(), err, st, integer_rows, X2.get());
        centroid_update(Xs, n_s, d, d_pad, ids.get(), C, B, C2.get(), cn, err, st, integer_rows);
        GTA_CUDA(cudaMemcpyAsync(C, C2.get(), sizeof(float) * static_cast<size_t>(B) * d_pad, cudaMemcpyDeviceToDevice, st));
    }
    if (assign_out) {
        assign_topk_impl(Xs, xn, n_s, d, d_pad, C, cn, B, 1, ids.get(), dd.get(), err, st);
        GTA_CUDA(cudaMemcpyAsync(assign_out, ids.get(), sizeof(int32_t) * n_s, cudaMemcpyDeviceToDevice, st));
    }
}

// Per-bucket all-pairs top-M for every membership row.
// k-means sample size: min(0.1, 1e7 / N) of N unless given, at least B.
int64_t kmeans_sample_size(int64_t N, int64_t requested, int B)
{
    int64_t n_s = requested > 0 ? std::min<int64_t>(requested, N)
                                : std::max<int64_t>(1, std::llround(std::min(0.1, 1e7 / double(N)) * double(N)));
    return std::max<int64_t>(n_s, B);
}

// k-means++ pool: min(sample, 20 B) rows (the ratio shrinks past 1024 buckets).
int64_t kmeans_pool_size(int64_t n_s, int B)
{
    const int ratio = B <= 1024 ? 20 : std::max(2, 20 * 1024 / B);
    return std::min<int64_t>(n_s, static_cast<int64_t>(ratio) * B);
}

uint64_t kmeans_pool_seed(uint64_t seed) { return seed ^ 0x9E3779B97F4A7C15ull; }

// Which membership rows a bucket kNN call computes.  Within a bucket the memberships are grouped
// by partner (the point's other bucket): first the points for which the bucket is the higher of
// their two (partner below it), then those for which it is the lower.  The lower-bucket list of a
// point is the running side of its merge; once it is known, its M-th distance bounds the merged
// list, so the higher-bucket row only needs the columns within that distance that are not also
// members of the lower bucket (those are in the lower list already, or beyond its M-th): the
// merged lists are unchanged (running side first on equal distance, ids of the running list
// dropped from the new one).
struct KnnPhase {
    int phase = 0;                     // 0: all rows; 1: lower-bucket rows; 2: higher-bucket rows, seeded; 3: 1 then 2
    const int64_t* split = nullptr;    // host [B]: first membership of each bucket with its partner above it
    const int32_t* partner = nullptr;  // device [memberships]: the partner of each membership (CSR order)
    const float* seed = nullptr;       // phase 2: device, by point id, stride seed_stride
    int64_t seed_stride = 1;
    const int64_t* mem_row = nullptr;  // phase 3: seeds read from the phase-1 rows of the lists
    int64_t n_points = 0;              // phase 3: N
    const int64_t* row_lo = nullptr;   // host [B] (with row_hi): only rows [row_lo[b], row_hi[b]) of
    const int64_t* row_hi = nullptr;   // bucket b (relative to its first row) get lists; null: all
};

// members: the row of X gathered into each membership slot (grouped by bucket);
// gid: the id written to the lists for each slot (members when null).
// Buckets [b_lo, b_hi) (all when b_hi < 0) of the membership CSR: list row j - offsets[b_lo] is
// membership j.  off_host: the offsets already on the host (else read from offsets_dev).
void bucket_knn_impl(const void* X, int dtype, int64_t n, int d, const int32_t* members, const int64_t* offsets_dev,
                     int B, int M, int32_t* list_ids, float* list_dists, int* err, cudaStream_t st,
                     const int32_t* gid = nullptr, int b_lo = 0, int b_hi = -1, const int64_t* off_host = nullptr,
                     const KnnPhase& ph = KnnPhase())
{
    (void)n;
    if (b_hi < 0) b_hi = B;
    std::vector<int64_t> off(static_cast<size_t>(B) + 1);
    if (off_host) {
        std::copy(off_host, off_host + B + 1, off.begin());
    } else {
        GTA_CUDA(cudaMemcpyAsync(off.data(), offsets_dev, sizeof(int64_t) * (B + 1), cudaMemcpyDeviceToHost, st));
        GTA_CUDA(cudaStreamSynchronize(st));
    }
    const int64_t j0 = off[static_cast<size_t>(b_lo)];
    const int64_t n_mem = off[static_cast<size_t>(b_hi)] - j0;
    if (n_mem == 0) return;
    GTA_REQUIRE(n_mem < (1ll << 31), kInvalid, "bucket_knn: too many memberships on one device");
    const int elem = knn_elem(dtype, d, M);
    if (elem == kElemF32 && ph.phase == 0) {
        // float rows: tensor-core screen on fp16 parts + exact rerank over the pool's f32 rows
        std::vector<int> order(static_cast<size_t>(b_hi - b_lo));
        std::iota(order.begin(), order.end(), b_lo);
        std::stable_sort(order.begin(), order.end(),
                         [&](int a, int b) { return off[a + 1] - off[a] > off[b + 1] - off[b]; });
        ScreenProblem sp;
        sp.X = X; sp.dtype = dtype; sp.d = d;
        sp.ids = members + j0; sp.gid = (gid ? gid : members) + j0; sp.n_rows = n_mem;
        for (int b : order) {
            if (off[b + 1] == off[b]) continue;
            sp.seg_lo.push_back(off[b] - j0);
            sp.seg_n.push_back(off[b + 1] - off[b]);
            if (ph.row_lo) {
                sp.seg_r0.push_back(ph.row_lo[b]);
                sp.seg_r1.push_back(ph.row_hi[b]);
            }
        }
        sp.m_out = M; sp.parts = 2; sp.out_ids = list_ids; sp.out_dists = list_dists; sp.err = err;
        sp.prof_name = "dist_topk_bucket";
        screen_knn(sp, st);
        return;
    }
    const int d_pad = pad_dim(d, elem);
    DevBuf<uint8_t> pool(static_cast<size_t>(n_mem) * d_pad * elem_bytes(elem), st);
    DevBuf<float> pnorm(static_cast<size_t>(n_mem), st);
    {
        ProfScope prof("gather", static_cast<double>(n_mem) * (d * elem_size(dtype) + d_pad * elem_bytes(elem)), st);
        convert_rows(X, dtype, d, members + j0, n_mem, pool.get(), elem, d_pad, pnorm.get(), st);
    }
    // work list: one CTA per 128-row tile of a bucket, largest buckets first
    std::vector<int> order(static_cast<size_t>(b_hi - b_lo));
    std::iota(order.begin(), order.end(), b_lo);
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return off[a + 1] - off[a] > off[b + 1] - off[b]; });
    GTA_REQUIRE(ph.phase == 0 || (ph.split && ph.partner && (ph.phase != 2 || ph.seed) && (ph.phase != 3 || ph.mem_row)),
                kInvalid, "bucket_knn: phased rows need the split, partner and seed arrays");
    // rows [r_lo, r_hi) of bucket b's segment for a phase
    auto rows_of = [&](int b, int phase, int64_t& r_lo, int64_t& r_hi) {
        const int64_t nb = off[b + 1] - off[b];
        const int64_t s = phase == 0 ? 0 : std::min(nb, std::max<int64_t>(0, ph.split[b] - off[b]));
        r_lo = phase == 1 ? s : 0;
        r_hi = phase == 2 ? s : nb;
        if (ph.row_lo) {
            r_lo = std::max(r_lo, ph.row_lo[b]);
            r_hi = std::max(r_lo, std::min(r_hi, ph.row_hi[b]));
        }
    };
    DistTopkProblem pr;
    pr.A = pool.get(); pr.a_total = n_mem; pr.B = pool.get(); pr.b_total = n_mem; pr.elem = elem; pr.d = d;
    pr.d_pad = d_pad; pr.a_norm = pnorm.get(); pr.b_norm = pnorm.get(); pr.b_gid = (gid ? gid : members) + j0;
    pr.m_out = M; pr.exclude_self = true;
    pr.out_ids = list_ids; pr.out_dists = list_dists; pr.err = err;
    pr.prof_name = "dist_topk_bucket";
    DevBuf<float> seeds;
    auto run = [&](int phase) {
        std::vector<WorkItem> wl;
        double flops = 0.0;
        for (int b : order) {
            const int64_t lo = off[b] - j0, nb = off[b + 1] - off[b];
            int64_t r_lo = 0, r_hi = 0;
            rows_of(b, phase, r_lo, r_hi);
            for (int64_t t = r_lo; t < r_hi; t += 128)
                wl.push_back(WorkItem{static_cast<int32_t>(lo + t), static_cast<int32_t>(std::min<int64_t>(128, r_hi - t)),
                                      static_cast<int32_t>(lo), static_cast<int32_t>(nb), static_cast<int32_t>(t), 0, 0, 0});
            flops += 2.0 * static_cast<double>(r_hi - r_lo) * static_cast<double>(nb) * d;
        }
        if (wl.empty()) return;
        auto work = upload(wl, st);
        DistTopkProblem q = pr;
        q.work = work.get(); q.n_work = static_cast<int>(wl.size()); q.flops = flops;
        if (phase == 2) {
            q.prof_name = "dist_topk_bucket_seeded";
            q.partner = ph.partner + j0;
            if (ph.phase == 3) { q.seed = seeds.get(); q.seed_stride = 1; }
            else { q.seed = ph.seed; q.seed_stride = ph.seed_stride; }
        }
        dist_topk(q, st);
    };
    if (ph.phase == 3) {
        run(1);
        seeds = DevBuf<float>(static_cast<size_t>(ph.n_points), st);
        seeds_from_lists(list_dists, ph.mem_row, ph.n_points, M, j0, n_mem, seeds.get(), st);
        run(2);
    } else {
        run(ph.phase);
    }
}

// A host dataset the build reads in place (gta_dataset.on_device == 2): the pages are registered
// (pinned, mapped, read-only) for the call and the kernels read rows through the mapped address
// over the host link; nothing holds the whole dataset in device memory.
struct HostRows {
    const void* dev = nullptr;
    void* reg = nullptr;  // the registered page range (ours to unregister), or null
    cudaStream_t st;      // the stream whose kernels read the rows
    HostRows(const void* data, size_t bytes, cudaStream_t stream) : st(stream)
    {
        const long page = sysconf(_SC_PAGESIZE) > 0 ? sysconf(_SC_PAGESIZE) : 4096;
        const uintptr_t b = reinterpret_cast<uintptr_t>(data) & ~static_cast<uintptr_t>(page - 1);
        const uintptr_t e = (reinterpret_cast<uintptr_t>(data) + bytes + page - 1) & ~static_cast<uintptr_t>(page - 1);
        const cudaError_t r = cudaHostRegister(reinterpret_cast<void*>(b), e - b,
                                               cudaHostRegisterMapped | cudaHostRegisterReadOnly |
                                                   cudaHostRegisterPortable);
        if (r == cudaSuccess) {
            reg = reinterpret_cast<void*>(b);
        } else {
            (void)cudaGetLastError();  // already registered (by the caller): its mapping serves
            GTA_REQUIRE(r == cudaErrorHostMemoryAlreadyRegistered, kCuda,
                        std::string("cudaHostRegister of the host dataset failed: ") + cudaGetErrorString(r));
        }
        void* dp = nullptr;
        GTA_CUDA(cudaHostGetDevicePointer(&dp, const_cast<void*>(data), 0));
        dev = dp;
    }
    ~HostRows()
    {
        // an error thrown between launches leaves kernels that read the mapping in flight: they
        // finish before the pages are unregistered (the normal path has synchronized already)
        if (reg) {
            (void)cudaStreamSynchronize(st);
            (void)cudaHostUnregister(reg);
        }
    }
    HostRows(const HostRows&) = delete;
    HostRows& operator=(const HostRows&) = delete;
};

struct BucketOut {
    int32_t* ids;      // device [N x M]
    float* dists;      // device [N x M]
    float* centroids;  // device [B x d] or null
    int32_t* top2;     // device [N x 2] or null
};

constexpr size_t kTop2ChunkBytes = size_t(4) << 30;  // f32 rows converted at once for the top-2 pass
std::mutex g_devmem_mu;
std::map<int, size_t> g_devmem_total;  // total memory of each device, queried once

void build_bucket_round(const gta_dataset& ds, const gta_bucket_params& p, const BucketOut& o, cudaStream_t st)
{
    const int64_t N = ds.n;
    const int d = ds.d;
    const int B = p.n_buckets;
    const int M = p.knn_degree;
    GTA_REQUIRE(ds.data && N >= 2 && d >= 1, kInvalid, "build_bucket: empty dataset");
    GTA_REQUIRE(ds.dtype == GTA_F32 || ds.dtype == GTA_U8 || ds.dtype == GTA_I8, kInvalid, "build_bucket: bad dtype");
    GTA_REQUIRE(B >= 2 && B <= N, kInvalid, "build_bucket: need 2 <= n_buckets <= N (2-way membership)");
    GTA_REQUIRE(M >= 1 && M <= 128, kInvalid, "build_bucket: knn_degree must be in [1, 128]");
    GTA_REQUIRE(N < (1ll << 30), kInvalid, "build_bucket: N must be below 2^30 per device");
    GTA_REQUIRE(p.kmeans_iters >= 0, kInvalid, "build_bucket: negative kmeans_iters");

    DevBuf<int> err(1, st);
    GTA_CUDA(cudaMemsetAsync(err.get(), 0, sizeof(int), st));
    ProfScope prof_all("build_bucket_total", 0.0, st);

    // dataset on the device in its own element type, or (on_device 2) read in place from host memory
    DevBuf<uint8_t> xhold;
    const void* X = ds.data;
    const size_t xbytes = static_cast<size_t>(N) * d * elem_size(ds.dtype);
    std::unique_ptr<HostRows> xhost;
    if (ds.on_device == 2) {
        xhost = std::make_unique<HostRows>(ds.data, xbytes, st);
        X = xhost->dev;
    } else if (!ds.on_device) {
        xhold = DevBuf<uint8_t>(xbytes, st);
        GTA_CUDA(cudaMemcpyAsync(xhold.get(), ds.data, xbytes, cudaMemcpyHostToDevice, st));
        X = xhold.get();
    }
    const int d32 = pad_dim(d, kElemF32);

    // ---- k-means over a sample
    const int64_t n_s = kmeans_sample_size(N, p.kmeans_sample, B);
    DevBuf<int32_t> sid(static_cast<size_t>(n_s), st);
    sample_ids(N, n_s, p.seed, sid.get(), st);
    DevBuf<float> Xs(static_cast<size_t>(n_s) * d32, st), xs_n(static_cast<size_t>(n_s), st);
    {
        ProfScope prof("sample_gather", static_cast<double>(n_s) * (d * elem_size(ds.dtype) + d32 * 4.0), st);
        convert_rows(X, ds.dtype, d, sid.get(), n_s, Xs.get(), kElemF32, d32, xs_n.get(), st);
    }
    DevBuf<float> C(static_cast<size_t>(B) * d32, st), cn(static_cast<size_t>(B), st);
    if (p.init_centroids) {
        copy_rows_padded(C.get(), d32, p.init_centroids, d, B, p.init_on_device != 0, st);
    } else {
        // the k-means++ pool: its own stratified draw over all N rows
        const int64_t pool_n = kmeans_pool_size(n_s, B);
        ProfScope prof("kmeans_init", 0.0, st);
        DevBuf<int32_t> pid(static_cast<size_t>(pool_n), st);
        sample_ids(N, pool_n, kmeans_pool_seed(p.seed), pid.get(), st);
        DevBuf<float> Xp(static_cast<size_t>(pool_n) * d32, st);
        convert_rows(X, ds.dtype, d, pid.get(), pool_n, Xp.get(), kElemF32, d32, nullptr, st);
        kmeanspp_init(Xp.get(), nullptr, pool_n, d, d32, B, p.seed, C.get(), err.get(), st);
    }
    convert_rows(C.get(), GTA_F32, d32, nullptr, B, nullptr, kElemF32, d32, cn.get(), st);
    {
        ProfScope prof("kmeans_fit_total", 0.0, st);
        RawRows raw;
        if (ds.dtype != GTA_F32) raw = RawRows{X, ds.dtype, d, sid.get()};  // 8-bit rows: a quarter of the f32 reads
        kmeans_fit_impl(Xs.get(), xs_n.get(), n_s, d, d32, C.get(), cn.get(), B, p.kmeans_iters, nullptr, err.get(), st,
                        ds.dtype != GTA_F32, raw);
    }
    Xs.release();
    xs_n.release();
    sid.release();
    if (o.centroids) unpad_rows(o.centroids, d, C.get(), d32, B, true, st);

    // ---- top-2 bucket membership of every point
    DevBuf<int32_t> top2(static_cast<size_t>(N) * 2, st);
    {
        ProfScope prof("top2_total", 0.0, st);
        DevBuf<float> t2d(static_cast<size_t>(N) * 2, st);
        if (assign_exact_applies(B, 2)) {  // straight from the dataset's own element type
            assign_exact(X, ds.dtype, N, d, d, nullptr, C.get(), d32, B, 2, top2.get(), t2d.get(), st);
        } else {  // the f32 copy of the rows in chunks of at most kTop2ChunkBytes
            const int64_t chunk = std::max<int64_t>(128, static_cast<int64_t>(kTop2ChunkBytes / (static_cast<size_t>(d32) * 4)));
            DevBuf<float> Xf(static_cast<size_t>(std::min(N, chunk)) * d32, st), xn(static_cast<size_t>(std::min(N, chunk)), st);
            DevBuf<int32_t> rid(static_cast<size_t>(std::min(N, chunk)), st);
            for (int64_t r0 = 0; r0 < N; r0 += chunk) {
                const int64_t nr = std::min(chunk, N - r0);
                const void* Xr = static_cast<const uint8_t*>(X) + static_cast<size_t>(r0) * d * elem_size(ds.dtype);
                {
                    ProfScope prof("convert_x", static_cast<double>(nr) * (d * elem_size(ds.dtype) + d32 * 4.0), st);
                    convert_rows(Xr, ds.dtype, d, nullptr, nr, Xf.get(), kElemF32, d32, xn.get(), st);
                }
                assign_topk_impl(Xf.get(), xn.get(), nr, d, d32, C.get(), cn.get(), B, 2, top2.get() + 2 * r0,
                                 t2d.get() + 2 * r0, err.get(), st, ds.dtype != GTA_F32);
            }
        }
    }
    if (o.top2) GTA_CUDA(cudaMemcpyAsync(o.top2, top2.get(), sizeof(int32_t) * 2 * N, cudaMemcpyDeviceToDevice, st));
    DevBuf<int32_t> members(static_cast<size_t>(N) * 2, st);
    DevBuf<int64_t> offsets(static_cast<size_t>(B) + 1, st), mem_row(static_cast<size_t>(N) * 2, st);
    // exact data with short lists: lower-bucket rows first, then the higher-bucket rows seeded
    // by them (same lists; see KnnPhase)
    const int elem = knn_elem(ds.dtype, d, M);
    const bool phased = dist_topk_seedable(elem, pad_dim(d, elem), M);
    DevBuf<int64_t> split_d;
    DevBuf<int32_t> partner;
    std::vector<int64_t> split_h;
    if (phased) {
        split_d = DevBuf<int64_t>(static_cast<size_t>(B), st);
        partner = DevBuf<int32_t>(static_cast<size_t>(N) * 2, st);
    }
    build_memberships(top2.get(), N, B, members.get(), offsets.get(), mem_row.get(), err.get(), st, split_d.get(),
                      partner.get());
    top2.release();
    if (phased) {
        split_h.resize(static_cast<size_t>(B));
        GTA_CUDA(cudaMemcpyAsync(split_h.data(), split_d.get(), sizeof(int64_t) * B, cudaMemcpyDeviceToHost, st));
        GTA_CUDA(cudaStreamSynchronize(st));
    }

    // ---- per-bucket all-pairs kNN, then merge each point's two lists.  When the memberships' pool
    // rows and lists do not fit the device budget, buckets are processed in ascending batches that
    // do, each batch's lists merged into the per-point lists as it completes (first memberships
    // copied, second ones merged: the same lists as the one-pass build).
    const int64_t n_mem = 2 * N;
    const double per_row = static_cast<double>(pad_dim(d, elem)) * elem_bytes(elem) + 8.0 * M + 8.0;
    double budget = static_cast<double>(p.device_budget);
    if (budget <= 0.0) {  // the free memory is queried only for stages that may not fit
        int dev = 0;
        GTA_CUDA(cudaGetDevice(&dev));
        size_t total_b = 0;
        {
            std::lock_guard<std::mutex> g(g_devmem_mu);
            auto it = g_devmem_total.find(dev);
            if (it == g_devmem_total.end()) {
                cudaDeviceProp prop{};
                GTA_CUDA(cudaGetDeviceProperties(&prop, dev));
                it = g_devmem_total.emplace(dev, prop.totalGlobalMem).first;
            }
            total_b = it->second;
        }
        budget = 0.25 * static_cast<double>(total_b);
        if (static_cast<double>(n_mem) * per_row > budget) {
            size_t free_b = 0, tot = 0;
            GTA_CUDA(cudaMemGetInfo(&free_b, &tot));
            budget = 0.8 * static_cast<double>(free_b);
        }
    }
    if (static_cast<double>(n_mem) * per_row <= budget) {
        DevBuf<int32_t> lid(static_cast<size_t>(n_mem) * M, st);
        DevBuf<float> ldist(static_cast<size_t>(n_mem) * M, st);
        {
            ProfScope prof("bucket_knn_total", 0.0, st);
            KnnPhase ph;
            if (phased) {
                ph.phase = 3; ph.split = split_h.data(); ph.partner = partner.get();
                ph.mem_row = mem_row.get(); ph.n_points = N;
            }
            bucket_knn_impl(X, ds.dtype, N, d, members.get(), offsets.get(), B, M, lid.get(), ldist.get(), err.get(), st,
                            nullptr, 0, -1, nullptr, ph);
        }
        merge_memberships(lid.get(), ldist.get(), mem_row.get(), N, M, o.ids, o.dists, st);
    } else {
        std::vector<int64_t> off(static_cast<size_t>(B) + 1);
        GTA_CUDA(cudaMemcpyAsync(off.data(), offsets.get(), sizeof(int64_t) * (B + 1), cudaMemcpyDeviceToHost, st));
        GTA_CUDA(cudaStreamSynchronize(st));
        const int64_t cap = std::max<int64_t>(1, static_cast<int64_t>(budget / per_row));
        ProfScope prof("bucket_knn_total", 0.0, st);
        // phased: a sweep over the batches for the lower-bucket rows (copied into the per-point
        // lists), then one for the higher-bucket rows seeded by those lists (merged into them)
        for (int sweep = phased ? 1 : 0; sweep <= (phased ? 2 : 0); ++sweep) {
            KnnPhase ph;
            if (phased) {
                ph.phase = sweep; ph.split = split_h.data(); ph.partner = partner.get();
                ph.seed = o.dists + (M - 1); ph.seed_stride = M;
            }
            for (int b_lo = 0; b_lo < B;) {
                int b_hi = b_lo + 1;  // at least one bucket per batch
                while (b_hi < B && off[b_hi + 1] - off[b_lo] <= cap) ++b_hi;
                const int64_t j0 = off[b_lo], nb = off[b_hi] - j0;
                if (nb > 0) {
                    DevBuf<int32_t> lid(static_cast<size_t>(nb) * M, st);
                    DevBuf<float> ldist(static_cast<size_t>(nb) * M, st);
                    bucket_knn_impl(X, ds.dtype, N, d, members.get(), offsets.get(), B, M, lid.get(), ldist.get(),
                                    err.get(), st, nullptr, b_lo, b_hi, off.data(), ph);
                    merge_membership_batch(lid.get(), ldist.get(), members.get(), mem_row.get(), j0, nb, N, M, o.ids,
                                           o.dists, st, sweep == 0 ? 3 : sweep);
                    GTA_CUDA(cudaStreamSynchronize(st));  // the batch's buffers are released next
                }
                b_lo = b_hi;
            }
        }
    }
    check_device_error(err.get(), st, "build_bucket");
}

// bucket2 -t: rounds with seeds seed, seed+1, ... (bucket.cu:9938-9940); each round's lists merged
// into the running lists with the resident merge rule (running first on equal distance, ids already
// present skipped; bucket.cu:5025-5131).  Centroids / top-2 are those of the last round.
void build_bucket_impl(const gta_dataset& ds, const gta_bucket_params& p, const BucketOut& o, cudaStream_t st)
{
    const int rounds = p.rounds > 1 ? p.rounds : 1;
    GTA_REQUIRE(p.rounds >= 0, kInvalid, "build_bucket: negative rounds");
    if (rounds == 1) {
        build_bucket_round(ds, p, o, st);
        return;
    }
    const int64_t N = ds.n;
    const int M = p.knn_degree;
    GTA_REQUIRE(ds.data && N >= 2 && M >= 1 && M <= 128, kInvalid, "build_bucket: bad dataset or knn_degree");
    gta_dataset dd = ds;
    DevBuf<uint8_t> xhold;
    if (ds.on_device == 0) {  // one upload for all rounds (on_device 2: every round reads the host rows)
        const size_t xbytes = static_cast<size_t>(N) * ds.d * elem_size(ds.dtype);
        xhold = DevBuf<uint8_t>(xbytes, st);
        GTA_CUDA(cudaMemcpyAsync(xhold.get(), ds.data, xbytes, cudaMemcpyHostToDevice, st));
        dd.data = xhold.get();
        dd.on_device = 1;
    }
    const size_t nm = static_cast<size_t>(N) * M;
    DevBuf<int32_t> new_ids(nm, st), run_ids(nm, st);
    DevBuf<float> new_d(nm, st), run_d(nm, st);
    for (int r = 0; r < rounds; ++r) {
        gta_bucket_params pr = p;
        pr.rounds = 1;
        pr.seed = p.seed + static_cast<uint64_t>(r);
        const bool last = r == rounds - 1;
        BucketOut ro{r == 0 ? o.ids : new_ids.get(), r == 0 ? o.dists : new_d.get(), last ? o.centroids : nullptr,
                     last ? o.top2 : nullptr};
        build_bucket_round(dd, pr, ro, st);
        if (r == 0) continue;
        GTA_CUDA(cudaMemcpyAsync(run_ids.get(), o.ids, sizeof(int32_t) * nm, cudaMemcpyDeviceToDevice, st));
        GTA_CUDA(cudaMemcpyAsync(run_d.get(), o.dists, sizeof(float) * nm, cudaMemcpyDeviceToDevice, st));
        merge_lists(run_ids.get(), run_d.get(), new_ids.get(), new_d.get(), N, M, o.ids, o.dists, st);
    }
}

// ---------------------------------------------------------------- reference bucketing (bucket2)
struct Bucket2Out {
    int32_t* ids;        // device [N x M]
    float* dists;        // device [N x M]
    int32_t* assign;     // device [N] or null
    int32_t* cid;        // device [B_req] or null
    int32_t n_buckets;   // set by the round
};

constexpr int kKparRounds = 3;            // bucket.cu:2964 FIXED_NITER
constexpr double kKparOvershoot = 1.5;    // bucket.cu:2965 TOTAL_OVERSHOOT
constexpr size_t kPoolBudgetBytes = size_t(8) << 30;  // gathered pool rows held at once

int64_t bucket2_requested(int64_t N, float ratio)
{
    const double r = ratio > 0.0f ? static_cast<double>(ratio) : 0.01;
    return std::max<int64_t>(2, static_cast<int64_t>(static_cast<double>(N) * r));
}

// The dataset prepared for nearest-centroid queries where centroids are data points: 8-bit rows
// held exactly as bf16 (tensor cores, exact integer distances), other data as padded f32 (tf32
// screen + exact rerank); few centroids (<= 384, k <= 4) take the exact FP32-pipe path.
struct Space {
    const void* X = nullptr;
    int dtype = GTA_F32;
    int64_t N = 0;
    int d = 0;
    bool ex8 = false;
    int elem = kElemF32;
    int d_pad = 0;
    size_t row_bytes = 0;
    DevBuf<uint8_t> rows;
    DevBuf<float> norms;

    Space(const void* X_, int dtype_, int64_t N_, int d_, cudaStream_t st) : X(X_), dtype(dtype_), N(N_), d(d_)
    {
        ex8 = exact_bf16(dtype, d);
        elem = ex8 ? kElemBF16 : kElemF32;
        d_pad = pad_dim(d, elem);
        row_bytes = static_cast<size_t>(d_pad) * (ex8 ? 2 : 4);
        rows = DevBuf<uint8_t>(static_cast<size_t>(N) * row_bytes, st);
        norms = DevBuf<float>(static_cast<size_t>(N), st);
        convert_rows(X, dtype, d, nullptr, N, rows.get(), elem, d_pad, norms.get(), st);
    }
    const void* row(int64_t i) const { return rows.get() + static_cast<size_t>(i) * row_bytes; }

    // top-k of the queries (all N points, or the rows q_ids) among the points c_ids
    void assign(const int32_t* q_ids, int64_t nq, const int32_t* c_ids, int nC, int k, int32_t* ids, float* dists,
                int* err, cudaStream_t st) const
    {
        if (assign_exact_applies(nC, k)) {
            const int d32 = pad_dim(d, kElemF32);
            DevBuf<float> Cf(static_cast<size_t>(nC) * d32, st);
            convert_rows(X, dtype, d, c_ids, nC, Cf.get(), kElemF32, d32, nullptr, st);
            assign_exact(X, dtype, nq, d, d, q_ids, Cf.get(), d32, nC, k, ids, dists, st);
            return;
        }
        DevBuf<uint8_t> Cr(static_cast<size_t>(nC) * row_bytes, st), Qr;
        DevBuf<float> cn(static_cast<size_t>(nC), st), qn;
        convert_rows(X, dtype, d, c_ids, nC, Cr.get(), elem, d_pad, cn.get(), st);
        const void* Q = rows.get();
        const float* qnp = norms.get();
        if (q_ids) {
            Qr = DevBuf<uint8_t>(static_cast<size_t>(nq) * row_bytes, st);
            qn = DevBuf<float>(static_cast<size_t>(nq), st);
            convert_rows(X, dtype, d, q_ids, nq, Qr.get(), elem, d_pad, qn.get(), st);
            Q = Qr.get();
            qnp = qn.get();
        }
        if (ex8)
            assign_topk_bf16(Q, qnp, nq, d, d_pad, Cr.get(), cn.get(), nC, k, ids, dists, err, st);
        else
            assign_topk_impl(static_cast<const float*>(Q), qnp, nq, d, d_pad, reinterpret_cast<const float*>(Cr.get()),
                             cn.get(), nC, k, ids, dists, err, st);
    }
};

// KMeans|| candidates (bucket.cu:2919-3117) and their uniform subsample (:3150-3172) -> point ids
std::vector<int32_t> kmeans_parallel_ids(const Space& sp, int64_t n_req, uint64_t seed, int* err, cudaStream_t st)
{
    const int64_t N = sp.N;
    const int32_t c0 = static_cast<int32_t>(mix64(seed ^ 0xA0761D6478BD642Full) % static_cast<uint64_t>(N));
    std::vector<int32_t> cand{c0};
    DevBuf<uint8_t> chosen(static_cast<size_t>(N), st), sel(static_cast<size_t>(N), st);
    GTA_CUDA(cudaMemsetAsync(chosen.get(), 0, static_cast<size_t>(N), st));
    GTA_CUDA(cudaMemsetAsync(chosen.get() + c0, 1, 1, st));
    DevBuf<float> min_d(static_cast<size_t>(N), st), d_new(static_cast<size_t>(N), st);
    DevBuf<int32_t> tmp_ids(static_cast<size_t>(N), st), new_ids(static_cast<size_t>(N), st), c0d(1, st);
    GTA_CUDA(cudaMemcpyAsync(c0d.get(), &c0, sizeof(int32_t), cudaMemcpyHostToDevice, st));
    DevBuf<double> psi(1, st);
    sp.assign(nullptr, N, c0d.get(), 1, 1, tmp_ids.get(), min_d.get(), err, st);  // distance to the first point
    const double lk = kKparOvershoot / kKparRounds * static_cast<double>(n_req);
    for (int r = 0; r < kKparRounds; ++r) {
        kpar_psi(min_d.get(), N, psi.get(), st);
        kpar_sample(min_d.get(), N, seed, r, lk, psi.get(), chosen.get(), sel.get(), st);
        const int64_t n_new = select_flagged(sel.get(), N, new_ids.get(), st);
        if (n_new == 0) break;
        const size_t old = cand.size();
        cand.resize(old + static_cast<size_t>(n_new));
        GTA_CUDA(cudaMemcpyAsync(cand.data() + old, new_ids.get(), sizeof(int32_t) * n_new, cudaMemcpyDeviceToHost, st));
        if (r + 1 < kKparRounds) {  // distances to the new candidates (not after the last round, :3080)
            sp.assign(nullptr, N, new_ids.get(), static_cast<int>(n_new), 1, tmp_ids.get(), d_new.get(), err, st);
            min_update(min_d.get(), d_new.get(), N, st);
        }
        GTA_CUDA(cudaStreamSynchronize(st));  // cand is read on the host below
    }
    const int64_t n_cand = static_cast<int64_t>(cand.size());
    if (n_cand <= n_req) return cand;
    // partial Fisher-Yates over the candidate positions with a splitmix64 stream
    std::vector<int32_t> perm(static_cast<size_t>(n_cand));
    std::iota(perm.begin(), perm.end(), 0);
    const uint64_t s2 = seed ^ 0x5851F42D4C957F2Dull;
    for (int64_t k = 0; k < n_req; ++k) {
        const int64_t j = k + static_cast<int64_t>(mix64(s2 + static_cast<uint64_t>(k)) %
                                                   static_cast<uint64_t>(n_cand - k));
        std::swap(perm[static_cast<size_t>(k)], perm[static_cast<size_t>(j)]);
    }
    std::vector<int32_t> ids(static_cast<size_t>(n_req));
    for (int64_t k = 0; k < n_req; ++k) ids[static_cast<size_t>(k)] = cand[static_cast<size_t>(perm[static_cast<size_t>(k)])];
    return ids;
}

void build_bucket2_round(const void* X, int dtype, int64_t N, int d, const gta_bucket2_params& p, uint64_t seed,
                         Bucket2Out& o, cudaStream_t st)
{
    const int M = p.knn_degree;
    const int64_t n_req = bucket2_requested(N, p.centroid_ratio);
    GTA_REQUIRE(n_req <= N, kInvalid, "build_bucket2: more buckets than points");
    DevBuf<int> err(1, st);
    GTA_CUDA(cudaMemsetAsync(err.get(), 0, sizeof(int), st));
    ProfScope prof_all("build_bucket2_total", 0.0, st);
    Space sp(X, dtype, N, d, st);

    // ---- Step 2: KMeans|| data-point centroids
    std::vector<int32_t> cid_h;
    {
        ProfScope prof("kmeans_parallel", 0.0, st);
        cid_h = kmeans_parallel_ids(sp, n_req, seed, err.get(), st);
    }
    const int32_t B = static_cast<int32_t>(cid_h.size());
    GTA_REQUIRE(B >= 2, kData, "build_bucket2: KMeans|| found fewer than two centroids");
    auto cid = upload(cid_h, st);

    // ---- Step 3: centroid kNN graph (self excluded): the pools' neighbour buckets
    int P = p.nprobe > 0 ? p.nprobe : (p.knn_k > 0 ? p.knn_k : 32);
    P = std::min<int>(P, B - 1);
    std::vector<int32_t> adj(static_cast<size_t>(B) * std::max(P, 0));
    if (P > 0) {
        ProfScope prof("centroid_knn", 0.0, st);
        DevBuf<int32_t> ki(static_cast<size_t>(B) * (P + 1), st);
        DevBuf<float> kd(static_cast<size_t>(B) * (P + 1), st);
        sp.assign(cid.get(), B, cid.get(), B, P + 1, ki.get(), kd.get(), err.get(), st);
        std::vector<int32_t> h(static_cast<size_t>(B) * (P + 1));
        GTA_CUDA(cudaMemcpyAsync(h.data(), ki.get(), sizeof(int32_t) * h.size(), cudaMemcpyDeviceToHost, st));
        GTA_CUDA(cudaStreamSynchronize(st));
        for (int32_t b = 0; b < B; ++b) {  // drop the bucket itself (else the farthest of the P + 1)
            int w = 0;
            bool dropped = false;
            for (int j = 0; j <= P && w < P; ++j) {
                const int32_t v = h[static_cast<size_t>(b) * (P + 1) + j];
                if (v == b && !dropped) { dropped = true; continue; }
                adj[static_cast<size_t>(b) * P + w++] = v;
            }
        }
    }

    // ---- Step 4: top-2 centroids, balanced 1-way assignment
    DevBuf<int32_t> assign(static_cast<size_t>(N), st);
    {
        ProfScope prof("top2_total", 0.0, st);
        DevBuf<int32_t> top2(static_cast<size_t>(N) * 2, st);
        DevBuf<float> t2d(static_cast<size_t>(N) * 2, st);
        sp.assign(nullptr, N, cid.get(), B, 2, top2.get(), t2d.get(), err.get(), st);
        balanced_assign(top2.get(), t2d.get(), p.assign_rule, cid.get(), B, N, assign.get(), err.get(), st);
    }
    DevBuf<int32_t> members(static_cast<size_t>(N), st);
    DevBuf<int64_t> offsets(static_cast<size_t>(B) + 1, st);
    group_by_key(assign.get(), N, B, members.get(), offsets.get(), err.get(), st);
    check_device_error(err.get(), st, "build_bucket2");  // buckets must be sound before the pools are planned
    std::vector<int64_t> off(static_cast<size_t>(B) + 1);
    GTA_CUDA(cudaMemcpyAsync(off.data(), offsets.get(), sizeof(int64_t) * (B + 1), cudaMemcpyDeviceToHost, st));
    GTA_CUDA(cudaStreamSynchronize(st));

    // ---- Step 6: every bucket's points against its pool (own bucket first, then its P neighbours)
    const int S = P + 1;
    std::vector<int32_t> seg_b(static_cast<size_t>(B) * S);
    std::vector<int64_t> pool_size(static_cast<size_t>(B));
    for (int32_t c = 0; c < B; ++c) {
        int64_t sz = 0;
        for (int j = 0; j < S; ++j) {
            int32_t b = j == 0 ? c : adj[static_cast<size_t>(c) * P + (j - 1)];
            if (b < 0 || b >= B) b = -1;
            seg_b[static_cast<size_t>(c) * S + j] = b;
            if (b >= 0) sz += off[b + 1] - off[b];
        }
        pool_size[static_cast<size_t>(c)] = sz;
    }
    auto seg_b_d = upload(seg_b, st);
    const int elem = knn_elem(dtype, d, M);
    const int d_pad = pad_dim(d, elem);
    const size_t row_bytes = static_cast<size_t>(d_pad) * elem_bytes(elem);
    const int64_t max_pool = *std::max_element(pool_size.begin(), pool_size.end());
    const int64_t cap_rows = std::max<int64_t>(max_pool, static_cast<int64_t>(kPoolBudgetBytes / row_bytes));
    DevBuf<int32_t> lids(static_cast<size_t>(N) * M, st);
    DevBuf<float> ldist(static_cast<size_t>(N) * M, st);
    {
        ProfScope prof("pool_knn_total", 0.0, st);
        for (int32_t c_lo = 0; c_lo < B;) {
            int32_t c_hi = c_lo;
            int64_t rows = 0;
            while (c_hi < B && rows + pool_size[static_cast<size_t>(c_hi)] <= cap_rows) rows += pool_size[static_cast<size_t>(c_hi++)];
            const int32_t nb = c_hi - c_lo;
            std::vector<int64_t> pool_off(static_cast<size_t>(nb)), seg_dst(static_cast<size_t>(nb) * S);
            int64_t run = 0;
            for (int32_t c = c_lo; c < c_hi; ++c) {
                pool_off[static_cast<size_t>(c - c_lo)] = run;
                for (int j = 0; j < S; ++j) {
                    seg_dst[static_cast<size_t>(c - c_lo) * S + j] = run;
                    const int32_t b = seg_b[static_cast<size_t>(c) * S + j];
                    if (b >= 0) run += off[b + 1] - off[b];
                }
            }
            const int64_t n_pool = run;
            const int64_t q0 = off[c_lo], n_q = off[c_hi] - q0;
            if (n_q > 0 && n_pool > 0) {
                auto seg_dst_d = upload(seg_dst, st);
                DevBuf<int32_t> pool_ids(static_cast<size_t>(n_pool), st);
                pool_fill(members.get(), offsets.get(), seg_b_d.get(), seg_dst_d.get(), S, c_lo, nb, pool_ids.get(), st);
                DevBuf<uint8_t> Bp(static_cast<size_t>(n_pool) * row_bytes, st), Ap(static_cast<size_t>(n_q) * row_bytes, st);
                DevBuf<float> bn(static_cast<size_t>(n_pool), st), an(static_cast<size_t>(n_q), st);
                {
                    ProfScope prof("gather", static_cast<double>(n_pool + n_q) * (d * elem_size(dtype) + row_bytes), st);
                    convert_rows(X, dtype, d, pool_ids.get(), n_pool, Bp.get(), elem, d_pad, bn.get(), st);
                    convert_rows(X, dtype, d, members.get() + q0, n_q, Ap.get(), elem, d_pad, an.get(), st);
                }
                // work list: one CTA per 128 query rows of a bucket, largest pools first
                std::vector<int32_t> ord(static_cast<size_t>(nb));
                std::iota(ord.begin(), ord.end(), c_lo);
                std::stable_sort(ord.begin(), ord.end(), [&](int32_t a, int32_t b) {
                    return pool_size[static_cast<size_t>(a)] > pool_size[static_cast<size_t>(b)];
                });
                std::vector<WorkItem> wl;
                double flops = 0.0;
                for (int32_t c : ord) {
                    const int64_t nc = off[c + 1] - off[c];
                    const int64_t ps = pool_size[static_cast<size_t>(c)];
                    flops += 2.0 * static_cast<double>(nc) * static_cast<double>(ps) * d;
                    for (int64_t t = 0; t < nc; t += 128)
                        wl.push_back(WorkItem{static_cast<int32_t>(off[c] - q0 + t),
                                              static_cast<int32_t>(std::min<int64_t>(128, nc - t)),
                                              static_cast<int32_t>(pool_off[static_cast<size_t>(c - c_lo)]),
                                              static_cast<int32_t>(ps), static_cast<int32_t>(t), 0, 0, 0});
                }
                if (!wl.empty()) {
                    auto work = upload(wl, st);
                    DistTopkProblem pr;
                    pr.A = Ap.get(); pr.a_total = n_q; pr.B = Bp.get(); pr.b_total = n_pool; pr.elem = elem; pr.d = d;
                    pr.d_pad = d_pad; pr.a_norm = an.get(); pr.b_norm = bn.get(); pr.b_gid = pool_ids.get();
                    pr.work = work.get(); pr.n_work = static_cast<int>(wl.size()); pr.m_out = M; pr.exclude_self = true;
                    pr.out_ids = lids.get() + q0 * M; pr.out_dists = ldist.get() + q0 * M; pr.err = err.get();
                    pr.prof_name = "dist_topk_pool";
                    pr.flops = flops;
                    dist_topk(pr, st);
                }
                GTA_CUDA(cudaStreamSynchronize(st));  // the batch's buffers are released next
            }
            c_lo = c_hi;
        }
    }
    // per-point lists (one membership each)
    DevBuf<int64_t> mem_row(static_cast<size_t>(N) * 2, st);
    one_way_rows(members.get(), N, mem_row.get(), st);
    merge_memberships(lids.get(), ldist.get(), mem_row.get(), N, M, o.ids, o.dists, st);
    if (o.assign) GTA_CUDA(cudaMemcpyAsync(o.assign, assign.get(), sizeof(int32_t) * N, cudaMemcpyDeviceToDevice, st));
    if (o.cid) GTA_CUDA(cudaMemcpyAsync(o.cid, cid.get(), sizeof(int32_t) * B, cudaMemcpyDeviceToDevice, st));
    o.n_buckets = B;
    check_device_error(err.get(), st, "build_bucket2");
}

void build_bucket2_impl(const gta_dataset& ds, const gta_bucket2_params& p, Bucket2Out& o, cudaStream_t st)
{
    const int64_t N = ds.n;
    const int M = p.knn_degree;
    GTA_REQUIRE(ds.data && N >= 2 && ds.d >= 1 && N < (1ll << 30), kInvalid, "build_bucket2: need 2 <= N < 2^30");
    GTA_REQUIRE(ds.dtype == GTA_F32 || ds.dtype == GTA_U8 || ds.dtype == GTA_I8, kInvalid, "build_bucket2: bad dtype");
    GTA_REQUIRE(M >= 1 && M <= 128, kInvalid, "build_bucket2: knn_degree must be in [1, 128]");
    GTA_REQUIRE(p.nprobe >= 0 && p.nprobe <= 127 && p.knn_k >= 0 && p.knn_k <= 127 && p.rounds >= 0 &&
                    p.centroid_ratio >= 0.0f && p.centroid_ratio <= 1.0f && (p.assign_rule == 0 || p.assign_rule == 1),
                kInvalid, "build_bucket2: need 0 <= nprobe, knn_k <= 127, 0 <= centroid_ratio <= 1, assign_rule 0 or 1");
    GTA_REQUIRE(ds.on_device == 0 || ds.on_device == 1, kInvalid,
                "build_bucket2: the dataset is a host (0) or device (1) pointer");
    const void* X = ds.data;
    DevBuf<uint8_t> xhold;
    if (!ds.on_device) {
        const size_t xbytes = static_cast<size_t>(N) * ds.d * elem_size(ds.dtype);
        xhold = DevBuf<uint8_t>(xbytes, st);
        GTA_CUDA(cudaMemcpyAsync(xhold.get(), ds.data, xbytes, cudaMemcpyHostToDevice, st));
        X = xhold.get();
    }
    const int rounds = p.rounds > 1 ? p.rounds : 1;
    const size_t nm = static_cast<size_t>(N) * M;
    DevBuf<int32_t> new_ids, run_ids;
    DevBuf<float> new_d, run_d;
    if (rounds > 1) {
        new_ids = DevBuf<int32_t>(nm, st); run_ids = DevBuf<int32_t>(nm, st);
        new_d = DevBuf<float>(nm, st); run_d = DevBuf<float>(nm, st);
    }
    for (int r = 0; r < rounds; ++r) {
        const bool last = r == rounds - 1;
        Bucket2Out ro{r == 0 ? o.ids : new_ids.get(), r == 0 ? o.dists : new_d.get(), last ? o.assign : nullptr,
                      last ? o.cid : nullptr, 0};
        build_bucket2_round(X, ds.dtype, N, ds.d, p, p.seed + static_cast<uint64_t>(r), ro, st);
        o.n_buckets = ro.n_buckets;
        if (r == 0) continue;
        GTA_CUDA(cudaMemcpyAsync(run_ids.get(), o.ids, sizeof(int32_t) * nm, cudaMemcpyDeviceToDevice, st));
        GTA_CUDA(cudaMemcpyAsync(run_d.get(), o.dists, sizeof(float) * nm, cudaMemcpyDeviceToDevice, st));
        merge_lists(run_ids.get(), run_d.get(), new_ids.get(), new_d.get(), N, M, o.ids, o.dists, st);
    }
}

void optimize_impl(const uint32_t* knn_dev, int64_t n, int m, int k, uint32_t* graph_dev, cudaStream_t st,
                   const int32_t* order = nullptr)
{
    GTA_REQUIRE(n >= 2 && m >= 2 && m <= 128 && k >= 1 && k <= m, kInvalid, "optimize: need n >= 2, 1 <= K <= M <= 128");
    DevBuf<int> err(1, st);
    GTA_CUDA(cudaMemsetAsync(err.get(), 0, sizeof(int), st));
    DevBuf<uint32_t> pruned(static_cast<size_t>(n) * k, st);
    ProfScope prof_all("optimize_total", 0.0, st);
    prune_detour(knn_dev, n, m, k, order, pruned.get(), err.get(), st);
    reverse_merge(pruned.get(), n, k, graph_dev, err.get(), st);
    check_device_error(err.get(), st, "optimize");
}

// ---------------------------------------------------------------- files
enum { kFileF32 = 0, kFileU8 = 1, kFileI8 = 2 };

int dtype_from_path(const std::string& path)
{
    auto ends = [&](const char* s) {
        const size_t n = std::strlen(s);
        return path.size() >= n && path.compare(path.size() - n, n, s) == 0;
    };
    if (ends(".u8bin")) return GTA_U8;
    if (ends(".i8bin")) return GTA_I8;
    if (ends(".fbin") || ends(".bin")) return GTA_F32;
    throw Error(kInvalid, "unsupported dataset extension: " + path);
}

void read_exact(std::ifstream& in, void* dst, size_t bytes, const std::string& what)
{
    in.read(static_cast<char*>(dst), static_cast<std::streamsize>(bytes));
    GTA_REQUIRE(in.good() || (in.eof() && static_cast<size_t>(in.gcount()) == bytes), kData, "short read: " + what);
}

template <typename HdrN, typename T>
void write_table(const char* path, HdrN n, int32_t m, const T* data)
{
    std::ofstream out(path, std::ios::binary | std::ios::trunc);
    GTA_REQUIRE(out.is_open(), kInvalid, std::string("cannot open for writing: ") + path);
    out.write(reinterpret_cast<const char*>(&n), sizeof(n));
    out.write(reinterpret_cast<const char*>(&m), sizeof(m));
    out.write(reinterpret_cast<const char*>(data), static_cast<std::streamsize>(sizeof(T) * static_cast<size_t>(n) * m));
    GTA_REQUIRE(out.good(), kData, std::string("write failed: ") + path);
}

void read_table_header(const char* path, int64_t* n, int32_t* m)
{
    std::ifstream in(path, std::ios::binary);
    GTA_REQUIRE(in.is_open(), kInvalid, std::string("cannot open: ") + path);
    int64_t nn = 0;
    int32_t mm = 0;
    read_exact(in, &nn, sizeof(nn), path);
    read_exact(in, &mm, sizeof(mm), path);
    GTA_REQUIRE(nn > 0 && mm > 0, kData, std::string("invalid header: ") + path);
    in.seekg(0, std::ios::end);
    const int64_t want = 12 + nn * static_cast<int64_t>(mm) * 4;
    GTA_REQUIRE(static_cast<int64_t>(in.tellg()) >= want, kData, std::string("truncated file: ") + path);
    *n = nn;
    *m = mm;
}

template <typename T>
void read_table(const char* path, T* out)
{
    int64_t n = 0;
    int32_t m = 0;
    read_table_header(path, &n, &m);
    std::ifstream in(path, std::ios::binary);
    in.seekg(12);
    read_exact(in, out, sizeof(T) * static_cast<size_t>(n) * m, path);
}

// ---- bucket-contiguous renumbering: host arrays are staged through device buffers

template <typename T>
const T* stage_in(const T* src, size_t count, bool on_device, DevBuf<T>& hold, cudaStream_t st)
{
    if (on_device || !src) return src;
    hold = DevBuf<T>(count, st);
    GTA_CUDA(cudaMemcpyAsync(hold.get(), src, sizeof(T) * count, cudaMemcpyHostToDevice, st));
    return hold.get();
}

template <typename T>
T* stage_out(T* dst, size_t count, bool on_device, DevBuf<T>& hold, cudaStream_t st)
{
    if (on_device || !dst) return dst;
    hold = DevBuf<T>(count, st);
    return hold.get();
}

template <typename T>
void copy_back(T* dst, const DevBuf<T>& hold, size_t count, bool on_device, cudaStream_t st)
{
    if (on_device || !dst) return;
    GTA_CUDA(cudaMemcpyAsync(dst, hold.get(), sizeof(T) * count, cudaMemcpyDeviceToHost, st));
}


// Parses a NumPy v1/v2/v3 header of a C-order little-endian int64 2-D array; returns the data offset.
int64_t npy_i64_header(std::ifstream& in, const std::string& path, int64_t* n, int32_t* m)
{
    unsigned char magic[8];
    read_exact(in, magic, 8, path);
    GTA_REQUIRE(magic[0] == 0x93 && std::memcmp(magic + 1, "NUMPY", 5) == 0, kData, "not a .npy file: " + path);
    uint32_t hl = 0;
    int64_t pre = 0;
    if (magic[6] == 1) {
        uint16_t h16 = 0;
        read_exact(in, &h16, 2, path);
        hl = h16;
        pre = 10;
    } else {
        read_exact(in, &hl, 4, path);
        pre = 12;
    }
    std::string hdr(hl, ' ');
    read_exact(in, hdr.data(), hl, path);
    GTA_REQUIRE(hdr.find("'<i8'") != std::string::npos, kData, "npy dtype must be little-endian int64: " + path);
    GTA_REQUIRE(hdr.find("'fortran_order': False") != std::string::npos, kData, "npy must be C order: " + path);
    const size_t sp = hdr.find("'shape': (");
    GTA_REQUIRE(sp != std::string::npos, kData, "npy header without shape: " + path);
    long long a = 0, b = 0;
    GTA_REQUIRE(std::sscanf(hdr.c_str() + sp + 10, "%lld, %lld", &a, &b) == 2 && a > 0 && b > 0 && b < (1ll << 31),
                kData, "npy must be a non-empty 2-D array: " + path);
    *n = a;
    *m = static_cast<int32_t>(b);
    return pre + hl;
}

}  // namespace
}  // namespace gta

using namespace gta;

extern "C" {

const char* gta_last_error(void) { return g_err.c_str(); }

int gta_release_workspace(void)
{
    return guard([&] {
        std::lock_guard<std::mutex> g(g_ws_mu);
        GTA_REQUIRE(t_depth == 0, kInvalid, "gta_release_workspace: called inside a library call");
        for (auto& e : g_arenas) {
            if (e.second->base) {
                int cur = 0;
                cudaGetDevice(&cur);
                cudaSetDevice(e.first.first);
                cudaStreamSynchronize(e.first.second);
                cudaFree(e.second->base);
                cudaSetDevice(cur);
            }
            delete e.second;
        }
        g_arenas.clear();
    });
}

int gta_profile_enable(int32_t on)
{
    return guard([&] {
        std::lock_guard<std::mutex> g(g_prof_mu);
        prof_clear();
        g_prof_on = on != 0;
    });
}

long long gta_launch_count(void) { return g_launches.load(); }

int gta_profile_counters(int32_t i, double* out, int32_t n)
{
    return guard([&] {
        std::lock_guard<std::mutex> g(g_prof_mu);
        GTA_REQUIRE(i >= 0 && i < static_cast<int32_t>(g_prof.size()), kInvalid, "gta_profile_counters: index out of range");
        const ProfRecord& r = g_prof[static_cast<size_t>(i)];
        std::vector<unsigned long long> h(static_cast<size_t>(r.n_counters));
        if (r.counters) {
            GTA_CUDA(cudaEventSynchronize(r.stop));
            GTA_CUDA(cudaMemcpy(h.data(), r.counters, sizeof(unsigned long long) * h.size(), cudaMemcpyDeviceToHost));
        }
        for (int32_t k = 0; k < n; ++k) out[k] = k < r.n_counters ? static_cast<double>(h[static_cast<size_t>(k)]) : 0.0;
    });
}

int gta_profile_count(void)
{
    std::lock_guard<std::mutex> g(g_prof_mu);
    return static_cast<int>(g_prof.size());
}

int gta_profile_get(int32_t i, char* name, int32_t name_len, float* ms, double* units)
{
    return guard([&] {
        std::lock_guard<std::mutex> g(g_prof_mu);
        GTA_REQUIRE(i >= 0 && i < static_cast<int32_t>(g_prof.size()), kInvalid, "gta_profile_get: index out of range");
        const ProfRecord& r = g_prof[static_cast<size_t>(i)];
        GTA_CUDA(cudaEventSynchronize(r.stop));
        float t = 0.0f;
        GTA_CUDA(cudaEventElapsedTime(&t, r.start, r.stop));
        if (ms) *ms = t;
        if (units) *units = r.units;
        if (name && name_len > 0) {
            std::strncpy(name, r.name.c_str(), static_cast<size_t>(name_len - 1));
            name[name_len - 1] = 0;
        }
    });
}
const char* gta_version(void) { return "gta-b200 0.1 (sm_100a)"; }

int gta_device_memory(int64_t* free_bytes, int64_t* total_bytes)
{
    return guard([&] {
        GTA_REQUIRE(free_bytes && total_bytes, kInvalid, "gta_device_memory: null argument");
        size_t f = 0, t = 0;
        GTA_CUDA(cudaMemGetInfo(&f, &t));
        *free_bytes = static_cast<int64_t>(f);
        *total_bytes = static_cast<int64_t>(t);
    });
}

int gta_build_bucket(const gta_dataset* ds, const gta_bucket_params* p, int32_t* knn_ids, float* knn_dists, void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(ds && p && knn_ids, kInvalid, "gta_build_bucket: null argument");
        cudaStream_t st = S(stream);
        const int64_t N = ds->n;
        const int M = p->knn_degree;
        const size_t nm = static_cast<size_t>(N) * (M > 0 ? M : 0);
        BucketOut o{};
        DevBuf<int32_t> ids;
        DevBuf<float> dists, cent;
        DevBuf<int32_t> t2;
        if (p->out_on_device) {
            o.ids = knn_ids;
            if (knn_dists) o.dists = knn_dists;
            else { dists = DevBuf<float>(nm, st); o.dists = dists.get(); }
            o.centroids = p->centroids_out;
            o.top2 = p->top2_out;
        } else {
            ids = DevBuf<int32_t>(nm, st);
            dists = DevBuf<float>(nm, st);
            o.ids = ids.get();
            o.dists = dists.get();
            if (p->centroids_out) { cent = DevBuf<float>(static_cast<size_t>(p->n_buckets) * ds->d, st); o.centroids = cent.get(); }
            if (p->top2_out) { t2 = DevBuf<int32_t>(static_cast<size_t>(N) * 2, st); o.top2 = t2.get(); }
        }
        build_bucket_impl(*ds, *p, o, st);
        if (!p->out_on_device) {
            GTA_CUDA(cudaMemcpyAsync(knn_ids, o.ids, sizeof(int32_t) * nm, cudaMemcpyDeviceToHost, st));
            if (knn_dists) GTA_CUDA(cudaMemcpyAsync(knn_dists, o.dists, sizeof(float) * nm, cudaMemcpyDeviceToHost, st));
            if (p->centroids_out)
                GTA_CUDA(cudaMemcpyAsync(p->centroids_out, o.centroids, sizeof(float) * p->n_buckets * ds->d,
                                         cudaMemcpyDeviceToHost, st));
            if (p->top2_out)
                GTA_CUDA(cudaMemcpyAsync(p->top2_out, o.top2, sizeof(int32_t) * 2 * N, cudaMemcpyDeviceToHost, st));
            GTA_CUDA(cudaStreamSynchronize(st));
        }
    });
}

int gta_build_bucket2(const gta_dataset* ds, const gta_bucket2_params* p, int32_t* knn_ids, float* knn_dists,
                      void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(ds && p && knn_ids, kInvalid, "gta_build_bucket2: null argument");
        cudaStream_t st = S(stream);
        const int64_t N = ds->n;
        const size_t nm = static_cast<size_t>(N) * (p->knn_degree > 0 ? p->knn_degree : 0);
        const int64_t n_req = bucket2_requested(N, p->centroid_ratio);
        const bool dev = p->out_on_device != 0;
        DevBuf<int32_t> ih, ah, ch;
        DevBuf<float> dh;
        Bucket2Out o{};
        if (dev) {
            o.ids = knn_ids;
            if (knn_dists) o.dists = knn_dists;
            else { dh = DevBuf<float>(nm, st); o.dists = dh.get(); }
            o.assign = p->assign_out;
            o.cid = p->centroid_ids_out;
        } else {
            ih = DevBuf<int32_t>(nm, st);
            dh = DevBuf<float>(nm, st);
            o.ids = ih.get();
            o.dists = dh.get();
            if (p->assign_out) { ah = DevBuf<int32_t>(static_cast<size_t>(N), st); o.assign = ah.get(); }
            if (p->centroid_ids_out) { ch = DevBuf<int32_t>(static_cast<size_t>(n_req), st); o.cid = ch.get(); }
        }
        build_bucket2_impl(*ds, *p, o, st);
        if (p->n_buckets_out) *p->n_buckets_out = o.n_buckets;
        if (!dev) {
            GTA_CUDA(cudaMemcpyAsync(knn_ids, o.ids, sizeof(int32_t) * nm, cudaMemcpyDeviceToHost, st));
            if (knn_dists) GTA_CUDA(cudaMemcpyAsync(knn_dists, o.dists, sizeof(float) * nm, cudaMemcpyDeviceToHost, st));
            if (p->assign_out)
                GTA_CUDA(cudaMemcpyAsync(p->assign_out, o.assign, sizeof(int32_t) * N, cudaMemcpyDeviceToHost, st));
            if (p->centroid_ids_out)
                GTA_CUDA(cudaMemcpyAsync(p->centroid_ids_out, o.cid, sizeof(int32_t) * o.n_buckets,
                                         cudaMemcpyDeviceToHost, st));
            GTA_CUDA(cudaStreamSynchronize(st));
        }
    });
}

int gta_optimize(const uint32_t* knn, int64_t n, int32_t m, int32_t k, uint32_t* graph, int32_t on_device, void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(knn && graph, kInvalid, "gta_optimize: null argument");
        cudaStream_t st = S(stream);
        if (on_device) {
            optimize_impl(knn, n, m, k, graph, st);
        } else {
            DevBuf<uint32_t> kd(static_cast<size_t>(n) * m, st), gd(static_cast<size_t>(n) * k, st);
            GTA_CUDA(cudaMemcpyAsync(kd.get(), knn, sizeof(uint32_t) * n * m, cudaMemcpyHostToDevice, st));
            optimize_impl(kd.get(), n, m, k, gd.get(), st);
            GTA_CUDA(cudaMemcpyAsync(graph, gd.get(), sizeof(uint32_t) * n * k, cudaMemcpyDeviceToHost, st));
            GTA_CUDA(cudaStreamSynchronize(st));
        }
    });
}

int gta_optimize_knn(const gta_dataset* ds, const int32_t* knn, int64_t n, int32_t m, int32_t k, uint32_t* graph,
                     int32_t on_device, void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(knn && graph && n >= 2 && m >= 2 && m <= 128 && k >= 1 && k <= m && n < (1ll << 31), kInvalid,
                    "gta_optimize_knn: need knn, graph, 2 <= n < 2^31, 1 <= K <= M <= 128");
        GTA_REQUIRE(!ds || (ds->data && ds->n == n && ds->d >= 1 && (ds->on_device == 0 || ds->on_device == 1) &&
                            (ds->on_device != 0) == (on_device != 0) &&
                            (ds->dtype == GTA_F32 || ds->dtype == GTA_U8 || ds->dtype == GTA_I8)),
                    kInvalid, "gta_optimize_knn: dataset must match the graph's N and placement");
        cudaStream_t st = S(stream);
        const size_t nm = static_cast<size_t>(n) * m;
        DevBuf<int32_t> kh;
        const int32_t* kd = knn;
        if (!on_device) {
            kh = DevBuf<int32_t>(nm, st);
            GTA_CUDA(cudaMemcpyAsync(kh.get(), knn, sizeof(int32_t) * nm, cudaMemcpyHostToDevice, st));
            kd = kh.get();
        }
        DevBuf<uint32_t> san(nm, st);
        sanitize(kd, n, m, san.get(), st);
        kh.release();
        if (ds) {  // stable sort of every sanitized row by exact L2 to its point
            const int d = ds->d;
            const int d32 = pad_dim(d, kElemF32);
            const size_t xbytes = static_cast<size_t>(n) * d * elem_size(ds->dtype);
            DevBuf<uint8_t> xh;
            const void* X = ds->data;
            if (!on_device) {
                xh = DevBuf<uint8_t>(xbytes, st);
                GTA_CUDA(cudaMemcpyAsync(xh.get(), ds->data, xbytes, cudaMemcpyHostToDevice, st));
                X = xh.get();
            }
            DevBuf<float> Xp(static_cast<size_t>(n) * d32, st);
            convert_rows(X, ds->dtype, d, nullptr, n, Xp.get(), kElemF32, d32, nullptr, st);
            xh.release();
            DevBuf<int32_t> sorted(nm, st);
            sort_rows_l2(Xp.get(), d, d32, reinterpret_cast<const int32_t*>(san.get()), n, m, sorted.get(), st);
            GTA_CUDA(cudaMemcpyAsync(san.get(), sorted.get(), sizeof(uint32_t) * nm, cudaMemcpyDeviceToDevice, st));
        }
        DevBuf<uint32_t> gd;
        uint32_t* gout = graph;
        if (!on_device) {
            gd = DevBuf<uint32_t>(static_cast<size_t>(n) * k, st);
            gout = gd.get();
        }
        optimize_impl(san.get(), n, m, k, gout, st);
        if (!on_device) {
            GTA_CUDA(cudaMemcpyAsync(graph, gout, sizeof(uint32_t) * n * k, cudaMemcpyDeviceToHost, st));
            GTA_CUDA(cudaStreamSynchronize(st));
        }
    });
}


int gta_bucket_order(const float* centroids, int32_t B, int32_t d, int32_t k, int32_t window, int32_t* order,
                     int32_t* centroid_knn, int32_t on_device, void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(centroids && order && B >= 2 && d >= 1 && k >= 1 && k < B && k <= 127, kInvalid,
                    "gta_bucket_order: need centroids, order, 1 <= k < B, k <= 127");
        cudaStream_t st = S(stream);
        const bool dev = on_device != 0;
        DevBuf<float> ch;
        const float* C = stage_in(centroids, static_cast<size_t>(B) * d, dev, ch, st);
        const int d32 = pad_dim(d, kElemF32);
        DevBuf<int> err(1, st);
        GTA_CUDA(cudaMemsetAsync(err.get(), 0, sizeof(int), st));
        DevBuf<float> Cp(static_cast<size_t>(B) * d32, st), cn(static_cast<size_t>(B), st);
        convert_rows(C, GTA_F32, d, nullptr, B, Cp.get(), kElemF32, d32, cn.get(), st);
        const int k1 = k + 1;
        DevBuf<int32_t> ids(static_cast<size_t>(B) * k1, st);
        DevBuf<float> dd(static_cast<size_t>(B) * k1, st);
        assign_topk_impl(Cp.get(), cn.get(), B, d, d32, Cp.get(), cn.get(), B, k1, ids.get(), dd.get(), err.get(), st);
        check_device_error(err.get(), st, "gta_bucket_order");
        std::vector<int32_t> h(static_cast<size_t>(B) * k1), adj(static_cast<size_t>(B) * k);
        GTA_CUDA(cudaMemcpyAsync(h.data(), ids.get(), sizeof(int32_t) * h.size(), cudaMemcpyDeviceToHost, st));
        GTA_CUDA(cudaStreamSynchronize(st));
        for (int32_t b = 0; b < B; ++b) {  // drop the bucket itself (else the farthest of the k + 1)
            int w = 0;
            bool dropped = false;
            for (int j = 0; j < k1 && w < k; ++j) {
                const int32_t v = h[static_cast<size_t>(b) * k1 + j];
                if (v == b && !dropped) { dropped = true; continue; }
                adj[static_cast<size_t>(b) * k + w++] = v;
            }
        }
        const int32_t win = window > 0 ? window : std::max<int32_t>(4 * k, 16);
        std::vector<int32_t> ord(static_cast<size_t>(B));
        bucket_order(adj.data(), B, k, win, ord.data());
        if (dev) {
            GTA_CUDA(cudaMemcpyAsync(order, ord.data(), sizeof(int32_t) * B, cudaMemcpyHostToDevice, st));
            if (centroid_knn)
                GTA_CUDA(cudaMemcpyAsync(centroid_knn, adj.data(), sizeof(int32_t) * adj.size(), cudaMemcpyHostToDevice, st));
            GTA_CUDA(cudaStreamSynchronize(st));  // the host vectors die here
        } else {
            std::memcpy(order, ord.data(), sizeof(int32_t) * B);
            if (centroid_knn) std::memcpy(centroid_knn, adj.data(), sizeof(int32_t) * adj.size());
        }
    });
}

int gta_bucket_reorder(const int32_t* assign, int64_t n, int32_t stride, int32_t B, const int32_t* order,
                       uint32_t* inverse_perm, int64_t* offsets, int32_t on_device, void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(assign && inverse_perm && n >= 1 && B >= 1 && stride >= 1, kInvalid, "gta_bucket_reorder: bad argument");
        cudaStream_t st = S(stream);
        const bool dev = on_device != 0;
        DevBuf<int32_t> ah, oh;
        DevBuf<uint32_t> ih;
        DevBuf<int64_t> fh;
        const int32_t* a = stage_in(assign, static_cast<size_t>(n) * stride, dev, ah, st);
        const int32_t* o = stage_in(order, static_cast<size_t>(B), dev, oh, st);
        uint32_t* inv = stage_out(inverse_perm, static_cast<size_t>(n), dev, ih, st);
        int64_t* off = stage_out(offsets, static_cast<size_t>(B) + 1, dev, fh, st);
        DevBuf<int> err(1, st);
        GTA_CUDA(cudaMemsetAsync(err.get(), 0, sizeof(int), st));
        bucket_reorder(a, n, stride, B, o, inv, off, err.get(), st);
        copy_back(inverse_perm, ih, static_cast<size_t>(n), dev, st);
        copy_back(offsets, fh, static_cast<size_t>(B) + 1, dev, st);
        check_device_error(err.get(), st, "gta_bucket_reorder");
    });
}

int gta_permute_rows(const void* X, int64_t n, int64_t row_bytes, const uint32_t* inverse_perm, void* out,
                     int32_t on_device, void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(X && inverse_perm && out && n >= 1 && row_bytes >= 1, kInvalid, "gta_permute_rows: bad argument");
        cudaStream_t st = S(stream);
        const bool dev = on_device != 0;
        const size_t bytes = static_cast<size_t>(n) * static_cast<size_t>(row_bytes);
        DevBuf<uint8_t> xh, oh;
        DevBuf<uint32_t> ih;
        const uint8_t* x = stage_in(static_cast<const uint8_t*>(X), bytes, dev, xh, st);
        const uint32_t* inv = stage_in(inverse_perm, static_cast<size_t>(n), dev, ih, st);
        uint8_t* o = stage_out(static_cast<uint8_t*>(out), bytes, dev, oh, st);
        DevBuf<int> err(1, st);
        GTA_CUDA(cudaMemsetAsync(err.get(), 0, sizeof(int), st));
        permute_rows(x, n, row_bytes, inv, o, err.get(), st);
        copy_back(static_cast<uint8_t*>(out), oh, bytes, dev, st);
        check_device_error(err.get(), st, "gta_permute_rows");
    });
}

int gta_permute_graph(const int32_t* g, int64_t n, int32_t m, const uint32_t* inverse_perm, int32_t to_original,
                      int32_t keep_padding, int32_t* out, int32_t on_device, void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(g && inverse_perm && out && n >= 1 && m >= 1, kInvalid, "gta_permute_graph: bad argument");
        cudaStream_t st = S(stream);
        const bool dev = on_device != 0;
        const size_t nm = static_cast<size_t>(n) * m;
        DevBuf<int32_t> gh, oh;
        DevBuf<uint32_t> ih;
        const int32_t* gg = stage_in(g, nm, dev, gh, st);
        const uint32_t* inv = stage_in(inverse_perm, static_cast<size_t>(n), dev, ih, st);
        int32_t* o = stage_out(out, nm, dev, oh, st);
        DevBuf<int> err(1, st);
        GTA_CUDA(cudaMemsetAsync(err.get(), 0, sizeof(int), st));
        permute_graph(gg, n, m, inv, to_original != 0, keep_padding != 0, o, err.get(), st);
        copy_back(out, oh, nm, dev, st);
        check_device_error(err.get(), st, "gta_permute_graph");
    });
}

int gta_build_cagra(const gta_dataset* ds, const gta_cagra_params* p, uint32_t* graph, void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(ds && p && graph, kInvalid, "gta_build_cagra: null argument");
        cudaStream_t st = S(stream);
        const int64_t N = ds->n;
        const int M = p->bucket.knn_degree, K = p->graph_degree;
        GTA_REQUIRE(K >= 1 && K <= M, kInvalid, "gta_build_cagra: need 1 <= graph_degree <= knn_degree");
        DevBuf<int32_t> ids(static_cast<size_t>(N) * M, st), t2;
        DevBuf<float> dists(static_cast<size_t>(N) * M, st), cent;
        BucketOut o{ids.get(), dists.get(), nullptr, nullptr};
        const bool dev = p->bucket.out_on_device != 0;
        if (p->bucket.centroids_out) {
            if (dev) o.centroids = p->bucket.centroids_out;
            else { cent = DevBuf<float>(static_cast<size_t>(p->bucket.n_buckets) * ds->d, st); o.centroids = cent.get(); }
        }
        if (p->bucket.top2_out && dev) o.top2 = p->bucket.top2_out;
        else { t2 = DevBuf<int32_t>(static_cast<size_t>(N) * 2, st); o.top2 = t2.get(); }
        build_bucket_impl(*ds, p->bucket, o, st);
        DevBuf<int32_t> order(static_cast<size_t>(N), st);
        locality_order(o.top2, N, p->bucket.n_buckets, order.get(), st);
        dists.release();
        DevBuf<uint32_t> san(static_cast<size_t>(N) * M, st);
        sanitize(ids.get(), N, M, san.get(), st);
        ids.release();
        DevBuf<uint32_t> gd;
        uint32_t* gout = graph;
        if (!dev) { gd = DevBuf<uint32_t>(static_cast<size_t>(N) * K, st); gout = gd.get(); }
        optimize_impl(san.get(), N, M, K, gout, st, order.get());
        if (!dev) {
            GTA_CUDA(cudaMemcpyAsync(graph, gout, sizeof(uint32_t) * N * K, cudaMemcpyDeviceToHost, st));
            if (p->bucket.centroids_out)
                GTA_CUDA(cudaMemcpyAsync(p->bucket.centroids_out, o.centroids, sizeof(float) * p->bucket.n_buckets * ds->d,
                                         cudaMemcpyDeviceToHost, st));
            if (p->bucket.top2_out)
                GTA_CUDA(cudaMemcpyAsync(p->bucket.top2_out, o.top2, sizeof(int32_t) * 2 * N, cudaMemcpyDeviceToHost, st));
            GTA_CUDA(cudaStreamSynchronize(st));
        }
    });
}

int gta_kmeans_fit(const float* X, int64_t n, int32_t d, float* centroids, int32_t B, int32_t iters,
                   int32_t* assign_out, void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(X && centroids && n >= 1 && d >= 1 && B >= 1 && iters >= 0, kInvalid, "gta_kmeans_fit: bad argument");
        cudaStream_t st = S(stream);
        const int d32 = pad_dim(d, kElemF32);
        DevBuf<int> err(1, st);
        GTA_CUDA(cudaMemsetAsync(err.get(), 0, sizeof(int), st));
        DevBuf<float> Xp(static_cast<size_t>(n) * d32, st), xn(static_cast<size_t>(n), st);
        convert_rows(X, GTA_F32, d, nullptr, n, Xp.get(), kElemF32, d32, xn.get(), st);
        DevBuf<float> C(static_cast<size_t>(B) * d32, st), cn(static_cast<size_t>(B), st);
        copy_rows_padded(C.get(), d32, centroids, d, B, true, st);
        convert_rows(C.get(), GTA_F32, d32, nullptr, B, nullptr, kElemF32, d32, cn.get(), st);
        kmeans_fit_impl(Xp.get(), xn.get(), n, d, d32, C.get(), cn.get(), B, iters, assign_out, err.get(), st);
        unpad_rows(centroids, d, C.get(), d32, B, true, st);
        check_device_error(err.get(), st, "gta_kmeans_fit");
    });
}

int gta_kmeans_init(const float* X, int64_t pool_n, int32_t d, int32_t B, uint64_t seed, float* centroids, void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(X && centroids && pool_n >= 1 && d >= 1 && B >= 1, kInvalid, "gta_kmeans_init: bad argument");
        cudaStream_t st = S(stream);
        const int d32 = pad_dim(d, kElemF32);
        DevBuf<float> Xp(static_cast<size_t>(pool_n) * d32, st), C(static_cast<size_t>(B) * d32, st);
        DevBuf<int> err(1, st);
        GTA_CUDA(cudaMemsetAsync(err.get(), 0, sizeof(int), st));
        convert_rows(X, GTA_F32, d, nullptr, pool_n, Xp.get(), kElemF32, d32, nullptr, st);
        kmeanspp_init(Xp.get(), nullptr, pool_n, d, d32, B, seed, C.get(), err.get(), st);
        unpad_rows(centroids, d, C.get(), d32, B, true, st);
        check_device_error(err.get(), st, "gta_kmeans_init");
    });
}

int gta_assign_topk(const float* X, int64_t n, int32_t d, const float* C, int32_t B, int32_t k, int32_t* ids,
                    float* dists, void* stream)
{
    return gta_assign_topk_ex(X, n, d, C, B, k, ids, dists, 0, stream);
}

int gta_assign_topk_ex(const float* X, int64_t n, int32_t d, const float* C, int32_t B, int32_t k, int32_t* ids,
                       float* dists, int32_t flags, void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(X && C && ids && dists && n >= 1 && d >= 1 && B >= 1 && (flags & ~GTA_ROWS_INTEGER) == 0, kInvalid,
                    "gta_assign_topk: bad argument");
        cudaStream_t st = S(stream);
        const int d32 = pad_dim(d, kElemF32);
        DevBuf<int> err(1, st);
        GTA_CUDA(cudaMemsetAsync(err.get(), 0, sizeof(int), st));
        DevBuf<float> Xp(static_cast<size_t>(n) * d32, st), xn(static_cast<size_t>(n), st);
        DevBuf<float> Cp(static_cast<size_t>(B) * d32, st), cn(static_cast<size_t>(B), st);
        convert_rows(X, GTA_F32, d, nullptr, n, Xp.get(), kElemF32, d32, xn.get(), st);
        convert_rows(C, GTA_F32, d, nullptr, B, Cp.get(), kElemF32, d32, cn.get(), st);
        assign_topk_impl(Xp.get(), xn.get(), n, d, d32, Cp.get(), cn.get(), B, k, ids, dists, err.get(), st,
                         (flags & GTA_ROWS_INTEGER) != 0);
        check_device_error(err.get(), st, "gta_assign_topk");
    });
}

int gta_build_memberships(const int32_t* top2, int64_t n, int32_t B, int32_t* members, int64_t* offsets,
                          int64_t* mem_row, void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(top2 && members && offsets && mem_row && n >= 1 && B >= 2, kInvalid, "gta_build_memberships: bad argument");
        cudaStream_t st = S(stream);
        DevBuf<int> err(1, st);
        GTA_CUDA(cudaMemsetAsync(err.get(), 0, sizeof(int), st));
        build_memberships(top2, n, B, members, offsets, mem_row, err.get(), st);
        check_device_error(err.get(), st, "gta_build_memberships");
    });
}

namespace {
// The membership CSR a stage entry point was given, checked before any kernel reads a row
// through it: the offsets (device, B + 1) copied to the host, non-decreasing from >= 0 and
// covering at most max_entries slots, and the row ids of those slots inside [0, n_rows).
std::vector<int64_t> checked_csr(const int32_t* ids, const int64_t* offsets_dev, int32_t B, int64_t max_entries,
                                 int64_t n_rows, int* err, cudaStream_t st, const char* who)
{
    GTA_REQUIRE(n_rows >= 0 && n_rows < (1ll << 31), kInvalid, std::string(who) + ": row count out of range");
    std::vector<int64_t> off(static_cast<size_t>(B) + 1);
    GTA_CUDA(cudaMemcpyAsync(off.data(), offsets_dev, sizeof(int64_t) * off.size(), cudaMemcpyDeviceToHost, st));
    GTA_CUDA(cudaStreamSynchronize(st));
    GTA_REQUIRE(off[0] >= 0, kData, std::string(who) + ": negative offset");
    for (int32_t b = 0; b < B; ++b)
        GTA_REQUIRE(off[b] <= off[b + 1], kData, std::string(who) + ": offsets must be non-decreasing");
    GTA_REQUIRE(off[B] <= max_entries, kData, std::string(who) + ": offsets cover more slots than the rows allow");
    if (off[B] > off[0]) {
        check_ids(ids + off[0], off[B] - off[0], static_cast<int32_t>(n_rows), err, st);
        check_device_error(err, st, who);
    }
    return off;
}
}  // namespace

int gta_bucket_knn(const void* X, int32_t dtype, int64_t n, int32_t d, const int32_t* members, const int64_t* offsets,
                   int32_t B, int32_t M, int32_t* list_ids, float* list_dists, void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(X && members && offsets && list_ids && list_dists && B >= 1 && M >= 1 && M <= 128, kInvalid,
                    "gta_bucket_knn: bad argument");
        cudaStream_t st = S(stream);
        DevBuf<int> err(1, st);
        GTA_CUDA(cudaMemsetAsync(err.get(), 0, sizeof(int), st));
        // at most two memberships per point (the 2-way CSR of gta_build_memberships)
        const std::vector<int64_t> off = checked_csr(members, offsets, B, 2 * n, n, err.get(), st, "gta_bucket_knn");
        bucket_knn_impl(X, dtype, n, d, members, offsets, B, M, list_ids, list_dists, err.get(), st, nullptr, 0, -1,
                        off.data());
        check_device_error(err.get(), st, "gta_bucket_knn");
    });
}

int gta_merge_memberships(const int32_t* list_ids, const float* list_dists, const int64_t* mem_row, int64_t n,
                          int32_t M, int32_t* out_ids, float* out_dists, void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(list_ids && list_dists && mem_row && out_ids && out_dists, kInvalid, "gta_merge_memberships: null argument");
        merge_memberships(list_ids, list_dists, mem_row, n, M, out_ids, out_dists, S(stream));
    });
}

int gta_merge_lists(const int32_t* run_ids, const float* run_dists, const int32_t* new_ids, const float* new_dists,
                    int64_t n, int32_t M, int32_t* out_ids, float* out_dists, void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(run_ids && run_dists && new_ids && new_dists && out_ids && out_dists, kInvalid,
                    "gta_merge_lists: null argument");
        merge_lists(run_ids, run_dists, new_ids, new_dists, n, M, out_ids, out_dists, S(stream));
    });
}

int gta_sanitize(const int32_t* knn, int64_t n, int32_t m, uint32_t* out, void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(knn && out && n >= 1 && m >= 1, kInvalid, "gta_sanitize: bad argument");
        sanitize(knn, n, m, out, S(stream));
    });
}

int gta_sort_rows(const float* X, int64_t n, int32_t d, const int32_t* knn, int32_t m, int32_t* out, void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(X && knn && out && n >= 1 && d >= 1, kInvalid, "gta_sort_rows: bad argument");
        cudaStream_t st = S(stream);
        const int d32 = pad_dim(d, kElemF32);
        DevBuf<float> Xp(static_cast<size_t>(n) * d32, st);
        convert_rows(X, GTA_F32, d, nullptr, n, Xp.get(), kElemF32, d32, nullptr, st);
        sort_rows_l2(Xp.get(), d, d32, knn, n, m, out, st);
        GTA_CUDA(cudaStreamSynchronize(st));
    });
}

int gta_prune(const uint32_t* knn, int64_t n, int32_t m, int32_t k, uint32_t* pruned, void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(knn && pruned, kInvalid, "gta_prune: null argument");
        cudaStream_t st = S(stream);
        DevBuf<int> err(1, st);
        GTA_CUDA(cudaMemsetAsync(err.get(), 0, sizeof(int), st));
        prune_detour(knn, n, m, k, nullptr, pruned, err.get(), st);
        check_device_error(err.get(), st, "gta_prune");
    });
}

int gta_reverse_merge(const uint32_t* pruned, int64_t n, int32_t k, uint32_t* out, void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(pruned && out && n >= 1, kInvalid, "gta_reverse_merge: bad argument");
        cudaStream_t st = S(stream);
        DevBuf<int> err(1, st);
        GTA_CUDA(cudaMemsetAsync(err.get(), 0, sizeof(int), st));
        reverse_merge(pruned, n, k, out, err.get(), st);
        check_device_error(err.get(), st, "gta_reverse_merge");
    });
}

// Same reverse-edge merge as gta_reverse_merge, for callers that cannot allocate
// device memory at call time; its scratch is a fixed array inside the library.
int gta_reverse_merge_noalloc(const uint32_t* pruned, int64_t n, int32_t k, uint32_t* out, void* stream)
{
    return guard([&] { reverse_merge_noalloc(pruned, n, k, out, static_cast<cudaStream_t>(stream)); });
}

int64_t gta_reverse_merge_noalloc_max_rows(void) { return reverse_merge_noalloc_max_rows(); }
int64_t gta_reverse_merge_noalloc_max_edges(void) { return reverse_merge_noalloc_max_edges(); }

// ---------------------------------------------------------------- graph search
int gta_search(const gta_dataset* base, const void* queries, int64_t nq, const uint32_t* graph, int32_t k_graph,
               const int32_t* entries, int32_t n_entry, int32_t topk, int32_t ef, int32_t* out_ids, float* out_dists,
               void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(base && base->data && queries && graph && entries && out_ids && out_dists && nq >= 0 &&
                        base->n >= 1 && base->d >= 1 && k_graph >= 1 && n_entry >= 1,
                    kInvalid, "gta_search: bad argument");
        GTA_REQUIRE(base->dtype == GTA_F32 || base->dtype == GTA_U8 || base->dtype == GTA_I8, kInvalid,
                    "gta_search: bad dtype");
        GTA_REQUIRE(base->on_device == 0 || base->on_device == 1, kInvalid,
                    "gta_search: the base is a host (0) or device (1) pointer");
        if (nq == 0) return;
        cudaStream_t st = S(stream);
        const int64_t n = base->n;
        const int d = base->d;
        const size_t row = static_cast<size_t>(d) * elem_size(base->dtype);
        const void* B = base->data;
        const void* Q = queries;
        const uint32_t* G = graph;
        const int32_t* E = entries;
        int32_t* oi = out_ids;
        float* od = out_dists;
        DevBuf<uint8_t> hb, hq, hg, he, hoi, hod;
        if (!base->on_device) {  // host inputs: copy them in, results back out
            hb = DevBuf<uint8_t>(row * n, st);
            hq = DevBuf<uint8_t>(row * nq, st);
            hg = DevBuf<uint8_t>(sizeof(uint32_t) * n * k_graph, st);
            he = DevBuf<uint8_t>(sizeof(int32_t) * nq * n_entry, st);
            hoi = DevBuf<uint8_t>(sizeof(int32_t) * nq * topk, st);
            hod = DevBuf<uint8_t>(sizeof(float) * nq * topk, st);
            GTA_CUDA(cudaMemcpyAsync(hb.get(), B, row * n, cudaMemcpyHostToDevice, st));
            GTA_CUDA(cudaMemcpyAsync(hq.get(), Q, row * nq, cudaMemcpyHostToDevice, st));
            GTA_CUDA(cudaMemcpyAsync(hg.get(), G, sizeof(uint32_t) * n * k_graph, cudaMemcpyHostToDevice, st));
            GTA_CUDA(cudaMemcpyAsync(he.get(), E, sizeof(int32_t) * nq * n_entry, cudaMemcpyHostToDevice, st));
            B = hb.get(); Q = hq.get();
            G = reinterpret_cast<const uint32_t*>(hg.get());
            E = reinterpret_cast<const int32_t*>(he.get());
            oi = reinterpret_cast<int32_t*>(hoi.get());
            od = reinterpret_cast<float*>(hod.get());
        }
        DevBuf<int> err(1, st);
        GTA_CUDA(cudaMemsetAsync(err.get(), 0, sizeof(int), st));
        graph_search(B, base->dtype, n, d, G, k_graph, Q, nq, E, n_entry, topk, ef, oi, od, err.get(), st);
        if (!base->on_device) {
            GTA_CUDA(cudaMemcpyAsync(out_ids, oi, sizeof(int32_t) * nq * topk, cudaMemcpyDeviceToHost, st));
            GTA_CUDA(cudaMemcpyAsync(out_dists, od, sizeof(float) * nq * topk, cudaMemcpyDeviceToHost, st));
        }
        check_device_error(err.get(), st, "gta_search");
    });
}

// ---------------------------------------------------------------- shard stages (multi-GPU build)
int gta_kmeans_sizes(int64_t n, const gta_bucket_params* p, int64_t* n_sample, int64_t* pool_n, uint64_t* pool_seed)
{
    return guard([&] {
        GTA_REQUIRE(p && n_sample && pool_n && pool_seed && n >= 2 && p->n_buckets >= 2 && p->n_buckets <= n, kInvalid,
                    "gta_kmeans_sizes: bad argument");
        *n_sample = kmeans_sample_size(n, p->kmeans_sample, p->n_buckets);
        *pool_n = kmeans_pool_size(*n_sample, p->n_buckets);
        *pool_seed = kmeans_pool_seed(p->seed);
    });
}

int gta_sample_ids(int64_t n, int64_t n_s, uint64_t seed, int32_t* ids, void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(ids && n >= 1 && n_s >= 1 && n_s <= n && n < (1ll << 31), kInvalid, "gta_sample_ids: bad argument");
        sample_ids(n, n_s, seed, ids, S(stream));
    });
}

int gta_gather_rows(const void* X, int32_t dtype, int64_t n, int32_t d, int64_t row0, const int32_t* ids,
                    int64_t n_ids, float* out, void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE((X || n == 0) && (ids || n_ids == 0) && (out || n_ids == 0) && d >= 1 && n >= 0 && n_ids >= 0,
                    kInvalid, "gta_gather_rows: bad argument");
        gather_range(X, dtype, d, row0, n, ids, n_ids, out, S(stream));
    });
}

int gta_centroid_sums(const float* X, int64_t n, int32_t d, const int32_t* assign, int32_t B, double* sums,
                      int64_t* counts, void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(sums && counts && d >= 1 && B >= 1 && n >= 0 && (n == 0 || (X && assign)), kInvalid,
                    "gta_centroid_sums: bad argument");
        cudaStream_t st = S(stream);
        if (n == 0) {
            GTA_CUDA(cudaMemsetAsync(sums, 0, sizeof(double) * static_cast<size_t>(B) * d, st));
            GTA_CUDA(cudaMemsetAsync(counts, 0, sizeof(int64_t) * static_cast<size_t>(B), st));
            return;
        }
        DevBuf<int> err(1, st);
        GTA_CUDA(cudaMemsetAsync(err.get(), 0, sizeof(int), st));
        centroid_partial(X, n, d, d, assign, B, sums, reinterpret_cast<long long*>(counts), err.get(), st);
        check_device_error(err.get(), st, "gta_centroid_sums");
    });
}

int gta_centroid_means(const double* sums, const int64_t* counts, int32_t B, int32_t d, float* centroids, void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(sums && counts && centroids && B >= 1 && d >= 1, kInvalid, "gta_centroid_means: bad argument");
        centroid_means(sums, reinterpret_cast<const long long*>(counts), centroids, B, d, centroids, S(stream));
    });
}

int gta_group_memberships(const int32_t* bucket, const int32_t* other, int64_t n, int32_t B, int32_t* order,
                          int64_t* offsets, void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(offsets && B >= 2 && n >= 0 && (n == 0 || (bucket && other && order)), kInvalid,
                    "gta_group_memberships: bad argument");
        cudaStream_t st = S(stream);
        if (n == 0) {
            GTA_CUDA(cudaMemsetAsync(offsets, 0, sizeof(int64_t) * (static_cast<size_t>(B) + 1), st));
            return;
        }
        group_rows(bucket, other, n, B, order, offsets, st);
    });
}

int gta_bucket_knn_rows(const void* R, int32_t dtype, int64_t n, int32_t d, const int32_t* order, const int32_t* gid,
                        const int64_t* offsets, int32_t B, int32_t M, int32_t* list_ids, float* list_dists, void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(offsets && B >= 1 && M >= 1 && M <= 128 && n >= 0 &&
                        (n == 0 || (R && order && gid && list_ids && list_dists)),
                    kInvalid, "gta_bucket_knn_rows: bad argument");
        if (n == 0) return;
        cudaStream_t st = S(stream);
        DevBuf<int> err(1, st);
        GTA_CUDA(cudaMemsetAsync(err.get(), 0, sizeof(int), st));
        // order: each received row once, grouped by bucket
        const std::vector<int64_t> off = checked_csr(order, offsets, B, n, n, err.get(), st, "gta_bucket_knn_rows");
        DevBuf<int32_t> gid_sorted(static_cast<size_t>(n), st);
        gather_i32(gid, order, n, gid_sorted.get(), st);
        bucket_knn_impl(R, dtype, n, d, order, offsets, B, M, list_ids, list_dists, err.get(), st, gid_sorted.get(), 0,
                        -1, off.data());
        check_device_error(err.get(), st, "gta_bucket_knn_rows");
    });
}

namespace {
void bucket_knn_rows_seeded(const void* R, int32_t dtype, int64_t n, int32_t d, const int32_t* order, const int32_t* gid,
                            const int64_t* offsets, const int32_t* partner, int32_t B, int32_t M, int32_t phase,
                            const float* seed, const int64_t* row_lo, const int64_t* row_hi, int32_t* list_ids,
                            float* list_dists, cudaStream_t st, const char* who)
{
    GTA_REQUIRE(offsets && B >= 1 && M >= 1 && M <= 128 && n >= 0 && (phase == 1 || phase == 2) &&
                    (n == 0 || (R && order && gid && partner && list_ids && list_dists)) &&
                    (phase == 1 || n == 0 || seed) && (row_lo == nullptr) == (row_hi == nullptr),
                kInvalid, std::string(who) + ": bad argument");
    if (n == 0) return;
    DevBuf<int> err(1, st);
    GTA_CUDA(cudaMemsetAsync(err.get(), 0, sizeof(int), st));
    // order: each received row once, grouped by bucket
    const std::vector<int64_t> off = checked_csr(order, offsets, B, n, n, err.get(), st, who);
    if (row_lo) {
        for (int b = 0; b < B; ++b)
            GTA_REQUIRE(0 <= row_lo[b] && row_lo[b] <= row_hi[b] && row_hi[b] <= off[b + 1] - off[b], kInvalid,
                        std::string(who) + ": row range outside its bucket");
    }
    const int elem = knn_elem(dtype, d, M);
    const bool seedable = dist_topk_seedable(elem, pad_dim(d, elem), M);
    if (!seedable && phase == 2) return;  // phase 1 wrote every row
    DevBuf<int32_t> gid_sorted(static_cast<size_t>(n), st);
    gather_i32(gid, order, n, gid_sorted.get(), st);
    KnnPhase ph;
    std::vector<int64_t> split_h;
    if (seedable) {
        DevBuf<int64_t> split_d(static_cast<size_t>(B), st);
        split_from_partner(partner, offsets, B, split_d.get(), st);
        split_h.resize(static_cast<size_t>(B));
        GTA_CUDA(cudaMemcpyAsync(split_h.data(), split_d.get(), sizeof(int64_t) * B, cudaMemcpyDeviceToHost, st));
        GTA_CUDA(cudaStreamSynchronize(st));
        ph.phase = phase; ph.split = split_h.data(); ph.partner = partner; ph.seed = seed; ph.seed_stride = 1;
    }
    ph.row_lo = row_lo;
    ph.row_hi = row_hi;
    bucket_knn_impl(R, dtype, n, d, order, offsets, B, M, list_ids, list_dists, err.get(), st, gid_sorted.get(), 0, -1,
                    off.data(), ph);
    check_device_error(err.get(), st, who);
}
}  // namespace

int gta_bucket_knn_rows_phased(const void* R, int32_t dtype, int64_t n, int32_t d, const int32_t* order,
                               const int32_t* gid, const int64_t* offsets, const int32_t* partner, int32_t B, int32_t M,
                               int32_t phase, const float* seed, int32_t* list_ids, float* list_dists, void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        bucket_knn_rows_seeded(R, dtype, n, d, order, gid, offsets, partner, B, M, phase, seed, nullptr, nullptr,
                               list_ids, list_dists, S(stream), "gta_bucket_knn_rows_phased");
    });
}

int gta_bucket_knn_rows_ranged(const void* R, int32_t dtype, int64_t n, int32_t d, const int32_t* order,
                               const int32_t* gid, const int64_t* offsets, const int32_t* partner, int32_t B, int32_t M,
                               int32_t phase, const float* seed, const int64_t* row_lo, const int64_t* row_hi,
                               int32_t* list_ids, float* list_dists, void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(row_lo && row_hi, kInvalid, "gta_bucket_knn_rows_ranged: null row range");
        bucket_knn_rows_seeded(R, dtype, n, d, order, gid, offsets, partner, B, M, phase, seed, row_lo, row_hi,
                               list_ids, list_dists, S(stream), "gta_bucket_knn_rows_ranged");
    });
}

int gta_shard_pack_memberships(const void* X, int32_t dtype, int64_t n_local, int32_t d, int64_t row0,
                               const int32_t* top2, int32_t B, const uint64_t* holders, int32_t world,
                               int64_t* send_counts, void* send_rows, int32_t* send_meta, int64_t capacity,
                               void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(send_counts && holders && B >= 1 && world >= 1 && world <= 64 && n_local >= 0 && d >= 1 &&
                        row0 >= 0 && (n_local == 0 || (X && top2)) && (send_rows == nullptr) == (send_meta == nullptr),
                    kInvalid, "gta_shard_pack_memberships: bad argument");
        GTA_REQUIRE(dtype == GTA_F32 || dtype == GTA_U8 || dtype == GTA_I8, kInvalid,
                    "gta_shard_pack_memberships: bad dtype");
        cudaStream_t st = S(stream);
        DevBuf<int> err(1, st);
        GTA_CUDA(cudaMemsetAsync(err.get(), 0, sizeof(int), st));
        ShardPackMem a{X, n_local, static_cast<int64_t>(d) * elem_size(dtype), row0, top2, B, world, holders,
                       send_rows, send_meta, capacity, err.get()};
        std::vector<int64_t> counts;
        shard_pack_memberships(a, counts, st);
        check_device_error(err.get(), st, "gta_shard_pack_memberships");
        std::copy(counts.begin(), counts.end(), send_counts);
    });
}

int gta_shard_pack_lists(const int32_t* list_ids, const float* list_dists, int64_t n, int32_t M, const int32_t* order,
                         const int32_t* gid, const int64_t* offsets, int32_t B, const int64_t* row_lo,
                         const int64_t* row_hi, const int64_t* starts, int32_t world, int64_t* send_counts,
                         int32_t* send_ids, float* send_dists, int32_t* send_meta, int64_t capacity, void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(send_counts && offsets && row_lo && row_hi && starts && B >= 1 && M >= 1 && world >= 1 &&
                        world <= 64 && n >= 0 && (n == 0 || (list_ids && list_dists && order && gid)) &&
                        (send_ids == nullptr) == (send_dists == nullptr) &&
                        (send_ids == nullptr) == (send_meta == nullptr),
                    kInvalid, "gta_shard_pack_lists: bad argument");
        for (int r = 0; r < world; ++r)
            GTA_REQUIRE(starts[r] <= starts[r + 1], kInvalid, "gta_shard_pack_lists: row ranges out of order");
        cudaStream_t st = S(stream);
        DevBuf<int> err(1, st);
        GTA_CUDA(cudaMemsetAsync(err.get(), 0, sizeof(int), st));
        ShardPackLists a{list_ids, list_dists, n, M, order, gid, offsets, B, world, row_lo, row_hi, starts,
                         send_ids, send_dists, send_meta, capacity, err.get()};
        std::vector<int64_t> counts;
        shard_pack_lists(a, counts, st);
        check_device_error(err.get(), st, "gta_shard_pack_lists");
        std::copy(counts.begin(), counts.end(), send_counts);
    });
}

int gta_shard_member_rows(const int32_t* meta, int64_t n, int64_t row0, int64_t n_local, const int32_t* top2,
                          int64_t* mem_row, void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(n >= 0 && n_local >= 0 && row0 >= 0 && (n == 0 || meta) && (n_local == 0 || (top2 && mem_row)),
                    kInvalid, "gta_shard_member_rows: bad argument");
        cudaStream_t st = S(stream);
        if (n_local == 0) {
            GTA_REQUIRE(n == 0, kData, "gta_shard_member_rows: lists for a rank without rows");
            return;
        }
        DevBuf<int> err(1, st);
        GTA_CUDA(cudaMemsetAsync(err.get(), 0, sizeof(int), st));
        shard_member_rows(meta, n, row0, n_local, top2, mem_row, err.get(), st);
        check_device_error(err.get(), st, "gta_shard_member_rows");
    });
}

int gta_shard_lower_seeds(const float* list_dists, int32_t M, int64_t n, const int32_t* order, const int32_t* gid,
                          const int64_t* offsets, const int32_t* partner, int32_t B, const int64_t* row_lo,
                          const int64_t* row_hi, int64_t N, float* seed, void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(offsets && row_lo && row_hi && B >= 1 && M >= 1 && n >= 0 && N >= 0 && (N == 0 || seed) &&
                        (n == 0 || (list_dists && order && gid && partner)),
                    kInvalid, "gta_shard_lower_seeds: bad argument");
        cudaStream_t st = S(stream);
        DevBuf<int> err(1, st);
        GTA_CUDA(cudaMemsetAsync(err.get(), 0, sizeof(int), st));
        shard_lower_seeds(list_dists, M, n, order, gid, offsets, partner, B, row_lo, row_hi, N, seed, err.get(), st);
        check_device_error(err.get(), st, "gta_shard_lower_seeds");
    });
}

int gta_sanitize_rows(const int32_t* knn, int64_t n_rows, int64_t row0, int64_t n, int32_t m, uint32_t* out,
                      void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(m >= 1 && n >= 1 && row0 >= 0 && n_rows >= 0 && row0 + n_rows <= n &&
                        (n_rows == 0 || (knn && out)),
                    kInvalid, "gta_sanitize_rows: bad argument");
        if (n_rows == 0) return;
        sanitize_rows(knn, n_rows, row0, n, m, out, S(stream));
    });
}

int gta_prune_rows(const uint32_t* knn, int64_t n, int32_t m, int32_t k, int64_t row0, int64_t n_rows,
                   const int32_t* top2, int32_t B, uint32_t* pruned, void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(knn && (pruned || n_rows == 0) && (!top2 || B >= 2), kInvalid, "gta_prune_rows: bad argument");
        if (n_rows == 0) return;
        cudaStream_t st = S(stream);
        DevBuf<int> err(1, st);
        GTA_CUDA(cudaMemsetAsync(err.get(), 0, sizeof(int), st));
        DevBuf<int32_t> order;
        if (top2) {
            order = DevBuf<int32_t>(static_cast<size_t>(n_rows), st);
            locality_order(top2, n_rows, B, order.get(), st);
        }
        prune_rows(knn, n, m, k, order.get(), row0, n_rows, pruned, err.get(), st);
        check_device_error(err.get(), st, "gta_prune_rows");
    });
}

int gta_reverse_merge_rows(const uint32_t* pruned, int64_t n, int32_t k, int64_t row0, int64_t n_rows, uint32_t* out,
                           void* stream)
{
    return guard([&] {
        GTA_WORKSPACE(stream);
        GTA_REQUIRE(pruned && n >= 1 && (out || n_rows == 0), kInvalid, "gta_reverse_merge_rows: bad argument");
        if (n_rows == 0) return;
        cudaStream_t st = S(stream);
        DevBuf<int> err(1, st);
        GTA_CUDA(cudaMemsetAsync(err.get(), 0, sizeof(int), st));
        reverse_merge_rows(pruned, n, k, row0, n_rows, out, err.get(), st);
        check_device_error(err.get(), st, "gta_reverse_merge_rows");
    });
}

// ---------------------------------------------------------------- files
int gta_read_dataset_header(const char* path, int64_t* n, int32_t* d, int32_t* dtype)
{
    return guard([&] {
        GTA_REQUIRE(path && n && d && dtype, kInvalid, "gta_read_dataset_header: null argument");
        const int dt = dtype_from_path(path);
        std::ifstream in(path, std::ios::binary);
        GTA_REQUIRE(in.is_open(), kInvalid, std::string("cannot open: ") + path);
        int32_t hdr[2] = {0, 0};
        read_exact(in, hdr, sizeof(hdr), path);
        GTA_REQUIRE(hdr[0] > 0 && hdr[1] > 0, kData, std::string("invalid BIGANN header (N<=0 or D<=0): ") + path);
        in.seekg(0, std::ios::end);
        const int64_t want = 8 + static_cast<int64_t>(hdr[0]) * hdr[1] * elem_size(dt);
        GTA_REQUIRE(static_cast<int64_t>(in.tellg()) >= want, kData, std::string("truncated dataset: ") + path);
        *n = hdr[0];
        *d = hdr[1];
        *dtype = dt;
    });
}

int gta_read_dataset(const char* path, int64_t row0, int64_t nrows, void* out)
{
    return guard([&] {
        int64_t n = 0;
        int32_t d = 0, dt = 0;
        const int rc = gta_read_dataset_header(path, &n, &d, &dt);
        if (rc != kOk) throw Error(rc, g_err);
        GTA_REQUIRE(out && row0 >= 0 && nrows >= 0 && row0 + nrows <= n, kInvalid, "gta_read_dataset: row range out of bounds");
        std::ifstream in(path, std::ios::binary);
        const size_t row_bytes = static_cast<size_t>(d) * elem_size(dt);
        in.seekg(static_cast<std::streamoff>(8 + row0 * static_cast<int64_t>(row_bytes)));
        read_exact(in, out, row_bytes * static_cast<size_t>(nrows), path);
    });
}

int gta_write_dataset(const char* path, const void* data, int64_t n, int32_t d, int32_t dtype)
{
    return guard([&] {
        GTA_REQUIRE(path && data && n > 0 && n < (1ll << 31) && d > 0, kInvalid, "gta_write_dataset: bad argument");
        std::ofstream out(path, std::ios::binary | std::ios::trunc);
        GTA_REQUIRE(out.is_open(), kInvalid, std::string("cannot open for writing: ") + path);
        const int32_t hdr[2] = {static_cast<int32_t>(n), d};
        out.write(reinterpret_cast<const char*>(hdr), sizeof(hdr));
        out.write(static_cast<const char*>(data), static_cast<std::streamsize>(static_cast<size_t>(n) * d * elem_size(dtype)));
        GTA_REQUIRE(out.good(), kData, std::string("write failed: ") + path);
    });
}

int gta_write_knn(const char* path, const int32_t* ids, int64_t n, int32_t m)
{
    return guard([&] { write_table<int64_t, int32_t>(path, n, m, ids); });
}
int gta_write_knn_dists(const char* path, const float* dists, int64_t n, int32_t m)
{
    return guard([&] { write_table<int64_t, float>(path, n, m, dists); });
}
int gta_read_knn_header(const char* path, int64_t* n, int32_t* m)
{
    return guard([&] { read_table_header(path, n, m); });
}
int gta_read_knn(const char* path, int32_t* ids) { return guard([&] { read_table<int32_t>(path, ids); }); }
int gta_write_graph(const char* path, const uint32_t* graph, int64_t n, int32_t k)
{
    return guard([&] { write_table<int64_t, uint32_t>(path, n, k, graph); });
}
int gta_read_graph_header(const char* path, int64_t* n, int32_t* k)
{
    return guard([&] { read_table_header(path, n, k); });
}
int gta_read_graph(const char* path, uint32_t* graph) { return guard([&] { read_table<uint32_t>(path, graph); }); }

int gta_write_u32(const char* path, const uint32_t* v, int64_t n)
{
    return guard([&] {
        GTA_REQUIRE(path && (v || n == 0) && n >= 0, kInvalid, "gta_write_u32: bad argument");
        std::ofstream out(path, std::ios::binary | std::ios::trunc);
        GTA_REQUIRE(out.is_open(), kInvalid, std::string("cannot open for writing: ") + path);
        out.write(reinterpret_cast<const char*>(v), static_cast<std::streamsize>(sizeof(uint32_t) * n));
        GTA_REQUIRE(out.good(), kData, std::string("write failed: ") + path);
    });
}

int gta_read_u32_count(const char* path, int64_t* n)
{
    return guard([&] {
        GTA_REQUIRE(path && n, kInvalid, "gta_read_u32_count: bad argument");
        std::ifstream in(path, std::ios::binary | std::ios::ate);
        GTA_REQUIRE(in.is_open(), kInvalid, std::string("cannot open: ") + path);
        const int64_t bytes = static_cast<int64_t>(in.tellg());
        GTA_REQUIRE(bytes % 4 == 0, kData, std::string("size is not a multiple of 4 bytes: ") + path);
        *n = bytes / 4;
    });
}

int gta_read_u32(const char* path, uint32_t* v)
{
    return guard([&] {
        GTA_REQUIRE(path && v, kInvalid, "gta_read_u32: bad argument");
        std::ifstream in(path, std::ios::binary | std::ios::ate);
        GTA_REQUIRE(in.is_open(), kInvalid, std::string("cannot open: ") + path);
        const int64_t bytes = static_cast<int64_t>(in.tellg());
        in.seekg(0);
        read_exact(in, v, static_cast<size_t>(bytes), path);
    });
}


int gta_read_npy_i64_header(const char* path, int64_t* n, int32_t* m)
{
    return guard([&] {
        GTA_REQUIRE(path && n && m, kInvalid, "gta_read_npy_i64_header: bad argument");
        std::ifstream in(path, std::ios::binary);
        GTA_REQUIRE(in.is_open(), kInvalid, std::string("cannot open: ") + path);
        npy_i64_header(in, path, n, m);
    });
}

int gta_read_npy_i64(const char* path, int32_t* ids)
{
    return guard([&] {
        GTA_REQUIRE(path && ids, kInvalid, "gta_read_npy_i64: bad argument");
        std::ifstream in(path, std::ios::binary);
        GTA_REQUIRE(in.is_open(), kInvalid, std::string("cannot open: ") + path);
        int64_t n = 0;
        int32_t m = 0;
        npy_i64_header(in, path, &n, &m);
        std::vector<int64_t> row(static_cast<size_t>(m));
        for (int64_t i = 0; i < n; ++i) {
            read_exact(in, row.data(), sizeof(int64_t) * m, path);
            for (int32_t j = 0; j < m; ++j) {
                const int64_t v = row[static_cast<size_t>(j)];
                GTA_REQUIRE(v >= -1 && v < (1ll << 31), kData, "npy value outside [-1, 2^31): " + std::string(path));
                ids[i * m + j] = static_cast<int32_t>(v);
            }
        }
    });
}

int gta_write_npy_i64(const char* path, const int32_t* ids, int64_t n, int32_t m)
{
    return guard([&] {
        GTA_REQUIRE(path && ids && n > 0 && m > 0, kInvalid, "gta_write_npy_i64: bad argument");
        std::string hdr = "{'descr': '<i8', 'fortran_order': False, 'shape': (" + std::to_string(n) + ", " +
                          std::to_string(m) + "), }";
        const size_t pre = 10;
        size_t total = pre + hdr.size() + 1;
        hdr.append((64 - total % 64) % 64, ' ');
        hdr.push_back('\n');
        std::ofstream out(path, std::ios::binary | std::ios::trunc);
        GTA_REQUIRE(out.is_open(), kInvalid, std::string("cannot open for writing: ") + path);
        const unsigned char magic[8] = {0x93, 'N', 'U', 'M', 'P', 'Y', 1, 0};
        out.write(reinterpret_cast<const char*>(magic), 8);
        const uint16_t hl = static_cast<uint16_t>(hdr.size());
        out.write(reinterpret_cast<const char*>(&hl), 2);
        out.write(hdr.data(), static_cast<std::streamsize>(hdr.size()));
        std::vector<int64_t> row(static_cast<size_t>(m));
        for (int64_t i = 0; i < n; ++i) {
            for (int32_t j = 0; j < m; ++j) row[static_cast<size_t>(j)] = ids[i * m + j];
            out.write(reinterpret_cast<const char*>(row.data()), static_cast<std::streamsize>(sizeof(int64_t) * m));
        }
        GTA_REQUIRE(out.good(), kData, std::string("write failed: ") + path);
    });
}

}  // extern "C"
