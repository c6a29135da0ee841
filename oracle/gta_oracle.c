/*
 * gta_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the reference's bucketed kNN-graph + CAGRA prune path
 * (loulankxh/GPU-talored-ANN).  It is the parity checker for the CUDA
 * library: only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline
 * leg load it.  The product library (libgta.so) never links, loads or calls
 * anything in this directory.
 *
 * Parity is pinned (tests/test_oracle_golden.py) against
 *   - the reference's own header-only C++ code (prune_windowed_core.hpp,
 *     edge_chunk_accumulator.hpp) compiled by oracle/Makefile into
 *     oracle/_ref/, through fixtures committed under tests/golden/;
 *   - the reference's Python functions (build_bucket.py, build_knn.py),
 *     through fixtures made by tests/golden/make_golden.py;
 *   - the known-answer cases of the reference's unit tests
 *     (tests/test_prune_windowed_core.cpp, tests/test_edge_chunk_accumulator.cpp).
 *
 * Every function names the reference file:line it restates (paths relative
 * to the reference project root).
 *
 * Distance convention shared with the CUDA library: the "exact" squared L2
 * distance of two rows is the fp32 chain acc = fmaf(a[i]-b[i], a[i]-b[i], acc)
 * over ascending dimensions (the reference's exact-rerank arithmetic,
 * bucketDemo/buildBucket/src/bucket.cu:4350-4363 s6_dot_rows uses the same
 * ascending-dimension fmaf order).  For 8-bit data every step is an integer
 * below 2^24, so the value is exact.  Lists are ordered by (distance, id).
 * Build with -ffp-contract=off so the compiler adds no other fused ops.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------ */
/* distances                                                          */
/* ------------------------------------------------------------------ */

static inline float exact_l2(const float* a, const float* b, int d)
{
    float acc = 0.0f;
    for (int i = 0; i < d; ++i) {
        float t = a[i] - b[i];
        acc = fmaf(t, t, acc);
    }
    return acc;
}

ORC_API float orc_exact_l2(const float* a, const float* b, int d) { return exact_l2(a, b, d); }

/* exact distances of n (row, row) pairs of X (n x d): out[i] = exact_l2(X[a[i]], X[b[i]]) */
ORC_API void orc_pair_l2(const float* X, int32_t d, const int32_t* a, const int32_t* b, int64_t n, float* out)
{
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) out[i] = exact_l2(X + (int64_t)a[i] * d, X + (int64_t)b[i] * d, d);
}

typedef struct { float d; int32_t id; } orc_pair;

static int pair_less(orc_pair x, orc_pair y) { return x.d < y.d || (x.d == y.d && x.id < y.id); }

static int pair_cmp(const void* pa, const void* pb)
{
    orc_pair a = *(const orc_pair*)pa, b = *(const orc_pair*)pb;
    if (pair_less(a, b)) return -1;
    if (pair_less(b, a)) return 1;
    return 0;
}

/* keep the k smallest (d,id) pairs of p[0..n) in out[0..k), ascending, pad (inf,-1) */
static void select_topk(orc_pair* p, int64_t n, int k, int32_t* out_id, float* out_d)
{
    qsort(p, (size_t)n, sizeof(orc_pair), pair_cmp);
    for (int j = 0; j < k; ++j) {
        if (j < n) { out_id[j] = p[j].id; out_d[j] = p[j].d; }
        else { out_id[j] = -1; out_d[j] = INFINITY; }
    }
}

/* ------------------------------------------------------------------ */
/* a2: top-k nearest centroids                                        */
/* bucketDemo/build_bucket.py:96-159 topk_from_A_to_B(X, C, topk);    */
/* ties -> smaller centroid id as bucketDemo/buildBucket/src/         */
/* bucket.cu:1225-1228 step4_less.                                    */
/* ------------------------------------------------------------------ */
ORC_API void orc_topk_assign(const float* X, int64_t N, int d, const float* C, int32_t B, int32_t k,
                             int32_t* out_id, float* out_d)
{
    #pragma omp parallel
    {
        orc_pair* p = (orc_pair*)malloc(sizeof(orc_pair) * (size_t)B);
        #pragma omp for schedule(dynamic, 64)
        for (int64_t i = 0; i < N; ++i) {
            const float* x = X + i * (int64_t)d;
            for (int32_t c = 0; c < B; ++c) { p[c].d = exact_l2(x, C + (int64_t)c * d, d); p[c].id = c; }
            select_topk(p, B, k, out_id + i * k, out_d + i * k);
        }
        free(p);
    }
}

/* ------------------------------------------------------------------ */
/* a1: Lloyd centroid update                                          */
/* bucketDemo/build_bucket.py:255-261 (refine_centers_kmeans):        */
/* mean of assigned rows, empty centroid keeps its old value.  The    */
/* sums are accumulated in fp64 in ascending point order (the CUDA    */
/* library's deterministic segmented sum uses the same order).        */
/* ------------------------------------------------------------------ */
ORC_API void orc_lloyd_update(const float* X, int64_t N, int d, const int32_t* assign, const float* C_in,
                              int32_t B, float* C_out)
{
    double* sums = (double*)calloc((size_t)B * d, sizeof(double));
    int64_t* cnt = (int64_t*)calloc((size_t)B, sizeof(int64_t));
    for (int64_t i = 0; i < N; ++i) {
        int32_t a = assign[i];
        if (a < 0 || a >= B) continue;
        cnt[a]++;
        const float* x = X + i * (int64_t)d;
        double* s = sums + (int64_t)a * d;
        for (int j = 0; j < d; ++j) s[j] += (double)x[j];
    }
    for (int32_t b = 0; b < B; ++b) {
        for (int j = 0; j < d; ++j) {
            int64_t o = (int64_t)b * d + j;
            C_out[o] = cnt[b] > 0 ? (float)(sums[o] / (double)cnt[b]) : C_in[o];
        }
    }
    free(sums);
    free(cnt);
}

/* ------------------------------------------------------------------ */
/* a4/a5/a6: per-bucket all-pairs kNN                                 */
/* bucketDemo/build_bucket.py:602-628 (topk_from_A_to_B(Qa, pool,     */
/* m+1) then the per-row self filter) with the bucket's own members   */
/* as the pool (2-way membership), exact fp32 distances, top-M by     */
/* (distance, id), pad -1 / +inf (bucket.cu:5013-5019).               */
/* members: CSR over buckets, offsets[B+1]; output row j belongs to   */
/* membership j (the j-th entry of members).                          */
/* ------------------------------------------------------------------ */
ORC_API void orc_bucket_knn(const float* X, int64_t N, int d, const int64_t* offsets, const int32_t* members,
                            int32_t n_buckets, int32_t M, int32_t* out_id, float* out_d)
{
    (void)N;
    for (int32_t b = 0; b < n_buckets; ++b) {
        const int64_t lo = offsets[b], hi = offsets[b + 1];
        const int64_t nb = hi - lo;
        if (nb <= 0) continue;
        #pragma omp parallel
        {
            orc_pair* p = (orc_pair*)malloc(sizeof(orc_pair) * (size_t)(nb > 0 ? nb : 1));
            #pragma omp for schedule(dynamic, 16)
            for (int64_t j = lo; j < hi; ++j) {
                const int32_t q = members[j];
                const float* xq = X + (int64_t)q * d;
                int64_t n = 0;
                for (int64_t t = lo; t < hi; ++t) {
                    const int32_t c = members[t];
                    if (c == q) continue;
                    p[n].d = exact_l2(xq, X + (int64_t)c * d, d);
                    p[n].id = c;
                    ++n;
                }
                select_topk(p, n, M, out_id + j * M, out_d + j * M);
            }
            free(p);
        }
    }
}

/* exact brute-force kNN of sampled queries over the whole dataset,   */
/* self excluded: bucketDemo/build_knn.py:98-149 build_exact_knn      */
/* (self masked to +inf at :36-38), top-k by (distance, id).          */
ORC_API void orc_exact_knn(const float* X, int64_t N, int d, const int64_t* queries, int64_t S, int32_t k,
                           int32_t* out_id, float* out_d)
{
    #pragma omp parallel
    {
        orc_pair* p = (orc_pair*)malloc(sizeof(orc_pair) * (size_t)N);
        #pragma omp for schedule(dynamic, 4)
        for (int64_t s = 0; s < S; ++s) {
            const int64_t q = queries[s];
            const float* xq = X + q * d;
            int64_t n = 0;
            for (int64_t c = 0; c < N; ++c) {
                if (c == q) continue;
                p[n].d = exact_l2(xq, X + c * d, d);
                p[n].id = (int32_t)c;
                ++n;
            }
            select_topk(p, n, k, out_id + s * k, out_d + s * k);
        }
        free(p);
    }
}

/* ------------------------------------------------------------------ */
/* a7: merge two ascending M-lists of one point                       */
/* bucketDemo/buildBucket/src/bucket.cu:5025-5059 resident_merge_kernel: */
/* two-pointer merge, running side first on equal distance, a new id  */
/* already present in the running list is skipped, pad -1 / +inf.     */
/* ------------------------------------------------------------------ */
static void merge_one(const int32_t* an, const float* ad, const int32_t* bn, const float* bd, int32_t* on,
                      float* od, int M)
{
    int na = 0; while (na < M && an[na] >= 0) ++na;
    int nb = 0; while (nb < M && bn[nb] >= 0) ++nb;
    int i = 0, j = 0, w = 0;
    while (w < M && (i < na || j < nb)) {
        if (j >= nb || (i < na && ad[i] <= bd[j])) {
            on[w] = an[i]; od[w] = ad[i]; ++w; ++i;
        } else {
            int32_t id = bn[j];
            int dup = 0;
            for (int k = 0; k < na; ++k) if (an[k] == id) { dup = 1; break; }
            if (!dup) { on[w] = id; od[w] = bd[j]; ++w; }
            ++j;
        }
    }
    for (; w < M; ++w) { on[w] = -1; od[w] = INFINITY; }
}

ORC_API void orc_merge_lists(const int32_t* run_n, const float* run_d, const int32_t* new_n, const float* new_d,
                             int32_t* out_n, float* out_d, int64_t N, int32_t M)
{
    #pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < N; ++r)
        merge_one(run_n + r * M, run_d + r * M, new_n + r * M, new_d + r * M, out_n + r * M, out_d + r * M, M);
}

/* per point: merge the list of its lower-bucket membership (running) */
/* with the list of its higher-bucket membership (new).               */
ORC_API void orc_merge_memberships(const int32_t* list_n, const float* list_d, const int64_t* mem_row, int64_t N,
                                   int32_t M, int32_t* out_n, float* out_d)
{
    #pragma omp parallel for schedule(static)
    for (int64_t p = 0; p < N; ++p) {
        int64_t r0 = mem_row[2 * p], r1 = mem_row[2 * p + 1];
        merge_one(list_n + r0 * M, list_d + r0 * M, list_n + r1 * M, list_d + r1 * M, out_n + p * M,
                  out_d + p * M, M);
    }
}

/* ------------------------------------------------------------------ */
/* sanitize: bucketDemo/buildBucket/src/optimize.cu:95-133            */
/* (sanitize_to_uint32_inplace) and bucket.cu:8447-8462: padding,     */
/* out-of-range ids and self loops become the row's first valid       */
/* neighbour, or (i+1)%N when the row has none.                       */
/* ------------------------------------------------------------------ */
ORC_API int64_t orc_sanitize(const int32_t* knn, int64_t N, int32_t M, uint32_t* out)
{
    int64_t n_pad = 0;
    #pragma omp parallel for reduction(+:n_pad) schedule(static)
    for (int64_t i = 0; i < N; ++i) {
        const int32_t* row = knn + i * M;
        uint32_t* o = out + i * M;
        uint32_t fallback = (uint32_t)((i + 1) % N);
        for (int j = 0; j < M; ++j) {
            int32_t v = row[j];
            if (v >= 0 && (int64_t)v < N && (int64_t)v != i) { fallback = (uint32_t)v; break; }
        }
        for (int j = 0; j < M; ++j) {
            int32_t v = row[j];
            if (v < 0 || (int64_t)v >= N || (int64_t)v == i) { o[j] = fallback; if (v < 0) ++n_pad; }
            else o[j] = (uint32_t)v;
        }
    }
    return n_pad;
}

/* ------------------------------------------------------------------ */
/* row sort by exact distance, stable on ties (column order):         */
/* bucketDemo/buildBucket/src/prune_windowed_core.hpp:134-175          */
/* sort_row_by_l2 (candidates < 0 dropped, -1 padding at the end).    */
/* ------------------------------------------------------------------ */
typedef struct { float d; int32_t id; int32_t col; } orc_cand;

static int cand_cmp(const void* pa, const void* pb)
{
    const orc_cand* a = (const orc_cand*)pa; const orc_cand* b = (const orc_cand*)pb;
    if (a->d < b->d) return -1;
    if (a->d > b->d) return 1;
    return (a->col > b->col) - (a->col < b->col);
}

ORC_API void orc_sort_rows_l2(const float* X, int d, const int32_t* knn, int64_t N, int32_t M, int32_t* out)
{
    #pragma omp parallel
    {
        orc_cand* c = (orc_cand*)malloc(sizeof(orc_cand) * (size_t)M);
        #pragma omp for schedule(static)
        for (int64_t i = 0; i < N; ++i) {
            int n = 0;
            for (int j = 0; j < M; ++j) {
                int32_t id = knn[i * M + j];
                if (id < 0) continue;
                c[n].d = exact_l2(X + i * d, X + (int64_t)id * d, d);
                c[n].id = id; c[n].col = j; ++n;
            }
            qsort(c, (size_t)n, sizeof(orc_cand), cand_cmp);
            for (int j = 0; j < M; ++j) out[i * M + j] = j < n ? c[j].id : -1;
        }
        free(c);
    }
}

/* ------------------------------------------------------------------ */
/* a8: CAGRA rank-based detour-count prune (full window)              */
/* bucketDemo/buildBucket/src/prune_windowed_core.hpp:190-232          */
/* compute_detour_counts: count[kAB] = #{kAD < kAB : row[kAB] is in    */
/* the row of row[kAD]}, each (kAD, kAB) counted once.                */
/* ------------------------------------------------------------------ */
ORC_API void orc_detour_counts(const uint32_t* g, int64_t N, int32_t M, int64_t a, uint32_t* cnt)
{
    (void)N;
    const uint32_t* ra = g + a * M;
    for (int k = 0; k < M; ++k) cnt[k] = 0;
    for (int kAD = 0; kAD < M - 1; ++kAD) {
        const uint32_t* rd = g + (int64_t)ra[kAD] * M;
        for (int kAB = kAD + 1; kAB < M; ++kAB) {
            const uint32_t b = ra[kAB];
            for (int kDB = 0; kDB < M; ++kDB)
                if (rd[kDB] == b) { cnt[kAB]++; break; }
        }
    }
}

/* prune_windowed_core.hpp:238-263 select_pruned_row: smallest detour */
/* count first, rank order within one count.                          */
static void select_row(const uint32_t* row, int M, const uint32_t* cnt, int K, uint32_t* out)
{
    int pk = 0;
    uint32_t num = 0;
    while (pk < K) {
        uint32_t next = UINT32_MAX;
        for (int k = 0; k < M; ++k) {
            uint32_t dk = cnt[k];
            if (dk > num && dk < next) next = dk;
            if (dk != num) continue;
            out[pk++] = row[k];
            if (pk >= K) break;
        }
        if (pk >= K || next == UINT32_MAX) break;
        num = next;
    }
}

ORC_API void orc_prune(const uint32_t* g, int64_t N, int32_t M, int32_t K, uint32_t* out)
{
    #pragma omp parallel
    {
        uint32_t* cnt = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)M);
        #pragma omp for schedule(dynamic, 256)
        for (int64_t a = 0; a < N; ++a) {
            orc_detour_counts(g, N, M, a, cnt);
            select_row(g + a * M, M, cnt, K, out + a * K);
        }
        free(cnt);
    }
}

/* ------------------------------------------------------------------ */
/* a9: reverse edges                                                  */
/* reverse list of j = sources i with j in pruned(i), ordered by      */
/* (rank of j in row i, i), capped at K: edge_chunk_accumulator.hpp:  */
/* 386-469 TopKReverseStore (L = K) / :235-284 build_rank_ordered_csr; */
/* merged weakest-to-strongest with the first K/2 forward edges       */
/* protected: :471-494 merge_rank_ordered_into_row.                   */
/* ------------------------------------------------------------------ */
static void merge_rev_row(uint32_t* row, const uint32_t* src, uint32_t count, uint32_t K)
{
    const uint32_t np = K / 2;
    uint32_t k = count;
    while (k > 0) {
        k--;
        uint32_t i = src[k];
        uint32_t pos = K;
        for (uint32_t p = 0; p < K; ++p) if (row[p] == i) { pos = p; break; }
        if (pos < np) continue;
        uint32_t ns = (pos == K) ? (K - np - 1) : (pos - np);
        for (uint32_t s = ns; s > 0; --s) row[np + s] = row[np + s - 1];
        row[np] = i;
    }
}

ORC_API void orc_merge_rev_row(uint32_t* row, const uint32_t* src, uint32_t count, uint32_t K)
{
    merge_rev_row(row, src, count, K);
}

ORC_API int orc_reverse_merge(uint32_t* graph, int64_t N, int32_t K)
{
    uint64_t* keys = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)N * (size_t)K);
    uint32_t* cnt = (uint32_t*)calloc((size_t)N, sizeof(uint32_t));
    if (!keys || !cnt) { free(keys); free(cnt); return 2; }
    /* sequential insertion keeps each destination's K smallest keys;  */
    /* the result does not depend on insertion order.                  */
    for (int64_t i = 0; i < N; ++i) {
        for (int32_t r = 0; r < K; ++r) {
            uint32_t dst = graph[i * K + r];
            if ((int64_t)dst >= N) continue;
            uint64_t key = ((uint64_t)(uint32_t)r << 32) | (uint64_t)(uint32_t)i;
            uint64_t* row = keys + (int64_t)dst * K;
            uint32_t c = cnt[dst], pos;
            if (c < (uint32_t)K) { pos = c; cnt[dst] = c + 1; }
            else if (key < row[K - 1]) pos = (uint32_t)K - 1;
            else continue;
            while (pos > 0 && row[pos - 1] > key) { row[pos] = row[pos - 1]; --pos; }
            row[pos] = key;
        }
    }
    #pragma omp parallel
    {
        uint32_t* src = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)K);
        #pragma omp for schedule(static)
        for (int64_t j = 0; j < N; ++j) {
            uint32_t c = cnt[j];
            for (uint32_t t = 0; t < c; ++t) src[t] = (uint32_t)(keys[j * K + t] & 0xffffffffu);
            merge_rev_row(graph + j * K, src, c, (uint32_t)K);
        }
        free(src);
    }
    free(keys);
    free(cnt);
    return 0;
}

/* cuvs::neighbors::cagra::helpers::optimize as called at             */
/* bucketDemo/buildBucket/src/optimize.cu:396: prune M -> K on an     */
/* already distance-sorted, sanitized graph, then reverse-edge merge. */
ORC_API int orc_optimize(const uint32_t* knn, int64_t N, int32_t M, int32_t K, uint32_t* out)
{
    if (K <= 0 || K > M) return 1;
    orc_prune(knn, N, M, K, out);
    return orc_reverse_merge(out, N, K);
}

ORC_API int orc_num_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* ------------------------------------------------------------------ */
/* graph search (bucketDemo/search.py:20-93 graph_search_single)      */
/* ------------------------------------------------------------------ */
/* The efSearch-style best-first search of the reference, per query:    */
/* the given entry points (already drawn and de-duplicated, ascending:  */
/* np.unique of rng.integers at :40-41) are visited in order; a min     */
/* "heap" of (distance, id) candidates (heapq on tuples: :52-53) is     */
/* expanded until the popped distance exceeds the worst of the best     */
/* list once that holds ef entries (:54-57); the best list is an array  */
/* in insertion order, appended while short and otherwise overwritten   */
/* at the first position of its maximum when the new distance is       */
/* smaller (:45-50, :73-80).  Neighbour ids outside [0, N) and visited  */
/* ids are skipped (:62-67).  Output: the best list sorted by distance  */
/* (ties by id), first topk, padded with -1 / +inf (:82-86).            */
/* Distances: the exact fp32 chain over ascending dims (for 8-bit data  */
/* every partial sum is an integer below 2^24, so the order of the      */
/* reference's float32 dot is immaterial).                              */
typedef struct { float d; uint32_t id; } orc_scand;

static int cand_less(orc_scand a, orc_scand b) { return a.d < b.d || (a.d == b.d && a.id < b.id); }

static void heap_push(orc_scand* h, int64_t* n, orc_scand c)
{
    int64_t i = (*n)++;
    h[i] = c;
    while (i > 0) {
        int64_t p = (i - 1) / 2;
        if (!cand_less(h[i], h[p])) break;
        orc_scand t = h[i]; h[i] = h[p]; h[p] = t;
        i = p;
    }
}

static orc_scand heap_pop(orc_scand* h, int64_t* n)
{
    orc_scand top = h[0];
    h[0] = h[--(*n)];
    int64_t i = 0;
    for (;;) {
        int64_t l = 2 * i + 1, r = l + 1, m = i;
        if (l < *n && cand_less(h[l], h[m])) m = l;
        if (r < *n && cand_less(h[r], h[m])) m = r;
        if (m == i) break;
        orc_scand t = h[i]; h[i] = h[m]; h[m] = t;
        i = m;
    }
    return top;
}

static void best_update(float* bd, uint32_t* bi, int32_t* bs, int32_t ef, float d, uint32_t id)
{
    if (*bs < ef) {
        bd[*bs] = d;
        bi[*bs] = id;
        ++*bs;
        return;
    }
    int32_t w = 0;
    for (int32_t j = 1; j < ef; ++j)
        if (bd[j] > bd[w]) w = j;
    if (d < bd[w]) { bd[w] = d; bi[w] = id; }
}

static float best_worst(const float* bd, int32_t bs)
{
    float w = bd[0];
    for (int32_t j = 1; j < bs; ++j)
        if (bd[j] > w) w = bd[j];
    return w;
}

static int cmp_best(const void* a, const void* b)
{
    const orc_scand* x = (const orc_scand*)a;
    const orc_scand* y = (const orc_scand*)b;
    if (x->d < y->d) return -1;
    if (x->d > y->d) return 1;
    return x->id < y->id ? -1 : (x->id > y->id);
}

/* base: N x d f32; graph: N x kg uint32; queries: nq x d f32; entries: nq x ne (ascending, -1 = unused). */
ORC_API void orc_graph_search(const float* base, int64_t N, int32_t d, const uint32_t* graph, int32_t kg,
                              const float* queries, int64_t nq, const int32_t* entries, int32_t ne, int32_t topk,
                              int32_t ef, int32_t* out_ids, float* out_dists)
{
#pragma omp parallel for schedule(dynamic, 4)
    for (int64_t q = 0; q < nq; ++q) {
        const float* x = queries + q * d;
        unsigned char* visited = (unsigned char*)calloc((size_t)N, 1);
        orc_scand* heap = (orc_scand*)malloc(sizeof(orc_scand) * (size_t)(N + ne + 1));
        float* bd = (float*)malloc(sizeof(float) * (size_t)ef);
        uint32_t* bi = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)ef);
        int64_t hn = 0;
        int32_t bs = 0;
        for (int32_t e = 0; e < ne; ++e) {
            const int32_t s = entries[q * ne + e];
            if (s < 0 || (int64_t)s >= N || visited[s]) continue;
            visited[s] = 1;
            const float ds = exact_l2(x, base + (int64_t)s * d, d);
            orc_scand c = {ds, (uint32_t)s};
            heap_push(heap, &hn, c);
            best_update(bd, bi, &bs, ef, ds, (uint32_t)s);
        }
        while (hn > 0) {
            const orc_scand u = heap_pop(heap, &hn);
            if (bs >= ef && u.d > best_worst(bd, bs)) break;
            const uint32_t* nb = graph + (int64_t)u.id * kg;
            for (int32_t j = 0; j < kg; ++j) {
                const uint32_t v = nb[j];
                if ((int64_t)v >= N || visited[v]) continue;
                visited[v] = 1;
                const float dv = exact_l2(x, base + (int64_t)v * d, d);
                orc_scand c = {dv, v};
                heap_push(heap, &hn, c);
                best_update(bd, bi, &bs, ef, dv, v);
            }
        }
        orc_scand* srt = (orc_scand*)malloc(sizeof(orc_scand) * (size_t)(bs > 0 ? bs : 1));
        for (int32_t j = 0; j < bs; ++j) { srt[j].d = bd[j]; srt[j].id = bi[j]; }
        qsort(srt, (size_t)bs, sizeof(orc_scand), cmp_best);
        for (int32_t j = 0; j < topk; ++j) {
            out_ids[q * topk + j] = j < bs ? (int32_t)srt[j].id : -1;
            out_dists[q * topk + j] = j < bs ? srt[j].d : INFINITY;
        }
        free(srt); free(bi); free(bd); free(heap); free(visited);
    }
}

/* ------------------------------------------------------------------ */
/* bucket-contiguous renumbering                                        */
/* ------------------------------------------------------------------ */

/* compute_bucket_reorder (bucketDemo/buildBucket/src/bucket.cu:8356-8417):
 * bucket b = assign[i * stride]; ranges laid out in `order` (NULL: 0..B-1);
 * inside a bucket ascending old id; inv[new] = old; offsets[pos] (B+1).
 * Returns the number of points placed (n when every point has a bucket). */
ORC_API int64_t orc_bucket_reorder(const int32_t* assign, int64_t n, int32_t stride, int32_t B, const int32_t* order,
                                   uint32_t* inv, int64_t* offsets)
{
    int64_t* count = (int64_t*)calloc((size_t)B, sizeof(int64_t));
    int64_t* start = (int64_t*)calloc((size_t)B, sizeof(int64_t));
    for (int64_t i = 0; i < n; ++i) {
        const int32_t b = assign[i * stride];
        if (b >= 0 && b < B) count[b]++;
    }
    int64_t run = 0;
    offsets[0] = 0;
    for (int32_t p = 0; p < B; ++p) {
        const int32_t b = order ? order[p] : p;
        start[b] = run;
        run += count[b];
        offsets[p + 1] = run;
    }
    for (int64_t i = 0; i < n; ++i) {
        const int32_t b = assign[i * stride];
        if (b >= 0 && b < B) inv[start[b]++] = (uint32_t)i;
    }
    free(count);
    free(start);
    return run;
}

/* translate_graph_to_original_order / translate_npy_to_original_order
 * (translate_graph_ids.hpp:75-200) for to_original = 1: row inv[i] gets row i with
 * ids mapped through inv; to_original = 0: row i gets old row inv[i] with ids
 * mapped old -> new.  Negative ids stay -1 (keep_padding) else count as bad, like
 * ids >= n.  Returns the number of bad ids (0 on success); -1 when inv is not a
 * permutation of [0, n). */
ORC_API int64_t orc_permute_graph(const int32_t* g, int64_t n, int32_t m, const uint32_t* inv, int32_t to_original,
                                  int32_t keep_padding, int32_t* out)
{
    int32_t* perm = (int32_t*)malloc(sizeof(int32_t) * (size_t)n);
    for (int64_t i = 0; i < n; ++i) perm[i] = -1;
    for (int64_t i = 0; i < n; ++i) {
        if ((int64_t)inv[i] >= n || perm[inv[i]] != -1) { free(perm); return -1; }
        perm[inv[i]] = (int32_t)i;
    }
    int64_t bad = 0;
    for (int64_t i = 0; i < n; ++i) {
        const int64_t src = to_original ? i : (int64_t)inv[i];
        const int64_t dst = to_original ? (int64_t)inv[i] : i;
        for (int32_t j = 0; j < m; ++j) {
            const int32_t v = g[src * m + j];
            int32_t w = -1;
            if (v < 0) bad += !keep_padding;
            else if ((int64_t)v >= n) ++bad;
            else w = to_original ? (int32_t)inv[v] : perm[v];
            out[dst * m + j] = w;
        }
    }
    free(perm);
    return bad;
}

/* compute_bucket_processing_order (bucket_order.hpp:143-200) over the flat
 * bucket graph adj (B x K; adjacency_from_flat_graph :202-218 drops ids that are
 * the bucket itself or >= B; negative ids are dropped here too).  Plain O(B^2)
 * selection: next = argmax (score, id) over touched unplaced buckets, else the
 * lowest unplaced id; score = shared neighbour entries with the last `window`
 * placed buckets. */
ORC_API void orc_bucket_order(const int32_t* adj, int32_t B, int32_t K, int32_t window, int32_t* order)
{
    if (window < 1) window = 1;
    int64_t* score = (int64_t*)calloc((size_t)B, sizeof(int64_t));
    char* placed = (char*)calloc((size_t)B, 1);
    char* touched = (char*)calloc((size_t)B, 1);
    int32_t* deg = (int32_t*)calloc((size_t)B, sizeof(int32_t));
    int32_t* nb = (int32_t*)malloc(sizeof(int32_t) * (size_t)B * (size_t)(K > 0 ? K : 1));
    for (int32_t v = 0; v < B; ++v)
        for (int32_t k = 0; k < K; ++k) {
            const int32_t u = adj[(int64_t)v * K + k];
            if (u >= 0 && u < B && u != v) nb[(int64_t)v * K + deg[v]++] = u;
        }
    /* score change of every unplaced v when x enters (+1) or leaves (-1) the window:
     * for each neighbour entry u of x, each entry of v equal to u */
#define ORC_SHIFT(x, delta)                                                           \
    do {                                                                              \
        for (int32_t a_ = 0; a_ < deg[x]; ++a_) {                                     \
            const int32_t u_ = nb[(int64_t)(x) * K + a_];                             \
            for (int32_t v_ = 0; v_ < B; ++v_) {                                      \
                if (placed[v_]) continue;                                             \
                for (int32_t b_ = 0; b_ < deg[v_]; ++b_)                              \
                    if (nb[(int64_t)v_ * K + b_] == u_) { score[v_] += (delta); touched[v_] = 1; } \
            }                                                                         \
        }                                                                             \
    } while (0)
    int32_t start = 0;
    for (int32_t v = 1; v < B; ++v)
        if (deg[v] > deg[start]) start = v;
    order[0] = start;
    placed[start] = 1;
    ORC_SHIFT(start, 1);
    for (int32_t i = 1; i < B; ++i) {
        if (i > window) ORC_SHIFT(order[i - window - 1], -1);
        int32_t pick = -1;
        for (int32_t v = 0; v < B; ++v)
            if (!placed[v] && touched[v] && (pick < 0 || score[v] > score[pick] || (score[v] == score[pick] && v > pick)))
                pick = v;
        if (pick < 0)
            for (int32_t v = 0; v < B && pick < 0; ++v)
                if (!placed[v]) pick = v;
        order[i] = pick;
        placed[pick] = 1;
        ORC_SHIFT(pick, 1);
    }
#undef ORC_SHIFT
    free(score); free(placed); free(touched); free(deg); free(nb);
}

/* ------------------------------------------------------------------ */
/* reference bucketing (the reference's bucket2 tool)                   */
/* ------------------------------------------------------------------ */

static uint64_t orc_mix64(uint64_t x)
{
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static uint64_t orc_kpar_bits(uint64_t seed, int round, uint64_t i)
{
    return orc_mix64(seed * 0x9E3779B97F4A7C15ull + 0xD1B54A32D192ED03ull * (uint64_t)(round + 1) + i) >> 11;
}

/* KMeans|| (bucketDemo/buildBucket/src/bucket.cu:2919-3117): first point from the seed; three
 * rounds; psi = strided-subsample fp64 sum of the current squared distances (stride N/16384,
 * lane-strided partial sums reduced by a 16-8-4-2-1 tree) scaled by N / samples; point i is
 * taken when not yet taken and u_i < 0.5 n_req d_i / psi; distances refreshed with the new
 * candidates except after the last round.  Then (:3150-3172) a uniform subsample of the
 * candidates down to n_req (partial Fisher-Yates).  Writes the centroid point ids, returns
 * their number (<= n_req). */
ORC_API int64_t orc_kmeans_parallel(const float* X, int64_t N, int d, int64_t n_req, uint64_t seed, int32_t* out)
{
    const int32_t c0 = (int32_t)(orc_mix64(seed ^ 0xA0761D6478BD642Full) % (uint64_t)N);
    unsigned char* chosen = (unsigned char*)calloc((size_t)N, 1);
    float* min_d = (float*)malloc(sizeof(float) * (size_t)N);
    int32_t* cand = (int32_t*)malloc(sizeof(int32_t) * (size_t)N);
    int64_t n_cand = 0;
    cand[n_cand++] = c0;
    chosen[c0] = 1;
    for (int64_t i = 0; i < N; ++i) min_d[i] = exact_l2(X + i * d, X + (int64_t)c0 * d, d);
    const double lk = 1.5 / 3.0 * (double)n_req;
    const int64_t stride = N / 16384 > 1 ? N / 16384 : 1;
    const int64_t sub_n = N / stride;
    for (int r = 0; r < 3; ++r) {
        double s[32];
        for (int l = 0; l < 32; ++l) {
            s[l] = 0.0;
            for (int64_t j = l; j < sub_n; j += 32) s[l] += (double)min_d[j * stride];
        }
        for (int o = 16; o > 0; o >>= 1)
            for (int l = 0; l < o; ++l) s[l] += s[l + o];
        const double psi = s[0] * ((double)N / (double)sub_n);
        const int64_t first_new = n_cand;
        for (int64_t i = 0; i < N; ++i) {
            const double u = (double)orc_kpar_bits(seed, r, (uint64_t)i) * 0x1.0p-53;
            if (!chosen[i] && u < (lk * (double)min_d[i]) / psi) {
                chosen[i] = 1;
                cand[n_cand++] = (int32_t)i;
            }
        }
        if (n_cand == first_new) break;
        if (r + 1 < 3) {
#pragma omp parallel for schedule(static)
            for (int64_t i = 0; i < N; ++i) {
                float m = min_d[i];
                for (int64_t c = first_new; c < n_cand; ++c) {
                    const float v = exact_l2(X + i * d, X + (int64_t)cand[c] * d, d);
                    if (v < m) m = v;
                }
                min_d[i] = m;
            }
        }
    }
    int64_t n_out = n_cand;
    if (n_cand <= n_req) {
        memcpy(out, cand, sizeof(int32_t) * (size_t)n_cand);
    } else {
        int32_t* perm = (int32_t*)malloc(sizeof(int32_t) * (size_t)n_cand);
        for (int64_t k = 0; k < n_cand; ++k) perm[k] = (int32_t)k;
        const uint64_t s2 = seed ^ 0x5851F42D4C957F2Dull;
        for (int64_t k = 0; k < n_req; ++k) {
            const int64_t j = k + (int64_t)(orc_mix64(s2 + (uint64_t)k) % (uint64_t)(n_cand - k));
            const int32_t t = perm[k]; perm[k] = perm[j]; perm[j] = t;
        }
        for (int64_t k = 0; k < n_req; ++k) out[k] = cand[perm[k]];
        free(perm);
        n_out = n_req;
    }
    free(chosen); free(min_d); free(cand);
    return n_out;
}

/* Balanced 1-way assignment (bucket.cu:1655-1660, :2276-2301): centroid points stay in their
 * own bucket, every bucket starts at size 1; the other points, in index order, each choose
 * against the sizes left by every earlier point (the reference's loop run by one thread: its
 * OpenMP threads update the sizes with relaxed atomics, whose interleaving is not reproducible).
 * rule 0 (the reference's default): the second-nearest centroid c2 when size(c2) < 0.8 size(c1)
 * in double; rule 1 (BUCKET2_ASSIGN_RULE=diskjoin, :2290-2292): c2 when size(c2) < size(c1) and
 * d2 < 1.2f * d1 in float, d = top2_d (the squared distances of the two centroids).  Returns
 * the number of top-2 entries out of range (0 on success). */
ORC_API int64_t orc_balanced_assign(const int32_t* top2, const float* top2_d, int64_t N, int32_t B,
                                    const int32_t* cid, int32_t rule, int32_t* assign)
{
    int64_t* size = (int64_t*)malloc(sizeof(int64_t) * (size_t)B);
    unsigned char* is_c = (unsigned char*)calloc((size_t)N, 1);
    int64_t bad = 0;
    for (int32_t c = 0; c < B; ++c) { size[c] = 1; assign[cid[c]] = c; is_c[cid[c]] = 1; }
    for (int64_t i = 0; i < N; ++i) {
        if (is_c[i]) continue;
        const int32_t c1 = top2[2 * i], c2 = top2[2 * i + 1];
        if (c1 < 0 || c1 >= B || c2 < 0 || c2 >= B) { ++bad; continue; }
        int take2;
        if (rule == 1) {
            const float d1 = top2_d[2 * i], d2 = top2_d[2 * i + 1];
            take2 = size[c2] < size[c1] && d2 < 1.2f * d1;
        } else {
            take2 = (double)size[c2] < 0.8 * (double)size[c1];
        }
        const int32_t ch = take2 ? c2 : c1;
        assign[i] = ch;
        size[ch]++;
    }
    free(size); free(is_c);
    return bad;
}

/* The pools of the resident round (bucket.cu:5317-5346): members[N] grouped by bucket in
 * ascending point id with off[B+1]; for bucket c its S = P + 1 segments, segment 0 bucket c
 * itself and segment j the neighbour adj[c][j-1] (-1 when outside [0, B)): seg_b[c*S + j], and
 * seg_ofs[c*S + j] the offset of the segment in c's pool (a -1 segment is empty); pool[c] = the
 * pool's length. */
ORC_API void orc_pool_tables(const int32_t* assign, int64_t N, int32_t B, const int32_t* adj, int32_t P,
                             int64_t* off, int32_t* members, int32_t* seg_b, int64_t* seg_ofs, int64_t* pool)
{
    for (int32_t c = 0; c <= B; ++c) off[c] = 0;
    for (int64_t i = 0; i < N; ++i) off[assign[i] + 1]++;
    for (int32_t c = 0; c < B; ++c) off[c + 1] += off[c];
    int64_t* cur = (int64_t*)malloc(sizeof(int64_t) * (size_t)(B > 0 ? B : 1));
    for (int32_t c = 0; c < B; ++c) cur[c] = off[c];
    for (int64_t i = 0; i < N; ++i) members[cur[assign[i]]++] = (int32_t)i;
    free(cur);
    const int64_t S = (int64_t)P + 1;
    for (int32_t c = 0; c < B; ++c) {
        int64_t o = 0;
        for (int64_t j = 0; j < S; ++j) {
            int32_t b = j == 0 ? c : adj[(int64_t)c * P + j - 1];
            if (b < 0 || b >= B) b = -1;
            seg_b[c * S + j] = b;
            seg_ofs[c * S + j] = o;
            if (b >= 0) o += off[b + 1] - off[b];
        }
        pool[c] = o;
    }
}

/* Per-bucket pool kNN (bucket.cu:5310-5365, the resident round): the pool of bucket c is its
 * points (ascending id) followed by those of adj[c][0..P) (ids >= B or negative skipped);
 * each point of c gets the exact top-M of its pool, itself excluded, by (distance, id). */
ORC_API void orc_pool_knn(const float* X, int64_t N, int d, const int32_t* assign, int32_t B, const int32_t* adj,
                          int32_t P, int32_t M, int32_t* out_ids, float* out_d)
{
    const int64_t S = (int64_t)P + 1;
    int64_t* off = (int64_t*)malloc(sizeof(int64_t) * ((size_t)B + 1));
    int32_t* mem = (int32_t*)malloc(sizeof(int32_t) * (size_t)(N > 0 ? N : 1));
    int32_t* seg_b = (int32_t*)malloc(sizeof(int32_t) * (size_t)(B * S));
    int64_t* seg_ofs = (int64_t*)malloc(sizeof(int64_t) * (size_t)(B * S));
    int64_t* psz = (int64_t*)malloc(sizeof(int64_t) * (size_t)B);
    orc_pool_tables(assign, N, B, adj, P, off, mem, seg_b, seg_ofs, psz);
#pragma omp parallel for schedule(dynamic)
    for (int32_t c = 0; c < B; ++c) {
        const int64_t ps = psz[c];
        int32_t* pool = (int32_t*)malloc(sizeof(int32_t) * (size_t)(ps > 0 ? ps : 1));
        orc_pair* cand = (orc_pair*)malloc(sizeof(orc_pair) * (size_t)(ps > 0 ? ps : 1));
        for (int64_t j = 0; j < S; ++j) {
            const int32_t b = seg_b[c * S + j];
            if (b < 0) continue;
            for (int64_t k = off[b]; k < off[b + 1]; ++k) pool[seg_ofs[c * S + j] + k - off[b]] = mem[k];
        }
        for (int64_t q = off[c]; q < off[c + 1]; ++q) {
            const int32_t pt = mem[q];
            int64_t nc = 0;
            for (int64_t k = 0; k < ps; ++k) {
                if (k == q - off[c]) continue;  /* the point itself (its own position in segment 0) */
                cand[nc].d = exact_l2(X + (int64_t)pt * d, X + (int64_t)pool[k] * d, d);
                cand[nc].id = pool[k];
                ++nc;
            }
            select_topk(cand, nc, M, out_ids + (int64_t)pt * M, out_d + (int64_t)pt * M);
        }
        free(pool); free(cand);
    }
    free(off); free(mem); free(seg_b); free(seg_ofs); free(psz);
}
