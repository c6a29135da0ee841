/*
 * gta.h -- C ABI of libgta, the B200 (sm_100a) bucketed kNN-graph / CAGRA build.
 *
 * Drop-in boundary for the reference's build path (loulankxh/GPU-talored-ANN;
 * paths below are relative to the reference project root).  Plain pointers and
 * sizes only; no exception crosses this boundary.
 *
 * Status codes (every int-returning entry point):
 *   GTA_OK 0, GTA_EINVAL 1 (bad argument), GTA_ENOMEM 2 (does not fit / out of
 *   memory; the reference's `optimize` exits 2 for "does not fit",
 *   bucketDemo/buildBucket/src/optimize.cu:307), GTA_ECUDA 3, GTA_ENCCL 4,
 *   GTA_EDATA 5 (input data failed a check: id out of range, not a permutation,
 *   malformed file).  gta_last_error() returns the message of the calling
 *   thread's last failure.
 *
 * Memory: pointers flagged `on_device` are CUDA device pointers on the current
 * device; all work is ordered on `stream` (a cudaStream_t, NULL = default
 * stream).  Stage entry points (gta_assign_topk ... gta_reverse_merge) take
 * device pointers only and are stream-ordered.  Scratch memory comes from a
 * workspace the library keeps per (device, stream): it grows to the largest
 * call seen on that stream and is reused by later calls on the same stream
 * (held until gta_release_workspace).  Calls on one stream are ordered by the
 * stream; the same stream must not be driven from two host threads at once.
 * Entry points that return results in host memory synchronize the stream.
 */
#ifndef GTA_H_
#define GTA_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GTA_OK 0
#define GTA_EINVAL 1
#define GTA_ENOMEM 2
#define GTA_ECUDA 3
#define GTA_ENCCL 4
#define GTA_EDATA 5

/* element types of a dataset (the BIGANN file extensions .fbin / .u8bin / .i8bin) */
#define GTA_F32 0
#define GTA_U8 1
#define GTA_I8 2

/* metrics: L2 = squared Euclidean; IP is served as L2 over rows the caller has
 * L2-normalised (identical neighbour order: |x-y|^2 = 2 - 2<x,y>). */
#define GTA_L2 0
#define GTA_IP 1

/* A dataset: n row-major rows of d elements (BIGANN layout,
 * bucketDemo/buildBucket/src/load.hpp:43-135 without the 8-byte header). */
typedef struct {
    const void* data;
    int64_t n;
    int32_t d;
    int32_t dtype;     /* GTA_F32 / GTA_U8 / GTA_I8 */
    int32_t metric;    /* GTA_L2 / GTA_IP */
    int32_t on_device; /* 0: host pointer (copied to the device once); 1: device pointer;
                          2: host memory read in place by gta_build_bucket / gta_build_cagra (the
                          pages are registered pinned, mapped and read-only for the call, the
                          kernels read rows through the host link and the whole dataset is never
                          copied to the device: datasets larger than the device's memory, with
                          device_budget bounding the bucket stage; other entry points take 0 or 1) */
} gta_dataset;

/* Parameters of the bucketed kNN build (bucket2 / build_bucket.py). */
typedef struct {
    int32_t n_buckets;      /* B: k-means centroids = buckets */
    int32_t kmeans_iters;   /* Lloyd iterations */
    int32_t knn_degree;     /* M: intermediate kNN degree (<= 128) */
    int32_t rounds;         /* bucket2 -t: whole builds with seeds seed, seed+1, ..., each
                               round's lists merged into the running lists (0 or 1: one round) */
    int64_t kmeans_sample;  /* points used by k-means; 0 = min(0.1, 1e7/N) of N */
    uint64_t seed;
    const float* init_centroids; /* optional B x d initial centroids (skips k-means++) */
    int32_t init_on_device;
    int32_t out_on_device;  /* outputs (knn lists, centroids_out, top2_out) are device pointers */
    float* centroids_out;   /* optional B x d final centroids */
    int32_t* top2_out;      /* optional N x 2 bucket ids (nearest, second nearest) */
    int64_t device_budget;  /* bytes the bucket kNN stage may hold at once (0: one pass when the
                               stage needs at most a quarter of the device's memory, else 80% of the
                               free device memory); when the memberships' pool rows and lists exceed
                               it, buckets are processed in ascending batches that fit, with the
                               same result */
} gta_bucket_params;

typedef struct {
    gta_bucket_params bucket;
    int32_t graph_degree;   /* K: final CAGRA degree (<= M) */
    int32_t reserved0;
} gta_cagra_params;

/* Parameters of the reference-bucketing build (the bucketing of the reference's
 * bucket2 tool): data-point centroids by KMeans||, every point in one bucket
 * (nearest or second-nearest centroid, balancing bucket sizes), each bucket's
 * points searched against a pool of the bucket and its nprobe nearest buckets. */
typedef struct {
    int32_t knn_degree;       /* M: per-point list length (bucket2 --neighbors-m), 1..128 */
    int32_t nprobe;           /* neighbour buckets in a pool (bucket2 --nprobe; 0 = knn_k), <= 127 */
    int32_t knn_k;            /* bucket2 --knn-k: the pool width when nprobe is 0 (0 = 32) */
    int32_t rounds;           /* bucket2 -t: builds with seeds seed, seed+1, ... merged (0 or 1: one) */
    float centroid_ratio;     /* buckets = max(2, N * ratio) requested (bucket2 --centroid-ratio; 0 = 0.01) */
    int32_t assign_rule;      /* the balanced choice: 0 the reference's default (second centroid when its
                                 bucket is below 0.8 x the first's), 1 its BUCKET2_ASSIGN_RULE=diskjoin
                                 (second when its bucket is smaller and d2 < 1.2 d1) */
    uint64_t seed;
    int32_t out_on_device;    /* outputs are device pointers */
    int32_t reserved1;
    int32_t* assign_out;      /* optional N: the bucket of every point (last round) */
    int32_t* centroid_ids_out;/* optional: the centroids' point ids (room for max(2, N * ratio)) */
    int32_t* n_buckets_out;   /* optional HOST pointer: the number of buckets of the last round */
} gta_bucket2_params;

/* ---------------------------------------------------------------- pipeline */

/* Bucketed kNN graph: k-means over a sample, 2-way top-2 bucket membership,
 * all-pairs distances inside every bucket on the tensor cores, exact fp32
 * distances, per-bucket top-M, merge of each point's two lists.
 * Writes knn_ids[N x M] (int32, -1 padding, ascending distance) and, when
 * non-NULL, knn_dists[N x M] (squared L2, +inf padding).
 * Replaces bucket2's Steps 2-6 (bucketDemo/buildBucket/src/bucket.cu:8523
 * run_pipeline_impl, :5310 GpuResidentKnn::run_round, :5552 write_outputs). */
int gta_build_bucket(const gta_dataset* ds, const gta_bucket_params* p, int32_t* knn_ids, float* knn_dists,
                     void* stream);

/* kNN graph with the reference's own bucketing (gta_bucket2_params): KMeans||
 * (three rounds taking each point with probability 0.5 B d(x)^2 / psi, then a
 * uniform subsample of the candidates to B), exact centroid kNN graph, top-2
 * centroids of every point with the balanced choice (the second when its bucket
 * is below 0.8 x the first's size, each point against the sizes left by the
 * points before it in index order; assign_rule selects the diskjoin rule),
 * then for every bucket the exact top-M of its points over
 * the pool of its own and its nprobe nearest buckets' points (self excluded).
 * Writes knn_ids / knn_dists [N x M] like gta_build_bucket.
 * Replaces bucket2 Steps 2-6 on the GPU-resident path
 * (bucketDemo/buildBucket/src/bucket.cu:2833 select_centroids_on_gpu_kmeans_parallel,
 * :3241 centroid_self_knn_bf, :1552 batch_assign_with_cagra_anns, :5310 run_round). */
int gta_build_bucket2(const gta_dataset* ds, const gta_bucket2_params* p, int32_t* knn_ids, float* knn_dists,
                      void* stream);

/* CAGRA optimize of an already distance-sorted, sanitized (N x M) uint32 kNN
 * graph: rank-based detour-count prune to K, then the reverse-edge merge.
 * Replaces cuvs::neighbors::cagra::helpers::optimize(res, knn(N,M), out(N,K))
 * (bucketDemo/buildBucket/src/optimize.cu:396, bucket.cu:8470). */
int gta_optimize(const uint32_t* knn, int64_t n, int32_t m, int32_t k, uint32_t* graph, int32_t on_device,
                 void* stream);

/* The optimize tool's steps on an int32 kNN graph (-1 padding): sanitize, then
 * (when ds is non-NULL) the stable per-row sort by exact L2 distance to the
 * row's point, then gta_optimize's prune + reverse edges -> graph[N x K].
 * ds == NULL is --skip-sort (rows already ascending, e.g. bucket2's lists).
 * on_device says where knn and graph live (and must equal ds->on_device).
 * Replaces optimize's main, Steps 2-4 (bucketDemo/buildBucket/src/optimize.cu:
 * sanitize_to_uint32_inplace :95-133, sort_knn_graph_host, helpers::optimize
 * :396) and the first half of bucket2's fused_optimize_translate (bucket.cu:8434). */
int gta_optimize_knn(const gta_dataset* ds, const int32_t* knn, int64_t n, int32_t m, int32_t k, uint32_t* graph,
                     int32_t on_device, void* stream);

/* Whole build: gta_build_bucket, sanitize, gta_optimize -> graph[N x K]
 * (uint32).  Replaces bucket2 --fused-optimize-degree
 * (bucketDemo/buildBucket/src/bucket.cu:8434 fused_optimize_translate). */
int gta_build_cagra(const gta_dataset* ds, const gta_cagra_params* p, uint32_t* graph, void* stream);

/* ---------------------------------------------------------------- stages (device pointers) */

/* k-means: `iters` Lloyd steps from `centroids` (B x d, in/out) over the rows
 * X[n x d] (f32).  assign_out (optional, n) gets the final nearest centroid.
 * Replaces refine_centers_kmeans (bucketDemo/build_bucket.py:232-262). */
int gta_kmeans_fit(const float* X, int64_t n, int32_t d, float* centroids, int32_t B, int32_t iters,
                   int32_t* assign_out, void* stream);

/* k-means++ initial centroids (B x d) from a pool of the first pool_n rows of X.
 * Replaces kmeans_pp_centers (bucketDemo/build_bucket.py:189-229). */
int gta_kmeans_init(const float* X, int64_t pool_n, int32_t d, int32_t B, uint64_t seed, float* centroids,
                    void* stream);

/* Top-k nearest centroids per row (exact fp32 distances, ties -> smaller id).
 * Replaces topk_from_A_to_B(X, C, k) (bucketDemo/build_bucket.py:96-159) and
 * the Step-4 top-2 assignment (bucketDemo/buildBucket/src/bucket.cu:1230, :1478). */
int gta_assign_topk(const float* X, int64_t n, int32_t d, const float* C, int32_t B, int32_t k, int32_t* ids,
                    float* dists, void* stream);

/* The same with flags.  GTA_ROWS_INTEGER: every value of X is an integer of magnitude
 * below 2048 (8-bit data), which lets the tensor-core screen split the centroids into two
 * tf32-exact parts (error 2^-20 instead of 2^-9, far fewer exact reranks); a caller that sets
 * it for other rows gets undefined lists. */
#define GTA_ROWS_INTEGER 1
int gta_assign_topk_ex(const float* X, int64_t n, int32_t d, const float* C, int32_t B, int32_t k, int32_t* ids,
                       float* dists, int32_t flags, void* stream);

/* Bucket membership CSR from top-2 ids (n x 2): members[2n] point ids sorted
 * by (bucket, point), offsets[B+1], mem_row[n x 2] (membership row of each
 * point in its lower / higher bucket).
 * Replaces the CSR build of GpuResidentKnn::run_round (bucket.cu:5317-5357). */
int gta_build_memberships(const int32_t* top2, int64_t n, int32_t B, int32_t* members, int64_t* offsets,
                          int64_t* mem_row, void* stream);

/* Per-bucket all-pairs top-M (self excluded) for every membership row.
 * X: n x d rows of `dtype`; members/offsets: the CSR above (offsets on the
 * device).  list_ids/list_dists: [2n x M].
 * Replaces resident_gather_pool_kernel + cuBLAS dots + block_topK_from_dots_kernel
 * (bucket.cu:4920, :5471-5484, :4102) and the s6 screen + exact rerank (:4315-4688). */
int gta_bucket_knn(const void* X, int32_t dtype, int64_t n, int32_t d, const int32_t* members,
                   const int64_t* offsets, int32_t B, int32_t M, int32_t* list_ids, float* list_dists, void* stream);

/* Merge each point's two membership lists (mem_row from gta_build_memberships)
 * into out[n x M].  Replaces resident_merge_kernel (bucket.cu:5025-5131). */
int gta_merge_memberships(const int32_t* list_ids, const float* list_dists, const int64_t* mem_row, int64_t n,
                          int32_t M, int32_t* out_ids, float* out_dists, void* stream);

/* Merge two ascending M-lists per row (running first on equal distance, new
 * ids already present skipped).  Same rule as above, row-aligned inputs. */
int gta_merge_lists(const int32_t* run_ids, const float* run_dists, const int32_t* new_ids, const float* new_dists,
                    int64_t n, int32_t M, int32_t* out_ids, float* out_dists, void* stream);

/* int32 kNN (-1 padding) -> uint32 graph: padding / out-of-range / self ->
 * first valid neighbour of the row, else (i+1)%n.
 * Replaces sanitize_to_uint32_inplace (bucketDemo/buildBucket/src/optimize.cu:95-133). */
int gta_sanitize(const int32_t* knn, int64_t n, int32_t m, uint32_t* out, void* stream);

/* Stable per-row sort of candidates by exact distance to the row's point
 * (X: n x d f32).  Replaces sort_row_by_l2 (prune_windowed_core.hpp:134-175)
 * and optimize's sort_knn_graph_host. */
int gta_sort_rows(const float* X, int64_t n, int32_t d, const int32_t* knn, int32_t m, int32_t* out, void* stream);

/* Detour-count prune M -> K of a sanitized, sorted graph (no reverse edges).
 * Replaces compute_detour_counts + select_pruned_row
 * (prune_windowed_core.hpp:190-263) / prune_windowed_gpu::run (prune_windowed_gpu.hpp:15-21). */
int gta_prune(const uint32_t* knn, int64_t n, int32_t m, int32_t k, uint32_t* pruned, void* stream);

/* Reverse-edge merge of a pruned (n x K) graph into out (n x K).
 * Replaces TopKReverseStore + merge_rank_ordered_into_row
 * (edge_chunk_accumulator.hpp:386-494) / optimize_chunked -m E. */
int gta_reverse_merge(const uint32_t* pruned, int64_t n, int32_t k, uint32_t* out, void* stream);

/* Reverse-edge merge that allocates nothing: the same result as
 * gta_reverse_merge, for callers that cannot allocate device memory when they
 * call in -- for example a serving process whose allocator has reserved all of
 * device memory up front, or a latency-critical loop where a cudaMalloc /
 * cudaFree would synchronize the device and stall its other streams.  This
 * entry point has no counterpart in the reference.
 *
 * Its scratch is one fixed array inside the library (about 19 MB, held on every
 * GPU that loads the library until the process exits), so it accepts at most
 * gta_reverse_merge_noalloc_max_rows() rows (131072) and
 * gta_reverse_merge_noalloc_max_edges() edges (n * k <= 2097152, k <= 128) and
 * rejects anything larger with GTA_EINVAL.  The first call on a device looks up
 * the array's device address (cudaGetSymbolAddress); make that first call
 * before any stream capture.  All calls share the array: calls whose work
 * overlaps on the GPU (different streams, or several host threads) race and
 * must be serialized by the caller. */
int gta_reverse_merge_noalloc(const uint32_t* pruned, int64_t n, int32_t k, uint32_t* out, void* stream);
int64_t gta_reverse_merge_noalloc_max_rows(void);
int64_t gta_reverse_merge_noalloc_max_edges(void);

/* ---------------------------------------------------------------- graph search */

/* Best-first graph search of nq queries over `graph` (base->n x k_graph uint32
 * ids): the rule of bucketDemo/search.py:20-93 graph_search_single -- the
 * entry points of each query (n_entry per query, ascending, -1 = unused; the
 * reference draws them with numpy's default_rng(42) and np.unique, see
 * gta.search_entries) are visited in order, the (distance, id)-smallest
 * candidate is expanded until its distance exceeds the worst of a full
 * ef-entry best list, the best list is appended while short and otherwise
 * its first maximum is replaced by a smaller distance.  Writes the topk
 * nearest of the best list per query (ascending distance, ties by id; -1 / +inf
 * padding).  Queries have base's dtype and d; base->on_device says whether all
 * arrays are device (stream-ordered) or host (synchronous) memory.  One warp
 * per query; 1 <= topk <= ef <= 256, d <= 1024.  Status 2 when a query visits
 * more nodes than the per-query visited set holds (12 288): lower ef. */
int gta_search(const gta_dataset* base, const void* queries, int64_t nq, const uint32_t* graph, int32_t k_graph,
               const int32_t* entries, int32_t n_entry, int32_t topk, int32_t ef, int32_t* out_ids, float* out_dists,
               void* stream);

/* ---------------------------------------------------------------- bucket-contiguous renumbering
 * bucket2 renumbers the points after the first round so that every bucket is a
 * contiguous id range (data_reordered.<ext>, inverse_perm.bin[new] = old), runs
 * the rest of the pipeline in that id space and translates the final graph back
 * (translate_ids).  Every entry takes an on_device flag: 1 = all arrays are
 * device pointers (stream-ordered), 0 = host arrays (synchronous). */

/* Processing order of B buckets (order[pos] = bucket): exact kNN graph of the
 * centroids (B x d f32, self excluded, k <= 127 columns, written to centroid_knn
 * when non-NULL, ties to the smaller id), then the greedy windowed order of
 * bucket_order.hpp:143-200 over it (window <= 0: max(4k, 16), bucket.cu:9023-9025).
 * Replaces bucket2 Step 3 (centroid_self_knn_bf, bucket.cu:3241) + the order. */
int gta_bucket_order(const float* centroids, int32_t B, int32_t d, int32_t k, int32_t window, int32_t* order,
                     int32_t* centroid_knn, int32_t on_device, void* stream);

/* New ids bucket by bucket in `order` (NULL: 0..B-1), ascending old id inside a
 * bucket: inverse_perm[new] = old (n), offsets[pos] = first new id of bucket
 * order[pos] (B+1, may be NULL).  The bucket of point i is assign[i * stride]
 * (stride 2 reads column 0 of a top-2 table).  Status 5 when a point has no
 * valid bucket or order is not a permutation.
 * Replaces compute_bucket_reorder (bucketDemo/buildBucket/src/bucket.cu:8356-8417). */
int gta_bucket_reorder(const int32_t* assign, int64_t n, int32_t stride, int32_t B, const int32_t* order,
                       uint32_t* inverse_perm, int64_t* offsets, int32_t on_device, void* stream);

/* out row i = X row inverse_perm[i] (n rows of row_bytes bytes): the reordered
 * dataset (bucket.cu:9253-9403, data_reordered.<ext>). */
int gta_permute_rows(const void* X, int64_t n, int64_t row_bytes, const uint32_t* inverse_perm, void* out,
                     int32_t on_device, void* stream);

/* Renumber an n x m graph.  to_original = 1: rows and ids from the reordered id
 * space back to the original one, out[inv[i]][j] = inv[g[i][j]]
 * (translate_graph_ids.hpp:75-200, the translate_ids tool); to_original = 0: the
 * other way, out[i][j] = perm[g[inv[i]][j]] with perm = inverse of inv.
 * keep_padding = 1 keeps negative ids as -1 (the .npy path); otherwise they are
 * an error like any id >= n.  Status 5 on a bad id or when inverse_perm is not a
 * permutation of [0, n). */
int gta_permute_graph(const int32_t* g, int64_t n, int32_t m, const uint32_t* inverse_perm, int32_t to_original,
                      int32_t keep_padding, int32_t* out, int32_t on_device, void* stream);

/* ---------------------------------------------------------------- shard stages
 * One rank's part of the multi-GPU build (the plan of the reference's
 * multi-GPU design: row-sharded k-means with all-reduced sums, buckets placed
 * on owner GPUs, points and lists exchanged all-to-all, the id table gathered
 * for the prune).  A rank holds global rows [row0, row0 + n_local) of an
 * N-row dataset; every id below is global.  The collectives between these
 * calls belong to the caller (torch.distributed / NCCL).  Device pointers,
 * stream-ordered. */

/* The sizes the build derives from N and its parameters: the k-means sample
 * (min(0.1, 1e7/N) of N unless p->kmeans_sample is set, at least B), the
 * k-means++ pool (min(sample, 20 B)) and the seed of the pool's draw. */
int gta_kmeans_sizes(int64_t n, const gta_bucket_params* p, int64_t* n_sample, int64_t* pool_n, uint64_t* pool_seed);

/* n_s ids drawn from [0, n), one uniformly from each of n_s equal strata
 * (ascending).  The build's k-means sample and k-means++ pool; stands in for
 * torch.randperm(N)[:pool_n] (bucketDemo/build_bucket.py:207). */
int gta_sample_ids(int64_t n, int64_t n_s, uint64_t seed, int32_t* ids, void* stream);

/* out[j] (d f32 values) = row ids[j] - row0 of the shard X (n rows of dtype),
 * or zeros where ids[j] is outside [row0, row0 + n): summing every rank's
 * output gives the rows of all ids. */
int gta_gather_rows(const void* X, int32_t dtype, int64_t n, int32_t d, int64_t row0, const int32_t* ids,
                    int64_t n_ids, float* out, void* stream);

/* Lloyd partials of a shard: per centroid the fp64 sum of its rows (B x d)
 * and their count (B).  After an all-reduce (sum) over ranks,
 * gta_centroid_means turns them into the new centroids in place (a centroid
 * with no rows keeps its value).  Replaces the scatter_add_ / bincount /
 * divide of refine_centers_kmeans (bucketDemo/build_bucket.py:252-259). */
int gta_centroid_sums(const float* X, int64_t n, int32_t d, const int32_t* assign, int32_t B, double* sums,
                      int64_t* counts, void* stream);
int gta_centroid_means(const double* sums, const int64_t* counts, int32_t B, int32_t d, float* centroids, void* stream);

/* Received memberships (bucket, other bucket) grouped by (bucket, other),
 * stable: order[n] lists them in that order, offsets[B+1] per bucket.  When
 * every rank sends its memberships in row order and they arrive in rank order,
 * this is the order of gta_build_memberships. */
int gta_group_memberships(const int32_t* bucket, const int32_t* other, int64_t n, int32_t B, int32_t* order,
                          int64_t* offsets, void* stream);

/* gta_bucket_knn over rows that were sent to this rank: R holds the n received
 * rows in arrival order, order/offsets come from gta_group_memberships, gid[n]
 * is each received row's global id.  List j (of [n x M]) belongs to received
 * row order[j] and holds global ids. */
int gta_bucket_knn_rows(const void* R, int32_t dtype, int64_t n, int32_t d, const int32_t* order, const int32_t* gid,
                        const int64_t* offsets, int32_t B, int32_t M, int32_t* list_ids, float* list_dists,
                        void* stream);

/* gta_bucket_knn_rows in two passes (the sharded build's seeded higher-bucket rows).
 * partner[j] is the other bucket of grouped row j (rows grouped by (bucket, partner) as
 * gta_group_memberships orders them).  phase 1 writes the rows whose partner is above their
 * bucket (the points' lower-bucket lists); phase 2 writes the others, each starting from the
 * bound seed[gid] (by global id: the point's lower-bucket list's m-th distance, +inf when
 * unknown) and skipping the columns whose partner equals the row's (points already in the lower
 * list).  Merged with gta_merge_memberships, the lists equal those of gta_bucket_knn_rows.
 * For shapes without seeded rows (f32 data, lists longer than 64) phase 1 writes every row and
 * phase 2 none.  list_ids / list_dists: rows of the other phase are left as they are.
 * Replaces the same interface as gta_bucket_knn_rows. */
int gta_bucket_knn_rows_phased(const void* R, int32_t dtype, int64_t n, int32_t d, const int32_t* order,
                               const int32_t* gid, const int64_t* offsets, const int32_t* partner, int32_t B, int32_t M,
                               int32_t phase, const float* seed, int32_t* list_ids, float* list_dists, void* stream);

/* gta_bucket_knn_rows_phased restricted to row ranges: only grouped rows
 * [offsets[b] + row_lo[b], offsets[b] + row_hi[b]) of bucket b get lists (row_lo, row_hi: HOST
 * arrays [B], 0 <= row_lo[b] <= row_hi[b] <= the bucket's size); every row of the bucket stays a
 * column.  Other rows of list_ids / list_dists are left as they are.  The sharded build's split
 * buckets: each rank that shares a bucket holds all its rows and fills a disjoint range, so the
 * ranges' lists together equal the bucket's lists of gta_bucket_knn_rows_phased.  Returns
 * GTA_EINVAL for a range outside its bucket.  Extends the interface gta_bucket_knn_rows
 * replaces (the per-bucket kNN of one bucket's memberships, multi-GPU: one bucket on several
 * devices). */
int gta_bucket_knn_rows_ranged(const void* R, int32_t dtype, int64_t n, int32_t d, const int32_t* order,
                               const int32_t* gid, const int64_t* offsets, const int32_t* partner, int32_t B, int32_t M,
                               int32_t phase, const float* seed, const int64_t* row_lo, const int64_t* row_hi,
                               int32_t* list_ids, float* list_dists, void* stream);

/* The sharded build's packing for its all-to-all exchanges (device pointers, one stream).
 * Items go to ranks by a stable multi-destination partition: rank by rank, in item order.
 *
 * gta_shard_pack_memberships: membership m = 2p + s (local point p, slot s of top2[p]) goes to
 * every rank r whose bit is set in holders[top2[m]] (device uint64 [B]: the ranks holding a piece
 * of the bucket; world <= 64).  send_counts (HOST [world]) receives the items per rank; with
 * send_rows and send_meta null only the counts are computed (size the buffers, then call again).
 * Otherwise item k of the packed order gets row p of X (n_local rows of d elements of dtype) in
 * send_rows[k] and (row0 + p, top2[m], top2[m ^ 1]) in send_meta[3k..3k+2]; capacity = rows the
 * buffers hold.  A bucket outside [0, B), or one without a holder, returns GTA_EDATA.
 * Replaces the reference's point exchange to bucket owners (bucket.cu multi-GPU plan: points to
 * the GPUs that own their buckets). */
int gta_shard_pack_memberships(const void* X, int32_t dtype, int64_t n_local, int32_t d, int64_t row0,
                               const int32_t* top2, int32_t B, const uint64_t* holders, int32_t world,
                               int64_t* send_counts, void* send_rows, int32_t* send_meta, int64_t capacity,
                               void* stream);

/* gta_shard_pack_lists: the lists a rank computed go back to their points' owners.  Grouped row j
 * (list_ids / list_dists [n x M], order / gid / offsets as for gta_bucket_knn_rows_ranged) is sent
 * when it lies in [row_lo[b], row_hi[b]) of its bucket b (HOST arrays [B]), to the rank r with
 * starts[r] <= gid[order[j]] < starts[r + 1] (HOST [world + 1]).  Packed as send_ids / send_dists
 * [k x M] and send_meta [k x 2] = (global id, bucket); counts and the null-buffer call as above.
 * Replaces the reference's list exchange back to the points' GPUs before the merge. */
int gta_shard_pack_lists(const int32_t* list_ids, const float* list_dists, int64_t n, int32_t M, const int32_t* order,
                         const int32_t* gid, const int64_t* offsets, int32_t B, const int64_t* row_lo,
                         const int64_t* row_hi, const int64_t* starts, int32_t world, int64_t* send_counts,
                         int32_t* send_ids, float* send_dists, int32_t* send_meta, int64_t capacity, void* stream);

/* gta_shard_member_rows: for received lists i (meta [n x 2] = (global id, bucket)) of this rank's
 * rows [row0, row0 + n_local) with buckets top2 [n_local x 2]: mem_row[2p + slot] = i, slot 0 for
 * the lower of the point's two buckets, -1 where no list arrived (the input of
 * gta_merge_memberships).  An id outside the rows, or a bucket not among the point's two, returns
 * GTA_EDATA. */
int gta_shard_member_rows(const int32_t* meta, int64_t n, int64_t row0, int64_t n_local, const int32_t* top2,
                          int64_t* mem_row, void* stream);

/* gta_shard_lower_seeds: seed[N] = +inf, then for every grouped row j in this rank's ranges
 * (row_lo / row_hi HOST [B]) whose bucket is below its partner: seed[gid[order[j]]] =
 * list_dists[j][M-1] (the point's lower-bucket M-th distance; the ranks' seeds are then
 * all-reduced with min before phase 2 of gta_bucket_knn_rows_ranged). */
int gta_shard_lower_seeds(const float* list_dists, int32_t M, int64_t n, const int32_t* order, const int32_t* gid,
                          const int64_t* offsets, const int32_t* partner, int32_t B, const int64_t* row_lo,
                          const int64_t* row_hi, int64_t N, float* seed, void* stream);

/* gta_sanitize for rows [row0, row0 + n_rows) of an n-row graph (knn and out
 * hold only those rows). */
int gta_sanitize_rows(const int32_t* knn, int64_t n_rows, int64_t row0, int64_t n, int32_t m, uint32_t* out,
                      void* stream);

/* gta_prune for rows [row0, row0 + n_rows) of the whole n x m graph knn;
 * pruned holds those rows (n_rows x k).  top2 (n_rows x 2, may be NULL) sets
 * the processing order only (rows grouped by their buckets for locality). */
int gta_prune_rows(const uint32_t* knn, int64_t n, int32_t m, int32_t k, int64_t row0, int64_t n_rows,
                   const int32_t* top2, int32_t B, uint32_t* pruned, void* stream);

/* gta_reverse_merge for destination rows [row0, row0 + n_rows) of the whole
 * n x k pruned graph; out holds those rows. */
int gta_reverse_merge_rows(const uint32_t* pruned, int64_t n, int32_t k, int64_t row0, int64_t n_rows, uint32_t* out,
                           void* stream);

/* ---------------------------------------------------------------- files (host) */

/* BIGANN dataset header (int32 N, int32 D); dtype from the extension
 * (.fbin/.bin -> F32, .u8bin -> U8, .i8bin -> I8).  load.hpp:43-135. */
int gta_read_dataset_header(const char* path, int64_t* n, int32_t* d, int32_t* dtype);
/* rows [row0, row0 + nrows) into out (nrows x d elements of the file's dtype). */
int gta_read_dataset(const char* path, int64_t row0, int64_t nrows, void* out);
int gta_write_dataset(const char* path, const void* data, int64_t n, int32_t d, int32_t dtype);

/* vector_knn.bin: int64 N, int32 M, int32[N*M] (-1 padding).  graph_io.hpp:26-30, bucket.cu:8311. */
int gta_write_knn(const char* path, const int32_t* ids, int64_t n, int32_t m);
int gta_read_knn_header(const char* path, int64_t* n, int32_t* m);
int gta_read_knn(const char* path, int32_t* ids);
/* vector_dists.bin: same header, float32 payload. */
int gta_write_knn_dists(const char* path, const float* dists, int64_t n, int32_t m);

/* CAGRA / final graph: int64 N, int32 K, uint32[N*K].  graph_io.hpp:8-11, optimize.cu:20-24. */
int gta_write_graph(const char* path, const uint32_t* graph, int64_t n, int32_t k);
int gta_read_graph_header(const char* path, int64_t* n, int32_t* k);
int gta_read_graph(const char* path, uint32_t* graph);

/* neighbors.npy: int64 (N, M) numpy array (load.hpp:535-618).  The reader takes
 * a C-order little-endian int64 2-D array and narrows it to int32 (values must
 * lie in [-1, 2^31); -1 = padding); status 5 otherwise. */
int gta_write_npy_i64(const char* path, const int32_t* ids, int64_t n, int32_t m);
int gta_read_npy_i64_header(const char* path, int64_t* n, int32_t* m);
int gta_read_npy_i64(const char* path, int32_t* ids);

/* Raw uint32 arrays without a header (inverse_perm.bin, bucket.cu:9445). */
int gta_write_u32(const char* path, const uint32_t* v, int64_t n);
int gta_read_u32_count(const char* path, int64_t* n);
int gta_read_u32(const char* path, uint32_t* v);

/* ---------------------------------------------------------------- profiling */
/* Per-stage CUDA-event timing inside the library (off by default).  Enabling
 * (or disabling) clears the records.  Each record: stage name, elapsed ms on
 * the stream its kernels ran on, and the stage's algorithmic work (flops for
 * the distance GEMM stages "dist_topk_*", bytes for the others). */
int gta_profile_enable(int32_t on);
int gta_profile_count(void);
int gta_profile_get(int32_t i, char* name, int32_t name_len, float* ms, double* units);
/* Device counters of profile record i (the distance kernel: passes into the row
 * lists, warp-wide list merges, rows); fills n values, zeros past the record's count. */
int gta_profile_counters(int32_t i, double* out, int32_t n);
/* Number of this library's own kernel launches since it was loaded. */
long long gta_launch_count(void);

/* ---------------------------------------------------------------- misc */
/* Free and total memory of the current device (bytes), for callers' fit checks
 * (the optimize tool's --gpu-fit-margin test, optimize.cu:243-251). */
int gta_device_memory(int64_t* free_bytes, int64_t* total_bytes);
/* Free the per-(device, stream) workspaces (synchronizes those streams). */
int gta_release_workspace(void);
const char* gta_last_error(void);
const char* gta_version(void);

#ifdef __cplusplus
}
#endif

#endif /* GTA_H_ */
