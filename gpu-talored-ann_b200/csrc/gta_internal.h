// gta_internal.h -- host-side internal interface of libgta (not part of the C ABI).
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#include <cuda_runtime.h>

namespace gta {

// Status codes of the C ABI (see include/gta.h).
enum : int { kOk = 0, kInvalid = 1, kNoMem = 2, kCuda = 3, kNccl = 4, kData = 5 };

struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

#define GTA_CUDA(call)                                                                                     \
    do {                                                                                                   \
        cudaError_t e_ = (call);                                                                           \
        if (e_ != cudaSuccess)                                                                             \
            throw ::gta::Error(e_ == cudaErrorMemoryAllocation ? ::gta::kNoMem : ::gta::kCuda,             \
                               std::string("CUDA error: ") + cudaGetErrorString(e_) + " at " __FILE__ ":" + \
                                   std::to_string(__LINE__));                                              \
    } while (0)

#define GTA_REQUIRE(cond, code, msg)                 \
    do {                                             \
        if (!(cond)) throw ::gta::Error(code, msg);  \
    } while (0)

// Device scratch of one library call.  Inside a top-level entry point
// (WorkspaceScope), buffers come from a per-(device, stream) arena that is
// reused by every later call on that stream: the arena grows to the call's
// high-water mark once and is then served without any allocation.  Outside a
// scope, or when the arena is too small, the stream-ordered allocator is used.
void* workspace_alloc(size_t bytes, cudaStream_t st, bool* from_arena);

class WorkspaceScope {
public:
    explicit WorkspaceScope(cudaStream_t st);
    ~WorkspaceScope();
    WorkspaceScope(const WorkspaceScope&) = delete;
    WorkspaceScope& operator=(const WorkspaceScope&) = delete;

private:
    bool active_ = false;
};

template <typename T>
struct DevBuf {
    T* p = nullptr;
    size_t n = 0;
    cudaStream_t st = nullptr;
    bool arena = false;
    DevBuf() = default;
    DevBuf(size_t count, cudaStream_t s) : n(count), st(s)
    {
        if (count) p = static_cast<T*>(workspace_alloc(sizeof(T) * count, s, &arena));
    }
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    DevBuf(DevBuf&& o) noexcept : p(o.p), n(o.n), st(o.st), arena(o.arena) { o.p = nullptr; o.n = 0; }
    DevBuf& operator=(DevBuf&& o) noexcept
    {
        release();
        p = o.p; n = o.n; st = o.st; arena = o.arena; o.p = nullptr; o.n = 0;
        return *this;
    }
    ~DevBuf() { release(); }
    void release()
    {
        if (p && !arena) cudaFreeAsync(p, st);
        p = nullptr;
        n = 0;
    }
    T* get() const { return p; }
};

// One CTA of the distance kernel: a tile of up to 128 A rows against a
// contiguous segment of B rows (all columns of one bucket, or all centroids).
struct WorkItem {
    int32_t a_row0;     // first A row of the tile
    int32_t a_rows;     // valid rows in the tile (1..128)
    int32_t b_row0;     // first B row of the segment
    int32_t b_rows;     // segment length (columns)
    int32_t self_col0;  // segment column of the tile's row 0 itself (self excluded), or -1
    int32_t item_row0;  // float screen only: the item's first row of candidate lists and outputs
    int32_t has_self;   // float screen only: A row r is column self_col0 + r (when in range)
    int32_t pad2;
};

// operand rows of the distance kernel: bf16 (8-bit data held exactly, kind::f16), f32 (tf32
// screen + exact rerank), u8 (the dataset's own bytes, kind::i8)
enum ElemType : int { kElemBF16 = 0, kElemF32 = 1, kElemU8 = 2 };
inline int elem_bytes(int elem) { return elem == kElemU8 ? 1 : elem == kElemBF16 ? 2 : 4; }

// Row-wise top-k of squared L2 distances between A rows and a B segment.
struct DistTopkProblem {
    const void* A = nullptr;       // [a_total x d_pad] bf16 or f32, rows 128-B multiples
    int64_t a_total = 0;
    const void* B = nullptr;       // [b_total x d_pad]
    int64_t b_total = 0;
    int elem = kElemF32;           // bf16: exact integer data (kind::f16); f32: tf32 screen + exact rerank
    int d = 0, d_pad = 0;
    const float* a_norm = nullptr; // [a_total] exact ||a||^2
    const float* b_norm = nullptr; // [b_total] exact ||b||^2
    const int32_t* b_gid = nullptr;// [b_total] output id of a B row (null: segment column)
    const WorkItem* work = nullptr;// device work list
    int n_work = 0;
    int m_out = 0;                 // list length written per A row
    bool exclude_self = false;
    int32_t* out_ids = nullptr;    // [a_total x m_out]
    float* out_dists = nullptr;
    int* err = nullptr;            // device error word
    const char* prof_name = "dist_topk";
    double flops = 0.0;            // algorithmic flops of the launch (sum of 2*rows*cols*d)
    // screen error model (tf32): relative operand-truncation error of the dot products and the
    // number of products accumulated; split operands (integer rows [x | x] against centroid rows
    // [hi | lo], both parts exact in tf32) cut the truncation term from 2^-9 to 2^-19
    double screen_trunc = 0x1p-9;
    int screen_k = 0;              // 0: d
    // rows the exact rerank reads for B (default B / d_pad): the unsplit centroids
    const void* b_exact = nullptr;
    int b_exact_pitch = 0;
    // seeded rows (exact data, lists of at most 64): each A row starts from the threshold
    // seed[gid * seed_stride] - ||a||^2 (gid = b_gid of the row; seed: a distance already known to
    // bound the row's merged list) and drops the columns whose partner[] equals the row's own
    // partner[] (points already seen through the row's other membership); null: no seeding
    const float* seed = nullptr;
    int64_t seed_stride = 1;
    const int32_t* partner = nullptr;  // [a_total] (A and B rows are the same pool)
};

void dist_topk(const DistTopkProblem& pr, cudaStream_t st);

// Float-row per-bucket kNN (screen.cu): pool row j is dataset row ids[j] (X: n x d rows of
// dtype, dense); the pool is grouped into segments (buckets, in processing order) and every row
// of a segment gets its exact top-m_out (fp32 chain) over the segment's rows (itself excluded),
// written with output ids gid[] into row j of out_ids / out_dists.  A tensor-core screen on fp16
// parts of the scaled rows keeps every column within a proven margin of the row's M-th; an exact
// rerank over the pool's f32 rows picks the list.  `parts` = 2 stores hi and lo parts (the split
// screen; rows with d >= 256 start on the hi part alone and return to the split in a wave that
// rescans too many rows), 1 the hi part only.  Segments longer than an L2-sized column chunk run
// as chunk waves whose exact lists are merged.
struct ScreenProblem {
    const void* X = nullptr;
    int dtype = 0;                  // GTA_F32 / GTA_U8 / GTA_I8 (include/gta.h)
    int d = 0;
    const int32_t* ids = nullptr;   // [n_rows] pool row -> dataset row
    const int32_t* gid = nullptr;   // [n_rows] pool row -> output id
    int64_t n_rows = 0;
    std::vector<int64_t> seg_lo, seg_n;  // segments: first pool row and length
    std::vector<int64_t> seg_r0, seg_r1; // rows [r0, r1) of each segment get lists (empty: all)
    int m_out = 0;
    int parts = 2;
    int32_t* out_ids = nullptr;     // [n_rows x m_out]
    float* out_dists = nullptr;
    int* err = nullptr;
    const char* prof_name = "dist_topk_bucket";
};
void screen_knn(const ScreenProblem& pr, cudaStream_t st);
int screen_list_len(int m);
// true when dist_topk accepts seeded rows for this shape (exact data, two-CTA variant)
bool dist_topk_seedable(int elem, int d_pad, int m_out);
// true when 8-bit operand rows (kElemU8, rows padded to 128 bytes) run for this list length
bool dist_topk_u8_fits(int d_pad, int m_out);

// ---- other kernels (kernels.cu) -------------------------------------------
// Convert rows of X (dtype: 0 f32, 1 u8, 2 i8) selected by row_ids (null = identity)
// into a padded bf16 or f32 matrix, with exact fp32 squared norms.
void convert_rows(const void* X, int dtype, int d, const int32_t* row_ids, int64_t n_out, void* out, int out_elem,
                  int d_pad, float* norms, cudaStream_t st);
void sample_ids(int64_t N, int64_t n_s, uint64_t seed, int32_t* out, cudaStream_t st);
void kmeanspp_init(const float* pool, const float* pool_norm, int64_t pool_n, int d, int d_pad, int32_t B,
                   uint64_t seed, float* centroids, int* err, cudaStream_t st);
// integer_rows: every row value is an integer (8-bit data), so the fp64 sums may be formed in
// any order (exact); otherwise they are accumulated in ascending point order
void centroid_update(const float* Xs, int64_t n_s, int d, int d_pad, const int32_t* assign, const float* C_in,
                     int32_t B, float* C_out, float* C_norm, int* err, cudaStream_t st, bool integer_rows = false);
void check_ids(const int32_t* ids, int64_t n, int32_t hi, int* err, cudaStream_t st);
// Memberships grouped by bucket, within a bucket by the point's other bucket (its partner),
// then by point.  split (optional, [B]): first membership of each bucket whose partner is above
// the bucket (before it: the points for which the bucket is the higher of the two); partner
// (optional, [2N]): the other bucket of each membership's point.
void build_memberships(const int32_t* top2, int64_t N, int32_t B, int32_t* members, int64_t* offsets,
                       int64_t* mem_row, int* err, cudaStream_t st, int64_t* split = nullptr,
                       int32_t* partner = nullptr);
// split[b] = first of bucket b's grouped rows (offsets) whose partner is above b; the rows of a
// bucket ascend by partner
void split_from_partner(const int32_t* partner, const int64_t* offsets, int32_t B, int64_t* split, cudaStream_t st);
// seed[p] = the M-th distance of point p's lower-bucket list (rows j0 .. j0 + n_rows of the
// list buffer, +inf when that row is elsewhere)
void seeds_from_lists(const float* list_d, const int64_t* mem_row, int64_t N, int M, int64_t j0, int64_t n_rows,
                      float* seed, cudaStream_t st);
void merge_memberships(const int32_t* list_n, const float* list_d, const int64_t* mem_row, int64_t N, int M,
                       int32_t* out_n, float* out_d, cudaStream_t st);
// membership rows j0 .. j0 + n - 1 (their lists in bl / bd) into the per-point lists, first memberships
// copied, second ones merged (the order of merge_memberships)
// passes: bit 0 copies the batch's lower-bucket lists, bit 1 merges its higher-bucket lists
void merge_membership_batch(const int32_t* bl, const float* bd, const int32_t* members, const int64_t* mem_row,
                            int64_t j0, int64_t n, int64_t N, int M, int32_t* out_n, float* out_d, cudaStream_t st,
                            int passes = 3);
void merge_lists(const int32_t* run_n, const float* run_d, const int32_t* new_n, const float* new_d, int64_t N,
                 int M, int32_t* out_n, float* out_d, cudaStream_t st);
void sanitize(const int32_t* knn, int64_t N, int M, uint32_t* out, cudaStream_t st);
void prune_detour(const uint32_t* g, int64_t N, int M, int K, const int32_t* order, uint32_t* out, int* err,
                  cudaStream_t st);
void locality_order(const int32_t* top2, int64_t N, int32_t B, int32_t* order, cudaStream_t st);
void reverse_merge(const uint32_t* pruned, int64_t N, int K, uint32_t* out, int* err, cudaStream_t st);
void reverse_merge_noalloc(const uint32_t* pruned, int64_t N, int K, uint32_t* out, cudaStream_t st);
int64_t reverse_merge_noalloc_max_rows();
int64_t reverse_merge_noalloc_max_edges();
void sort_rows_l2(const float* X, int d, int d_pad, const int32_t* knn, int64_t N, int M, int32_t* out,
                  cudaStream_t st);
void max_sqrt(const float* v, int64_t n, float* out, cudaStream_t st);
// best-first graph search, one warp per query (search.cu)
void graph_search(const void* base, int dtype, int64_t n, int d, const uint32_t* graph, int kg, const void* queries,
                  int64_t nq, const int32_t* entries, int ne, int topk, int ef, int32_t* out_ids, float* out_dists,
                  int* err, cudaStream_t st);
// exact assignment to few centroids on the FP32 pipe (assign.cu); X rows of `dtype` with row
// stride ldx elements, centroids f32 with row stride ldc
constexpr int kAssignExactMaxB = 384;
bool assign_exact_applies(int B, int k);
// (row_ids: row of X for each point, null = identity)
void assign_exact(const void* X, int dtype, int64_t n, int ldx, int d, const int32_t* row_ids, const float* C, int ldc,
                  int B, int k, int32_t* ids, float* dists, cudaStream_t st);
// reference-bucketing build (bucket2.cu): splitmix64 streams shared with the oracle
__host__ __device__ __forceinline__ uint64_t mix64(uint64_t x)
{
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
// 53 random bits for point i in KMeans|| round r (u = bits * 2^-53)
__host__ __device__ __forceinline__ uint64_t kpar_uniform_bits(uint64_t seed, int round, uint64_t i)
{
    return mix64(seed * 0x9E3779B97F4A7C15ull + 0xD1B54A32D192ED03ull * static_cast<uint64_t>(round + 1) + i) >> 11;
}
constexpr int64_t kKparPsiTarget = 16384;  // psi subsample size (bucket.cu:2999)
void kpar_psi(const float* min_d, int64_t n, double* psi, cudaStream_t st);
void kpar_sample(const float* min_d, int64_t n, uint64_t seed, int round, double lk, const double* psi, uint8_t* chosen,
                 uint8_t* sel, cudaStream_t st);
int64_t select_flagged(const uint8_t* flags, int64_t n, int32_t* out, cudaStream_t st);  // ids in order; syncs
void min_update(float* min_d, const float* d_new, int64_t n, cudaStream_t st);
// ---- sharded build (shard.cu): the exchanges' packing
// perm: for each rank in turn, the items whose mask carries the rank's bit, in item order;
// counts[r] (host) the number of items for rank r.
void stable_partition(const uint64_t* masks, int64_t n, int world, DevBuf<int64_t>& perm, std::vector<int64_t>& counts,
                      cudaStream_t st);
struct ShardPackMem {
    const void* X;            // n_local rows of row_bytes bytes (this rank's dataset rows)
    int64_t n_local, row_bytes, row0;
    const int32_t* top2;      // [n_local x 2]: the two buckets of every local point
    int32_t B, world;
    const uint64_t* holders;  // [B]: bit r set when rank r holds a piece of the bucket
    void* send_rows;          // null: counts only
    int32_t* send_meta;       // [total x 3]: (global id, bucket, other bucket)
    int64_t capacity;         // rows the send buffers hold
    int* err;
};
void shard_pack_memberships(const ShardPackMem& a, std::vector<int64_t>& counts, cudaStream_t st);
struct ShardPackLists {
    const int32_t* lid;       // [n_r x M] lists of the grouped received rows
    const float* ldist;
    int64_t n_r;
    int32_t M;
    const int32_t* order;     // grouped row j = received row order[j]
    const int32_t* gid;       // [n_r] global id of every received row
    const int64_t* offsets;   // [B + 1] grouped rows of each bucket
    int32_t B, world;
    const int64_t* row_lo;    // host [B]: this rank's row range of each bucket
    const int64_t* row_hi;
    const int64_t* starts;    // host [world + 1]: rank r owns global rows [starts[r], starts[r+1])
    int32_t* send_ids;        // null: counts only
    float* send_dists;
    int32_t* send_meta;       // [total x 2]: (global id, bucket)
    int64_t capacity;
    int* err;
};
void shard_pack_lists(const ShardPackLists& a, std::vector<int64_t>& counts, cudaStream_t st);
void shard_member_rows(const int32_t* meta, int64_t n_b, int64_t row0, int64_t n_local, const int32_t* top2,
                       int64_t* mem_row, int* err, cudaStream_t st);
void shard_lower_seeds(const float* ldist, int32_t M, int64_t n_r, const int32_t* order, const int32_t* gid,
                       const int64_t* offsets, const int32_t* partner, int32_t B, const int64_t* row_lo_h,
                       const int64_t* row_hi_h, int64_t N, float* seed, int* err, cudaStream_t st);

void balanced_assign(const int32_t* top2, const float* top2_d, int rule, const int32_t* cid, int32_t n_c, int64_t n,
                     int32_t* assign, int* err, cudaStream_t st);
void pool_fill(const int32_t* members, const int64_t* offsets, const int32_t* seg_b, const int64_t* seg_dst, int32_t S,
               int32_t c_lo, int32_t n_buckets, int32_t* pool_ids, cudaStream_t st);
void one_way_rows(const int32_t* members, int64_t n, int64_t* mem_row, cudaStream_t st);
// order = 0..n-1 sorted stably by key (keys in [0, B), else err), offsets[b] = first index of key b
void group_by_key(const int32_t* keys, int64_t n, int32_t B, int32_t* order, int64_t* offsets, int* err, cudaStream_t st);
// split operands for the tf32 screen of integer-valued rows against f32 centroids (assign.cu):
// rows [x | x | 0] and centroid rows [hi | lo | 0] of pitch `pitch` (>= 2d, 32-float multiple)
void dup_rows(const float* X, int d, int ld, int64_t n, float* out, int pitch, cudaStream_t st);
void split_rows_tf32(const float* C, int d, int ld, int64_t n, float* out, int pitch, cudaStream_t st);
// bucket-contiguous renumbering (reorder.cu)
void bucket_reorder(const int32_t* assign, int64_t n, int32_t stride, int32_t B, const int32_t* order,
                    uint32_t* inverse_perm, int64_t* offsets, int* err, cudaStream_t st);
void permute_rows(const void* X, int64_t n, int64_t row_bytes, const uint32_t* inverse_perm, void* out, int* err,
                  cudaStream_t st);
void permute_graph(const int32_t* g, int64_t n, int32_t m, const uint32_t* inverse_perm, bool to_original,
                   bool keep_padding, int32_t* out, int* err, cudaStream_t st);
void bucket_order(const int32_t* adj, int32_t B, int32_t K, int32_t window, int32_t* order);  // host
// shard variants (one rank's part of a multi-GPU build)
void gather_range(const void* X, int dtype, int d, int64_t row0, int64_t n, const int32_t* ids, int64_t n_ids,
                  float* out, cudaStream_t st);
void gather_i32(const int32_t* src, const int32_t* idx, int64_t n, int32_t* out, cudaStream_t st);
void centroid_partial(const float* Xs, int64_t n_s, int d, int d_pad, const int32_t* assign, int32_t B, double* sums,
                      long long* counts, int* err, cudaStream_t st);
void centroid_means(const double* sums, const long long* counts, const float* C_in, int32_t B, int d, float* C_out,
                    cudaStream_t st);
void group_rows(const int32_t* bucket, const int32_t* other, int64_t n, int32_t B, int32_t* order, int64_t* offsets,
                cudaStream_t st);
void sanitize_rows(const int32_t* knn, int64_t n_rows, int64_t row0, int64_t N, int M, uint32_t* out, cudaStream_t st);
void prune_rows(const uint32_t* g, int64_t N, int M, int K, const int32_t* order, int64_t row0, int64_t n_rows,
                uint32_t* out, int* err, cudaStream_t st);
void reverse_merge_rows(const uint32_t* pruned, int64_t N, int K, int64_t row0, int64_t n_rows, uint32_t* out,
                        int* err, cudaStream_t st);
void check_device_error(const int* err, cudaStream_t st, const char* what);

}  // namespace gta
