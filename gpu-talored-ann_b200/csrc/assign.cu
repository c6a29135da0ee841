// Exact nearest-centroid assignment for few centroids (k-means Lloyd steps and the top-2
// bucket pass when B is small): every (point, centroid) distance is the exact fp32 chain
// acc = fmaf(x[i] - c[i], x[i] - c[i], acc) over ascending dimensions -- the distance of
// the reference's exact rerank (bucketDemo/buildBucket/src/bucket.cu:4350-4363) -- so no
// tensor-core screen and no rerank pass are needed, and the result is bit-identical to
// the screened path.  Top-k kept per point by (distance, centroid id); ties keep the
// smaller id (bucket.cu:1225-1228).
//
// With B <= a few hundred centroids the contraction is 2*n*B*d flops but the tensor-core
// path pays a fixed pipeline start-up per 128 rows and a second (rerank) launch; this
// kernel reads each row once in its own element type (no f32 copy of the dataset) and is
// bound by the FP32 pipe: one packed f32x2 subtract and one packed f32x2 fma per (point,
// pair of centroids, dimension).
#include <cstdint>

#include "../../include/gta.h"
#include "common.cuh"
#include "gta_internal.h"
#include "prof.h"

namespace gta {

namespace {

constexpr int kAThreads = 128;  // threads per CTA
constexpr int kAP = 2;          // points per thread (each loaded centroid value serves both)
constexpr int kAJ = 32;         // centroids per chunk (16 packed accumulator pairs per point)
constexpr int kAD = 16;         // dimensions per chunk

template <typename T>
__device__ __forceinline__ void load_dims(const T* __restrict__ row, int k0, int d, bool vec, float (&x)[kAD]);

template <>
__device__ __forceinline__ void load_dims<float>(const float* __restrict__ row, int k0, int d, bool vec, float (&x)[kAD])
{
    if (vec && k0 + kAD <= d) {
        const float4* r4 = reinterpret_cast<const float4*>(row + k0);
#pragma unroll
        for (int q = 0; q < kAD / 4; ++q) {
            const float4 v = __ldg(r4 + q);
            x[4 * q] = v.x; x[4 * q + 1] = v.y; x[4 * q + 2] = v.z; x[4 * q + 3] = v.w;
        }
    } else {
#pragma unroll
        for (int q = 0; q < kAD; ++q) x[q] = (k0 + q < d) ? __ldg(row + k0 + q) : 0.0f;
    }
}

template <typename B8>
__device__ __forceinline__ void load_dims_8bit(const B8* __restrict__ row, int k0, int d, bool vec, float (&x)[kAD])
{
    if (vec && k0 + kAD <= d) {
        const uint4* r4 = reinterpret_cast<const uint4*>(row + k0);
#pragma unroll
        for (int q = 0; q < kAD / 16; ++q) {
            const uint4 v = __ldg(r4 + q);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int b = 0; b < 16; ++b) {
                const uint32_t byte = (w[b >> 2] >> (8 * (b & 3))) & 0xffu;
                x[16 * q + b] = static_cast<float>(static_cast<B8>(byte));
            }
        }
    } else {
#pragma unroll
        for (int q = 0; q < kAD; ++q) x[q] = (k0 + q < d) ? static_cast<float>(row[k0 + q]) : 0.0f;
    }
}

template <>
__device__ __forceinline__ void load_dims<uint8_t>(const uint8_t* __restrict__ row, int k0, int d, bool vec, float (&x)[kAD])
{
    load_dims_8bit(row, k0, d, vec, x);
}

template <>
__device__ __forceinline__ void load_dims<int8_t>(const int8_t* __restrict__ row, int k0, int d, bool vec, float (&x)[kAD])
{
    load_dims_8bit(row, k0, d, vec, x);
}

template <int K>
__device__ __forceinline__ void keep_k(float (&bd)[K], int32_t (&bi)[K], float cv, int32_t ci)
{
#pragma unroll
    for (int r = 0; r < K; ++r) {
        if (cv < bd[r] || (cv == bd[r] && ci < bi[r])) {
            const float tv = bd[r];
            const int32_t ti = bi[r];
            bd[r] = cv; bi[r] = ci;
            cv = tv; ci = ti;
        }
    }
}

// CT[k][j] = C[j][k] for k < d, j < B; zero elsewhere (d32 x B32, both multiples of 32).
__global__ void centroids_t_kernel(const float* __restrict__ C, int B, int d, int ldc, int B32, int d32,
                                   float* __restrict__ CT)
{
    const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (e >= static_cast<int64_t>(B32) * d32) return;
    const int k = static_cast<int>(e / B32), j = static_cast<int>(e % B32);
    CT[e] = (j < B && k < d) ? C[static_cast<int64_t>(j) * ldc + k] : 0.0f;
}

// 128 threads = 4 warps; every thread keeps kAP points.  With S in {1, 2, 4} groups, warp w
// serves group s = w % S and the points (w / S) * 32 * kAP + i * 32 + lane (i < kAP) of the
// CTA's 128 * kAP / S points; group s takes the centroid chunks s, s + S, ...  The centroid
// values of one dimension are the same for the whole warp (a uniform, L1-resident load of the
// transposed centroids).  The groups' top-k lists are merged through shared memory at the end.
template <typename T, int K>
__global__ void __launch_bounds__(kAThreads) assign_exact_kernel(const T* __restrict__ X, int64_t n, int ldx, int d,
                                                                 const int32_t* __restrict__ row_ids,
                                                                 const float* __restrict__ CT, int B, int B32, int S,
                                                                 int vec, int32_t* __restrict__ ids,
                                                                 float* __restrict__ dists)
{
    __shared__ float ld_s[kAThreads * kAP * K];
    __shared__ int32_t li_s[kAThreads * kAP * K];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int grp = w % S;
    const int pts = kAThreads * kAP / S;
    int pl[kAP];
    int64_t pp[kAP];
    bool live[kAP];
    const T* row[kAP];
#pragma unroll
    for (int i = 0; i < kAP; ++i) {
        pl[i] = (w / S) * 32 * kAP + i * 32 + lane;
        pp[i] = static_cast<int64_t>(blockIdx.x) * pts + pl[i];
        live[i] = pp[i] < n;
        const int64_t r = live[i] ? (row_ids ? static_cast<int64_t>(row_ids[pp[i]]) : pp[i]) : 0;
        row[i] = X + r * static_cast<int64_t>(ldx);
    }
    float bd[kAP][K];
    int32_t bi[kAP][K];
#pragma unroll
    for (int i = 0; i < kAP; ++i)
#pragma unroll
        for (int r = 0; r < K; ++r) { bd[i][r] = INFINITY; bi[i][r] = -1; }

    for (int j0 = grp * kAJ; j0 < B; j0 += S * kAJ) {
        unsigned long long acc[kAP][kAJ / 2];
#pragma unroll
        for (int i = 0; i < kAP; ++i)
#pragma unroll
            for (int j = 0; j < kAJ / 2; ++j) acc[i][j] = 0ull;
        for (int k0 = 0; k0 < d; k0 += kAD) {
            float x[kAP][kAD];
#pragma unroll
            for (int i = 0; i < kAP; ++i) {
                if (live[i]) load_dims<T>(row[i], k0, d, vec != 0, x[i]);
                else {
#pragma unroll
                    for (int q = 0; q < kAD; ++q) x[i][q] = 0.0f;
                }
            }
            const float* ct = CT + static_cast<int64_t>(k0) * B32 + j0;
#pragma unroll
            for (int kk = 0; kk < kAD; ++kk) {
                unsigned long long xx[kAP];
#pragma unroll
                for (int i = 0; i < kAP; ++i) xx[i] = f2_pack(x[i][kk], x[i][kk]);
                const ulonglong2* c4 = reinterpret_cast<const ulonglong2*>(ct + static_cast<int64_t>(kk) * B32);
#pragma unroll
                for (int q = 0; q < kAJ / 4; ++q) {
                    const ulonglong2 c = __ldg(c4 + q);  // centroids 4q .. 4q + 3 as two packed pairs
#pragma unroll
                    for (int i = 0; i < kAP; ++i) {
                        const unsigned long long t0 = f2_sub(xx[i], c.x);
                        const unsigned long long t1 = f2_sub(xx[i], c.y);
                        acc[i][2 * q] = f2_fma(t0, t0, acc[i][2 * q]);
                        acc[i][2 * q + 1] = f2_fma(t1, t1, acc[i][2 * q + 1]);
                    }
                }
            }
        }
        // keep the K smallest by (distance, id), candidates in ascending id
#pragma unroll
        for (int i = 0; i < kAP; ++i)
#pragma unroll
            for (int j = 0; j < kAJ / 2; ++j) {
                float lo, hi;
                f2_unpack(acc[i][j], lo, hi);
                if (j0 + 2 * j < B) keep_k<K>(bd[i], bi[i], lo, j0 + 2 * j);
                if (j0 + 2 * j + 1 < B) keep_k<K>(bd[i], bi[i], hi, j0 + 2 * j + 1);
            }
    }
    if (S > 1) {  // merge the S groups' lists of each point
#pragma unroll
        for (int i = 0; i < kAP; ++i)
#pragma unroll
            for (int r = 0; r < K; ++r) {
                ld_s[(grp * pts + pl[i]) * K + r] = bd[i][r];
                li_s[(grp * pts + pl[i]) * K + r] = bi[i][r];
            }
        __syncthreads();
        if (grp != 0) return;
        for (int g = 1; g < S; ++g)
#pragma unroll
            for (int i = 0; i < kAP; ++i)
#pragma unroll
                for (int r = 0; r < K; ++r)
                    keep_k<K>(bd[i], bi[i], ld_s[(g * pts + pl[i]) * K + r], li_s[(g * pts + pl[i]) * K + r]);
    }
#pragma unroll
    for (int i = 0; i < kAP; ++i) {
        if (!live[i]) continue;
#pragma unroll
        for (int r = 0; r < K; ++r) {
            ids[pp[i] * K + r] = bi[i][r];
            if (dists) dists[pp[i] * K + r] = bd[i][r];
        }
    }
}

template <typename T>
void launch_exact(const T* X, int64_t n, int ldx, int d, const int32_t* row_ids, const float* C, int ldc, int B, int k,
                  int32_t* ids, float* dists, cudaStream_t st)
{
    const bool vec = ((static_cast<int64_t>(ldx) * sizeof(T)) % 16 == 0) && (reinterpret_cast<uintptr_t>(X) % 16 == 0);
    const int B32 = (B + kAJ - 1) / kAJ * kAJ, d32 = (d + kAD - 1) / kAD * kAD;
    DevBuf<float> CT(static_cast<size_t>(B32) * d32, st);
    const int64_t nct = static_cast<int64_t>(B32) * d32;
    centroids_t_kernel<<<static_cast<unsigned>((nct + 255) / 256), 256, 0, st>>>(C, B, d, ldc, B32, d32, CT.get());
    int dev = 0, n_sm = 0;
    GTA_CUDA(cudaGetDevice(&dev));
    GTA_CUDA(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev));
    // split the centroids over S warps per point while the CTAs would fill fewer than ~8 waves
    // of 4 resident CTAs per SM
    const int64_t slots = static_cast<int64_t>(n_sm) * 4 * kAThreads * kAP;
    const int n_chunks = B32 / kAJ;
    int S = 1;
    while (S < 4 && 2 * S <= n_chunks && n * S < 8 * slots) S *= 2;
    const int pts = kAThreads * kAP / S;
    const unsigned grid = static_cast<unsigned>((n + pts - 1) / pts);
    const float* ct = CT.get();
#define GTA_ASSIGN_LAUNCH(KK) \
    assign_exact_kernel<T, KK><<<grid, kAThreads, 0, st>>>(X, n, ldx, d, row_ids, ct, B, B32, S, vec, ids, dists)
    switch (k) {
        case 1: GTA_ASSIGN_LAUNCH(1); break;
        case 2: GTA_ASSIGN_LAUNCH(2); break;
        case 3: GTA_ASSIGN_LAUNCH(3); break;
        default: GTA_ASSIGN_LAUNCH(4); break;
    }
#undef GTA_ASSIGN_LAUNCH
}

// [x | x | 0] rows for the split screen (x: d of the ld-strided f32 rows)
__global__ void dup_rows_kernel(const float* __restrict__ X, int d, int ld, int64_t n, float* __restrict__ out, int pitch)
{
    const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (e >= n * pitch) return;
    const int64_t r = e / pitch;
    const int k = static_cast<int>(e - r * pitch);
    out[e] = k < d ? X[r * ld + k] : (k < 2 * d ? X[r * ld + k - d] : 0.0f);
}

// [hi | lo | 0] centroid rows: hi = c with its low 13 mantissa bits cleared, lo the same of c - hi;
// both are exact tf32 values (whatever the tensor core does with the bits below tf32), and
// |c - hi - lo| <= 2^-20 |c|
__device__ __forceinline__ float tf32_trunc(float v) { return __uint_as_float(__float_as_uint(v) & 0xFFFFE000u); }

__global__ void split_rows_kernel(const float* __restrict__ C, int d, int ld, int64_t n, float* __restrict__ out,
                                  int pitch)
{
    const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (e >= n * pitch) return;
    const int64_t r = e / pitch;
    const int k = static_cast<int>(e - r * pitch);
    float v = 0.0f;
    if (k < d) {
        v = tf32_trunc(C[r * ld + k]);
    } else if (k < 2 * d) {
        const float c = C[r * ld + k - d];
        v = tf32_trunc(c - tf32_trunc(c));
    }
    out[e] = v;
}

}  // namespace

void dup_rows(const float* X, int d, int ld, int64_t n, float* out, int pitch, cudaStream_t st)
{
    const int64_t tot = n * pitch;
    dup_rows_kernel<<<static_cast<unsigned>((tot + 255) / 256), 256, 0, st>>>(X, d, ld, n, out, pitch);
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

void split_rows_tf32(const float* C, int d, int ld, int64_t n, float* out, int pitch, cudaStream_t st)
{
    const int64_t tot = n * pitch;
    split_rows_kernel<<<static_cast<unsigned>((tot + 255) / 256), 256, 0, st>>>(C, d, ld, n, out, pitch);
    count_launches(1);
    GTA_CUDA(cudaGetLastError());
}

bool assign_exact_applies(int B, int k) { return B <= kAssignExactMaxB && k >= 1 && k <= 4; }

void assign_exact(const void* X, int dtype, int64_t n, int ldx, int d, const int32_t* row_ids, const float* C, int ldc,
                  int B, int k, int32_t* ids, float* dists, cudaStream_t st)
{
    GTA_REQUIRE(assign_exact_applies(B, k) && n >= 0 && d >= 1 && ldx >= d && ldc >= d, kInvalid,
                "assign_exact: need B <= 384, 1 <= k <= 4");
    if (n == 0) return;
    ProfScope prof("assign_exact", 2.0 * static_cast<double>(n) * B * d, st);
    switch (dtype) {
        case GTA_F32: launch_exact(static_cast<const float*>(X), n, ldx, d, row_ids, C, ldc, B, k, ids, dists, st); break;
        case GTA_U8: launch_exact(static_cast<const uint8_t*>(X), n, ldx, d, row_ids, C, ldc, B, k, ids, dists, st); break;
        case GTA_I8: launch_exact(static_cast<const int8_t*>(X), n, ldx, d, row_ids, C, ldc, B, k, ids, dists, st); break;
        default: throw Error(kInvalid, "assign_exact: unknown dtype");
    }
    count_launches(2);
    GTA_CUDA(cudaGetLastError());
}

}  // namespace gta
