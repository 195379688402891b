// RVQ encoder and k-means on the GPU (sm_100a): the offline compressor's
// hot loops (compress_full_model.py:196-234 pairwise_sqdist / assign_codes /
// kmeans_train, and 337-366 encode_rvq_tensor), which the reference runs on
// the CPU in chunks.
//
// Distances follow pairwise_sqdist's formula, in fp32:
//   dist(x, c) = (|x|^2 + |c|^2) - 2 (x . c),   argmin over c, first minimum wins
// (torch.argmin's rule).  The reference's CPU BLAS may sum the 8 products in
// another order, so two codes whose distances differ in the last bits can be
// ordered differently; everywhere else the chosen code is the same.
//
// One thread per vector; the stage's codebook and its |c|^2 sit in shared
// memory and every thread walks all codes (broadcast reads).  The encoder
// runs all stages of a vector in one thread: assign, record the code,
// subtract the codeword from the residual (fp32, as `residual -= part`).
//
// k-means statistics are accumulated in 64-bit fixed point (value * 2^32,
// integer atomics), so the centroid sums do not depend on the order in which
// threads add: the same input always gives the same centroids.

#include <mutex>
#include <string.h>

#include "rvq_common.cuh"

namespace rvq {
namespace enc {

constexpr int kD = 8;
constexpr int kThreads = 256;
constexpr int kMaxCodes = 4096;                      // shared memory: 4096 x 9 floats = 144 KB
constexpr int kMaxLocal = 1024;                      // k for block-local k-means totals (+72 KB)
constexpr double kFixScale = 4294967296.0;           // 2^32

__device__ __forceinline__ float sqnorm8(const float (&v)[kD]) {
    float s = 0.f;
#pragma unroll
    for (int t = 0; t < kD; ++t) s = fmaf(v[t], v[t], s);
    return s;
}

// Nearest code of v in the staged codebook (first minimum).
__device__ __forceinline__ int nearest(const float (&v)[kD], const float* cbs, const float* c2s, int ncodes) {
    const float x2 = sqnorm8(v);
    float best = __int_as_float(0x7f800000);
    int bi = 0;
    for (int c = 0; c < ncodes; ++c) {
        const float4 a = *reinterpret_cast<const float4*>(cbs + c * kD);
        const float4 b = *reinterpret_cast<const float4*>(cbs + c * kD + 4);
        float dot = v[0] * a.x;
        dot = fmaf(v[1], a.y, dot);
        dot = fmaf(v[2], a.z, dot);
        dot = fmaf(v[3], a.w, dot);
        dot = fmaf(v[4], b.x, dot);
        dot = fmaf(v[5], b.y, dot);
        dot = fmaf(v[6], b.z, dot);
        dot = fmaf(v[7], b.w, dot);
        const float dist = __fsub_rn(__fadd_rn(x2, c2s[c]), 2.0f * dot);
        if (dist < best) {                           // NaN never wins; ties keep the first
            best = dist;
            bi = c;
        }
    }
    return bi;
}

__device__ __forceinline__ void stage_codebook(const float* cb, int ncodes, float* cbs, float* c2s) {
    for (int i = threadIdx.x; i < ncodes * kD; i += blockDim.x) cbs[i] = cb[i];
    __syncthreads();
    for (int c = threadIdx.x; c < ncodes; c += blockDim.x) {
        float v[kD];
#pragma unroll
        for (int t = 0; t < kD; ++t) v[t] = cbs[c * kD + t];
        c2s[c] = sqnorm8(v);
    }
    __syncthreads();
}

// All stages: codes[k][i] = nearest(residual_k), residual_{k+1} = residual_k - cb_k[code].
__global__ void __launch_bounds__(kThreads) encode_kernel(const float* __restrict__ x, int64_t n,
                                                          const float* __restrict__ cb, int stages, int ncodes,
                                                          void* codes, int code_bytes, float* residual_out) {
    extern __shared__ float sm[];
    float* cbs = sm;
    float* c2s = sm + ncodes * kD;
    const int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    float v[kD];
    if (i < n) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(x + i * kD));
        const float4 b = __ldg(reinterpret_cast<const float4*>(x + i * kD + 4));
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
    for (int k = 0; k < stages; ++k) {
        if (k) __syncthreads();                      // every thread is done with the previous stage
        stage_codebook(cb + (int64_t)k * ncodes * kD, ncodes, cbs, c2s);
        if (i < n) {
            const int c = nearest(v, cbs, c2s, ncodes);
            if (code_bytes == 1) reinterpret_cast<uint8_t*>(codes)[(int64_t)k * n + i] = (uint8_t)c;
            else reinterpret_cast<int16_t*>(codes)[(int64_t)k * n + i] = (int16_t)c;
#pragma unroll
            for (int t = 0; t < kD; ++t) v[t] = __fsub_rn(v[t], cbs[c * kD + t]);
        }
    }
    if (i < n && residual_out) {
        float4* o = reinterpret_cast<float4*>(residual_out + i * kD);
        o[0] = make_float4(v[0], v[1], v[2], v[3]);
        o[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
}

// One Lloyd step's statistics: assign[i] = nearest centroid, and in fixed
// point sums[c][t] += x[i][t] * 2^32, counts[c] += 1.
// LOCAL: the block first adds into shared-memory totals (k <= kMaxLocal),
// then adds each nonzero total to global memory once.
__global__ void __launch_bounds__(kThreads) kmeans_kernel(const float* __restrict__ x, int64_t n,
                                                          const float* __restrict__ cent, int k, int32_t* assign,
                                                          unsigned long long* sums, unsigned long long* counts,
                                                          int local) {
    extern __shared__ float sm[];
    float* cbs = sm;
    float* c2s = sm + k * kD;
    unsigned long long* ls = reinterpret_cast<unsigned long long*>(sm + ((k * (kD + 1) + 1) & ~1));
    unsigned long long* lc = ls + k * kD;
    if (sums && local)
        for (int j = threadIdx.x; j < k * (kD + 1); j += blockDim.x) ls[j] = 0ull;
    stage_codebook(cent, k, cbs, c2s);                       // ends with a barrier
    const int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (i < n) {
        float v[kD];
        const float4 a = __ldg(reinterpret_cast<const float4*>(x + i * kD));
        const float4 b = __ldg(reinterpret_cast<const float4*>(x + i * kD + 4));
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        const int c = nearest(v, cbs, c2s, k);
        if (assign) assign[i] = c;
        if (sums) {
            unsigned long long* ts = local ? ls : sums;
            unsigned long long* tc = local ? lc : counts;
#pragma unroll
            for (int t = 0; t < kD; ++t)
                atomicAdd(ts + c * kD + t, (unsigned long long)__double2ll_rn((double)v[t] * kFixScale));
            atomicAdd(tc + c, 1ull);
        }
    }
    if (sums && local) {
        __syncthreads();
        for (int j = threadIdx.x; j < k * kD; j += blockDim.x)
            if (ls[j]) atomicAdd(sums + j, ls[j]);
        for (int j = threadIdx.x; j < k; j += blockDim.x)
            if (lc[j]) atomicAdd(counts + j, lc[j]);
    }
}

std::mutex g_mu;
bool g_ready[64] = {}, g_ok[64] = {};

int prepare() {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64) {
        last_cuda_error_slot() = (int)e;
        return RVQ_ERR_UNAVAILABLE;
    }
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_ready[dev]) {
        g_ready[dev] = true;
        const int smem = kMaxCodes * (kD + 1) * 4 + 8;
        e = cudaFuncSetAttribute(encode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(kmeans_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        g_ok[dev] = e == cudaSuccess;
        if (e != cudaSuccess) last_cuda_error_slot() = (int)e;
    }
    return g_ok[dev] ? RVQ_OK : RVQ_ERR_UNAVAILABLE;
}

int finish() {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        last_cuda_error_slot() = (int)e;
        return RVQ_ERR_CUDA;
    }
    return RVQ_OK;
}

}  // namespace enc
}  // namespace rvq

using namespace rvq;
using namespace rvq::enc;

extern "C" {

int rvq_encode_vectors(const float* x, int64_t n, const float* codebooks, int stages, int ncodes, int d, void* codes,
                       int code_kind, float* residual_out, void* stream) {
    if (n < 0 || stages < 1 || ncodes < 1 || (n > 0 && (!x || !codes)) || !codebooks) return RVQ_ERR_INVALID;
    if (d != kD) return RVQ_ERR_UNSUPPORTED;
    if (ncodes > kMaxCodes || n >= (1ll << 40)) return RVQ_ERR_TOO_LARGE;
    if (code_kind != RVQ_U8 && code_kind != RVQ_I16) return RVQ_ERR_UNSUPPORTED;
    if (code_kind == RVQ_U8 && ncodes > 256) return RVQ_ERR_INVALID;
    if (((uintptr_t)x & 15) || (residual_out && ((uintptr_t)residual_out & 15))) return RVQ_ERR_INVALID;
    int rc = prepare();
    if (rc != RVQ_OK || n == 0) return rc;
    const int64_t blocks = (n + kThreads - 1) / kThreads;
    encode_kernel<<<(unsigned)blocks, kThreads, (size_t)ncodes * (kD + 1) * 4, (cudaStream_t)stream>>>(
        x, n, codebooks, stages, ncodes, codes, code_kind == RVQ_U8 ? 1 : 2, residual_out);
    return finish();
}

int rvq_kmeans_step(const float* x, int64_t n, const float* centroids, int k, int d, int32_t* assign,
                    unsigned long long* sums, unsigned long long* counts, void* stream) {
    if (n < 0 || k < 1 || (n > 0 && !x) || !centroids || (sums && !counts)) return RVQ_ERR_INVALID;
    if (d != kD) return RVQ_ERR_UNSUPPORTED;
    if (k > kMaxCodes || n >= (1ll << 40)) return RVQ_ERR_TOO_LARGE;
    if ((uintptr_t)x & 15) return RVQ_ERR_INVALID;
    int rc = prepare();
    if (rc != RVQ_OK || n == 0) return rc;
    const int64_t blocks = (n + kThreads - 1) / kThreads;
    const int local = sums != nullptr && k <= kMaxLocal;
    size_t smem = (size_t)(((k * (kD + 1) + 1) & ~1)) * 4;
    if (local) smem += (size_t)k * (kD + 1) * 8;
    kmeans_kernel<<<(unsigned)blocks, kThreads, smem, (cudaStream_t)stream>>>(x, n, centroids, k, assign, sums,
                                                                             counts, local);
    return finish();
}

}  // extern "C"
