// Device helpers of the batch-1 decode-step operations (bf16 rounding,
// projection-output operands, warp sums, per-head RMSNorm + rotary
// embedding, cache-row loads).  Included by rvq_step.cu (one launch per
// operation) and rvq_persist.cu (the persistent decode step).
#pragma once

#include <type_traits>

#include "rvq_common.cuh"

namespace rvq {
namespace stepops {

// fp32 load: through the read-only path, or through L2 (kL2: data that other
// CTAs of the same launch wrote)
template <bool kL2>
__device__ __forceinline__ float ldf(const float* p) {
    if constexpr (kL2) return __ldcg(p);
    else return __ldg(p);
}

// element i of a 16- or 32-bit vector as fp32, through L2
__device__ __forceinline__ float ldcg_f32(const void* p, int64_t i, int kind) {
    if (kind == RVQ_F32) return __ldcg(reinterpret_cast<const float*>(p) + i);
    const unsigned short u = __ldcg(reinterpret_cast<const unsigned short*>(p) + i);
    return kind == RVQ_F16 ? __half2float(__ushort_as_half(u)) : __bfloat162float(__ushort_as_bfloat16(u));
}

__device__ __forceinline__ float bf16r(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

__device__ __forceinline__ float bf16_at(const void* p, int64_t i) {
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}

__device__ __forceinline__ void put_bf16(void* p, int64_t i, float v) {
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
}

// Value i of a vector operand (see rvq_vec).  Partials are added in tile
// order; their loads are issued 8 at a time ahead of the adds, so a 38-tile
// sum costs 5 memory round trips instead of 38.
template <bool kL2 = false>
__device__ __forceinline__ float vec_value(const rvq_vec& v, int64_t i) {
    if (v.kind == RVQ_F32) {
        const float* p = reinterpret_cast<const float*>(v.ptr) + i;
        const int64_t n = v.n;
        const int nt = v.ntiles;
        float s = ldf<kL2>(p);
        int t = 1;
        for (; t + 8 <= nt; t += 8) {
            float c[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) c[k] = ldf<kL2>(p + (int64_t)(t + k) * n);
#pragma unroll
            for (int k = 0; k < 8; ++k) s += c[k];
        }
        float c[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) c[k] = (t + k < nt) ? ldf<kL2>(p + (int64_t)(t + k) * n) : 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k)
            if (t + k < nt) s += c[k];
        return bf16r(s);
    }
    return kL2 ? ldcg_f32(v.ptr, i, v.kind) : load_as_f32(v.ptr, i, v.kind);
}

// vec_value with up to 32 partial loads in flight per thread (the tile sum is
// still taken in tile order): for consumers with few threads per element.
template <bool kL2 = false>
__device__ __forceinline__ float vec_value_deep(const rvq_vec& v, int64_t i) {
    if (v.kind != RVQ_F32 || v.ntiles <= 8) return vec_value<kL2>(v, i);
    const float* p = reinterpret_cast<const float*>(v.ptr) + i;
    const int64_t n = v.n;
    const int nt = v.ntiles;
    if (nt <= 32) {                                  // one round: 32 loads (clamped to the last tile)
        float c[32];
#pragma unroll
        for (int k = 0; k < 32; ++k) c[k] = ldf<kL2>(p + (int64_t)min(k, nt - 1) * n);
        float s = c[0];
#pragma unroll
        for (int k = 1; k < 32; ++k)
            if (k < nt) s += c[k];
        return bf16r(s);
    }
    float s = ldf<kL2>(p);
    int t = 1;
    for (; t + 32 <= nt; t += 32) {                  // whole chunks: 32 loads, then the adds in order
        float c[32];
#pragma unroll
        for (int k = 0; k < 32; ++k) c[k] = ldf<kL2>(p + (int64_t)(t + k) * n);
#pragma unroll
        for (int k = 0; k < 32; ++k) s += c[k];
    }
    for (; t + 8 <= nt; t += 8) {
        float c[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) c[k] = ldf<kL2>(p + (int64_t)(t + k) * n);
#pragma unroll
        for (int k = 0; k < 8; ++k) s += c[k];
    }
    for (; t < nt; ++t) s += ldf<kL2>(p + (int64_t)t * n);
    return bf16r(s);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// RMSNorm (weight w) + rotary embedding of one head held by one warp:
// lane holds elements d = lane + 32 j, j < hd / 32.  Returns through `o`.
template <int HD>
__device__ __forceinline__ void norm_rope_head(const float* x, const float* w, float eps, const float* cv,
                                               const float* sv, float* o) {
    constexpr int J = HD / 32;
    const int lane = threadIdx.x & 31;
    float v[J];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < J; ++j) {
        v[j] = x[lane + 32 * j];
        ss = fmaf(v[j], v[j], ss);
    }
    ss = warp_sum(ss);
    const float inv = rsqrtf(ss / (float)HD + eps);
#pragma unroll
    for (int j = 0; j < J; ++j) v[j] = bf16r(w[lane + 32 * j] * bf16r(v[j] * inv));
    // rotate_half: d < HD/2 -> -v[d + HD/2], else v[d - HD/2]; held by the same lane
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const int d = lane + 32 * j;
        const float rot = j < J / 2 ? -v[j + J / 2] : v[j - J / 2];
        o[j] = bf16r(bf16r(v[j] * cv[d]) + bf16r(rot * sv[d]));
    }
}

// E consecutive bf16 of a cache row as floats.
template <int E>
__device__ __forceinline__ void load_row_slice(const __nv_bfloat16* src, float (&out)[E]) {
    if constexpr (E == 2) {
        const __nv_bfloat162 w = *reinterpret_cast<const __nv_bfloat162*>(src);
        out[0] = __low2float(w);
        out[1] = __high2float(w);
    } else {
        using V = typename std::conditional<E == 4, uint2, uint4>::type;
        const V w = *reinterpret_cast<const V*>(src);
        const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&w);
#pragma unroll
        for (int t = 0; t < E; ++t) out[t] = __bfloat162float(e[t]);
    }
}

}  // namespace stepops
}  // namespace rvq
