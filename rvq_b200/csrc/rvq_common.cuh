// Shared device/host helpers of the rvq_b200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "rvq_b200.h"

namespace rvq {

// ---------------------------------------------------------------------------
// Division by a run-time invariant divisor (Granlund & Montgomery, "Division
// by invariant integers using multiplication", PLDI 1994, round-up variant):
// with l = ceil(log2 d) and m = floor(2^32 (2^l - d) / d) + 1,
//   n / d == (umulhi(n, m) + n) >> l   for every 32-bit n.
// The sum is formed in 64 bits so n may use all 32 bits.
// ---------------------------------------------------------------------------
struct FastDiv {
    uint32_t d;
    uint32_t m;
    uint32_t l;
};

inline FastDiv make_fastdiv(uint32_t d) {
    FastDiv f;
    f.d = d;
    uint32_t l = 0;
    while ((1ull << l) < d) ++l;
    f.l = l;
    f.m = (uint32_t)((((1ull << 32) * ((1ull << l) - d)) / d) + 1ull);
    return f;
}

__host__ __device__ __forceinline__ uint32_t fastdiv(uint32_t n, const FastDiv& f) {
#ifdef __CUDA_ARCH__
    uint32_t hi = __umulhi(n, f.m);
#else
    uint32_t hi = (uint32_t)(((uint64_t)n * f.m) >> 32);
#endif
    return (uint32_t)(((uint64_t)hi + n) >> f.l);
}

// ---------------------------------------------------------------------------
// Element conversions.  All casts to 16-bit types round to nearest even and
// keep subnormals (no -ftz in this build).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float load_as_f32(const void* p, int64_t i, int kind) {
    if (kind == RVQ_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
    if (kind == RVQ_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    return reinterpret_cast<const float*>(p)[i];
}

__device__ __forceinline__ void store_from_f32(void* p, int64_t i, int kind, float v) {
    if (kind == RVQ_F16) reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
    else if (kind == RVQ_BF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
    else reinterpret_cast<float*>(p)[i] = v;
}

// fp32 <- fp16 (exact) + fp32, one rounding: the sm_100 mixed-precision add.
__device__ __forceinline__ float add_f16_f32(uint16_t h, float c) {
    float d;
    asm("add.rn.f32.f16 %0, %1, %2;" : "=f"(d) : "h"(h), "f"(c));
    return d;
}

// Both halves of a packed fp16 pair added into two fp32 accumulators, each
// with one IEEE round-to-nearest add (add.rn.f32.f16 on the register halves:
// no separate unpacking instructions).
__device__ __forceinline__ void add_f16x2_f32(float& lo_acc, float& hi_acc, uint32_t w) {
    asm("{\n .reg .b16 lo, hi;\n mov.b32 {lo, hi}, %2;\n add.rn.f32.f16 %0, lo, %0;\n add.rn.f32.f16 %1, hi, %1;\n}\n"
        : "+f"(lo_acc), "+f"(hi_acc)
        : "r"(w));
}

// a *= s, b *= s as one packed fp32x2 multiply (sm_100 mul.rn.f32x2: each
// lane an IEEE round-to-nearest fp32 product, bit-identical to two __fmul_rn).
__device__ __forceinline__ void mul2_f32(float& a, float& b, float s) {
    asm("{\n .reg .b64 A, B, C;\n mov.b64 A, {%0, %1};\n mov.b64 B, {%2, %2};\n mul.rn.f32x2 C, A, B;\n"
        " mov.b64 {%0, %1}, C;\n}\n"
        : "+f"(a), "+f"(b)
        : "f"(s));
}

// 32 bytes (two 16-byte vectors) with one 256-bit store that does not allocate
// in L1 (write-once data).  dst must be 32-byte aligned.
__device__ __forceinline__ void store_v8_na(void* dst, const uint4& a, const uint4& b) {
    asm volatile("st.global.L1::no_allocate.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};\n" ::"l"(dst), "r"(a.x),
                 "r"(a.y), "r"(a.z), "r"(a.w), "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w)
                 : "memory");
}

__device__ __forceinline__ uint32_t pack2(float a, float b, int out_kind) {
    if (out_kind == RVQ_BF16) {
        __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&v);
    }
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch (sm_90+).  A kernel launched with launch_pdl
// may start while the previous kernel of its stream is still running, once
// every CTA of that kernel has called pdl_launch_dependents().  It may read
// only data that no earlier kernel of the stream writes (weights, code words,
// codebooks) before pdl_wait(), which returns when the previous kernel has
// completed and its writes are visible; it writes nothing before pdl_wait().
// Every kernel calls pdl_wait() on every path, so completion is transitive
// along the stream.
// ---------------------------------------------------------------------------
// Reduce 8 per-lane values (rows 0..7) over the warp: returns the total of row
// (lane >> 2) & 7 (in every lane of that row's quad).  9 shuffles, fixed order.
__device__ __forceinline__ float reduce8(const float (&v)[8]) {
    const int lane = threadIdx.x & 31;
    const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
    float u[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float send = b4 ? v[i] : v[i + 4];
        const float keep = b4 ? v[i + 4] : v[i];
        u[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
    float w[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const float send = b3 ? u[i] : u[i + 2];
        const float keep = b3 ? u[i + 2] : u[i];
        w[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
    const float send = b2 ? w[0] : w[1];
    const float keep = b2 ? w[1] : w[0];
    float z = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    z += __shfl_xor_sync(0xffffffffu, z, 2);
    z += __shfl_xor_sync(0xffffffffu, z, 1);
    return z;
}

__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Last CUDA error seen by the library on the calling thread (shared by all
// translation units through this inline function's static).
inline int& last_cuda_error_slot() {
    static thread_local int v = 0;
    return v;
}

inline int elem_bytes(int kind) {
    switch (kind) {
        case RVQ_F16: case RVQ_BF16: case RVQ_I16: return 2;
        case RVQ_F32: return 4;
        case RVQ_U8: return 1;
        default: return 0;
    }
}

}  // namespace rvq
