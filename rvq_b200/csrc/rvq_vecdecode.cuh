// Bit-exact reconstruction of one RVQ vector (K=4 stages, 256 codes, d=8) to
// bf16, shared by the fused kernels that consume weights without writing them
// to HBM:
//   w[t] = RNE_bf16( fp32(scale) * (((0 + cb0[c0][t]) + cb1[c1][t]) + cb2[c2][t]) + cb3[c3][t] )
// -- the fp32 sum in stage order starting from +0, the same bits rvq_decode
// writes into a bf16 slot (_rvq_decode_into_kernel, triton_decode_kernels.py:
// 78-104).
//
// The codebook sits in shared memory as fp16 with 8 copies per entry: entry
// (k, c), copy p at byte (k / 2) << 16 | c << 8 | (k % 2) << 7 | p << 4
// (128 KB), so one prmt of a code word (stage k's code in byte k) with the
// lane's constant bits gives the address, and the 8 lanes of a quarter-warp
// phase (p = lane & 7) always read 8 different bank quads.
#pragma once

#include "rvq_common.cuh"

namespace rvq {
namespace vdec {

constexpr int kStages = 4;
constexpr int kCodes = 256;
constexpr int kCopies = 8;
constexpr int kCbBytes = kStages * kCodes * 16 * kCopies;    // 128 KB

// Per-lane constant bits of the prmt address for stage k (byte 0: stage
// parity and copy, byte 2: stage pair).
__device__ __forceinline__ void lane_bits(int lane, uint32_t (&lb)[kStages]) {
#pragma unroll
    for (int k = 0; k < kStages; ++k)
        lb[k] = ((uint32_t)(k & 1) << 7) | ((uint32_t)(lane & 7) << 4) | ((uint32_t)(k >> 1) << 16);
}

// Load codebook entry e (8 values): returned as is for an fp16 codebook, else
// into f as fp32.
__device__ __forceinline__ uint4 cb_entry_f16(const void* cb, int cb_kind, int e, float (&f)[8]) {
    if (cb_kind == RVQ_F16) return __ldg(reinterpret_cast<const uint4*>(cb) + e);
    if (cb_kind == RVQ_F32) {                            // 32-byte entries: two 16-byte loads
        const float4 a = __ldg(reinterpret_cast<const float4*>(cb) + 2 * e);
        const float4 b = __ldg(reinterpret_cast<const float4*>(cb) + 2 * e + 1);
        f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
    } else {
#pragma unroll
        for (int t = 0; t < 8; ++t) f[t] = load_as_f32(cb, (int64_t)e * 8 + t, cb_kind);
    }
    return make_uint4(0u, 0u, 0u, 0u);
}

// fp16 form of a loaded entry (fp32 values f, or q itself for an fp16 codebook);
// sets *inexact when a value is not an exact fp16 number.
__device__ __forceinline__ uint4 cb_entry_pack(int cb_kind, const uint4& q, const float (&f)[8], int* inexact) {
    if (cb_kind == RVQ_F16) return q;
    uint32_t w[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const float f0 = f[2 * t], f1 = f[2 * t + 1];
        const __half2 h = __floats2half2_rn(f0, f1);
        *inexact |= (__float_as_uint(__low2float(h)) != __float_as_uint(f0)) |
                    (__float_as_uint(__high2float(h)) != __float_as_uint(f1)) | isnan(f0) | isnan(f1);
        w[t] = *reinterpret_cast<const uint32_t*>(&h);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ void cb_entry_store(char* cbs, int e, int lane, const uint4& q) {
    char* base = cbs + ((e >> 9) << 16) + ((e & 255) << 8) + (((e >> 8) & 1) << 7);
#pragma unroll
    for (int i = 0; i < kCopies; ++i) {
        const int cp = (i + lane) & (kCopies - 1);
        *reinterpret_cast<uint4*>(base + cp * 16) = q;
    }
}

// Stage the [4][256][8] codebook (fp32, fp16 or bf16 kind) into `cbs` as fp16
// with 8 copies; all `nthreads` threads of the CTA call it (thread index
// `tid`).  Returns true if every value is an exact fp16 number (false: the
// caller reads the codebook from global memory instead).  Each thread loads
// two entries before converting and storing them (one memory round trip when
// nthreads >= 512).  Ends with a CTA-wide barrier.
__device__ __forceinline__ bool stage_cb8(const void* cb, int cb_kind, char* cbs, int tid, int nthreads) {
    const int lane = tid & 31;
    int inexact = 0;
    for (int e0 = tid; e0 < kStages * kCodes; e0 += 2 * nthreads) {
        const int e1 = e0 + nthreads;
        const bool has1 = e1 < kStages * kCodes;
        float f0[8], f1[8];
        const uint4 q0 = cb_entry_f16(cb, cb_kind, e0, f0);
        uint4 q1 = make_uint4(0u, 0u, 0u, 0u);
        if (has1) q1 = cb_entry_f16(cb, cb_kind, e1, f1);
        cb_entry_store(cbs, e0, lane, cb_entry_pack(cb_kind, q0, f0, &inexact));
        if (has1) cb_entry_store(cbs, e1, lane, cb_entry_pack(cb_kind, q1, f1, &inexact));
    }
    return !__syncthreads_or(inexact);
}

// The 8 bf16 weights (packed pairs, element 2i in the low half) of the vector
// whose stage codes are the bytes of `w`, scaled by `s`.  SMEM: codebook
// staged by stage_cb8; otherwise read from `cb` in global memory.
template <bool SMEM>
__device__ __forceinline__ uint4 weights_bf16(const char* cbs, const void* cb, int cb_kind, uint32_t w,
                                              const uint32_t (&lb)[kStages], float s) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (SMEM) {
#pragma unroll
        for (int k = 0; k < kStages; ++k) {
            const uint4 q = *reinterpret_cast<const uint4*>(cbs + __byte_perm(w, lb[k], 0x7604 | (k << 4)));
            add_f16x2_f32(acc[0], acc[1], q.x);
            add_f16x2_f32(acc[2], acc[3], q.y);
            add_f16x2_f32(acc[4], acc[5], q.z);
            add_f16x2_f32(acc[6], acc[7], q.w);
        }
    } else {
        for (int k = 0; k < kStages; ++k) {
            const int64_t row = (int64_t)(k * kCodes + ((w >> (8 * k)) & 0xffu)) * 8;
#pragma unroll
            for (int t = 0; t < 8; ++t) acc[t] = __fadd_rn(acc[t], load_as_f32(cb, row + t, cb_kind));
        }
    }
    mul2_f32(acc[0], acc[1], s);
    mul2_f32(acc[2], acc[3], s);
    mul2_f32(acc[4], acc[5], s);
    mul2_f32(acc[6], acc[7], s);
    uint4 r;
    r.x = pack2(acc[0], acc[1], RVQ_BF16);
    r.y = pack2(acc[2], acc[3], RVQ_BF16);
    r.z = pack2(acc[4], acc[5], RVQ_BF16);
    r.w = pack2(acc[6], acc[7], RVQ_BF16);
    return r;
}

// Faster form for consumers that need y within a tolerance, not bit-exact
// weights: ((c0 + c1) + c2) + c3 summed in fp16 (three packed add.rn.f16x2
// per pair), widened to fp32, scaled and rounded to bf16 -- 20 instead of 32
// arithmetic instructions per vector; each weight is within a few fp16 ulps
// of the exact sum before the bf16 rounding.  Codebook staged by stage_cb8.
// SCALE false leaves the scale to the caller (a per-row scale applied to y).
template <bool SCALE = true>
__device__ __forceinline__ uint4 weights_bf16_fast(const char* cbs, uint32_t w, const uint32_t (&lb)[kStages],
                                                   float s) {
    uint4 q[kStages];
#pragma unroll
    for (int k = 0; k < kStages; ++k)
        q[k] = *reinterpret_cast<const uint4*>(cbs + __byte_perm(w, lb[k], 0x7604 | (k << 4)));
    const uint32_t* a = reinterpret_cast<const uint32_t*>(&q[0]);
    const uint32_t* b = reinterpret_cast<const uint32_t*>(&q[1]);
    const uint32_t* c = reinterpret_cast<const uint32_t*>(&q[2]);
    const uint32_t* d = reinterpret_cast<const uint32_t*>(&q[3]);
    uint32_t out[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint32_t h;
        asm("add.rn.f16x2 %0, %1, %2;" : "=r"(h) : "r"(a[i]), "r"(b[i]));
        asm("add.rn.f16x2 %0, %0, %1;" : "+r"(h) : "r"(c[i]));
        asm("add.rn.f16x2 %0, %0, %1;" : "+r"(h) : "r"(d[i]));
        float lo, hi;
        asm("{\n .reg .b16 l, h;\n mov.b32 {l, h}, %2;\n cvt.f32.f16 %0, l;\n cvt.f32.f16 %1, h;\n}\n"
            : "=f"(lo), "=f"(hi)
            : "r"(h));
        if (SCALE) mul2_f32(lo, hi, s);
        out[i] = pack2(lo, hi, RVQ_BF16);
    }
    return make_uint4(out[0], out[1], out[2], out[3]);
}

}  // namespace vdec
}  // namespace rvq
