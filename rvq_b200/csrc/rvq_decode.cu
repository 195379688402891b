// RVQ decode kernels for B200 (sm_100a) and their C ABI.
//
// Computes, for every vector n of every job (reference semantics:
// _rvq_decode_into_kernel, triton_decode_kernels.py:74-111, and
// _decode_rvq_into, infer_compressed_layerwise_single_slot.py:123-149):
//
//   acc[t] = ((0 + cb[0][i0][t]) + cb[1][i1][t]) + ... + cb[K-1][iK-1][t]   (fp32)
//   out[8n+t] = cast(acc[t] * float(scale[n / group_vecs]))  for 8n+t < trimmed
//   out[trimmed + i] = cast(tail[i])
//
// Design (HBM-write bound; 20 bytes of traffic per 8 bf16 weights at K=4):
// * One persistent launch decodes a list of jobs (all RVQ entries and raw
//   norm copies of a layer slot).  The work is cut into tiles of 128
//   vectors; CTA b owns the contiguous tile range [T*b/G, T*(b+1)/G), so every
//   CTA streams one or two contiguous regions and loads at most a couple of
//   codebooks.
// * 1 CTA of 1024 threads per SM.  The CTA stages the job's codebook in
//   shared memory as fp16 with 8 copies per entry: lane L reads copy (L & 7),
//   so the 8 lanes of each quarter-warp phase of a 16-byte shared load always
//   hit 8 different bank quads -- random codes never conflict.  K=4 x 256
//   codes x 16 B x 8 copies = 128 KB.  Fast-path jobs place entry (k, c),
//   copy p at byte (k / 2) << 16 | c << 8 | (k % 2) << 7 | p << 4; other jobs
//   at ((k * ncodes + c) << copies_log2 | p) * 16.
// * A codebook handed over as fp32 (what the engine uploads) is converted to
//   fp16 while it is staged; the CTA checks that every value survives the
//   round trip exactly and otherwise keeps fp32 entries instead, so the
//   result never depends on that choice.
// * Fast path (K=4, 256 codes, u8 codes, 16-bit output): lane L of a warp owns
//   vectors 4L .. 4L + 3 of its 128-vector tile, so its 32-bit index word of a
//   plane holds exactly its 4 codes (one coalesced 128-byte load per plane and
//   warp); a code byte becomes the staged entry's shared-memory byte offset
//   with one prmt, and the lane writes its vectors in pairs with 256-bit
//   stores (32 contiguous bytes per lane, no L1 allocation for the
//   write-once slot).
// * fp32 accumulation uses add.rn.f32.f16 (fp16 -> fp32 conversion fused into
//   the add; exact conversion, one rounding, same result as cvt + add.rn).

#include <stdio.h>
#include <string.h>

#include <mutex>

#include "rvq_common.cuh"

namespace rvq {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr int kTileVecs = 128;                 // vectors per warp tile
constexpr int kJ = kTileVecs / 32;             // vectors per lane per tile
constexpr int kCopyTileBytes = 2048;           // bytes per warp tile of a raw copy
constexpr int kInt8TileElems = 512;            // int8 elements per warp tile (16 per lane)
constexpr int kSmemBudget = 200 * 1024;        // codebook staging limit per CTA
constexpr int kMaxDevices = 64;

enum JobKind : uint8_t { JOB_RVQ = 0, JOB_COPY = 1, JOB_INT8 = 2 };
enum GatherMode : uint8_t { GATHER_SMEM_F16 = 0, GATHER_SMEM_F32 = 1, GATHER_GLOBAL = 2 };

struct Job {
    const void* idx;        // RVQ: code planes; COPY: source; INT8: q
    const void* cb;
    const void* scales;
    const void* tail;
    void* out;
    uint32_t nvec;          // RVQ: vectors; COPY: bytes; INT8: trimmed elements
    uint32_t stage_stride;  // elements
    FastDiv gv;             // RVQ: vectors per scale; INT8: elements per scale
    uint32_t full_vecs;     // vectors with all 8 elements < trimmed
    uint32_t tail_numel;
    uint64_t trimmed;
    uint32_t tile_begin;
    uint32_t tile_count;
    uint16_t stages;
    uint16_t ncodes;        // 0 encodes 65536 (never produced by int16 indices)
    uint8_t kind;
    uint8_t index_bytes;    // 1, 2, or 4 for the quad layout (RVQ_U8X4)
    uint8_t cb_kind;
    uint8_t scale_kind;
    uint8_t tail_kind;
    uint8_t out_kind;
    uint8_t copies_log2;    // fp16 staging copies = 1 << copies_log2
    uint8_t f16_fits;       // fp16 staging fits in shared memory
    uint8_t f32_fits;       // fp32 staging fits in shared memory
    uint8_t out_aligned;    // out is 16-byte aligned
    uint8_t fast_ok;        // eligible for the streaming fast path (see fill_rvq_job)
    uint8_t slot_ok;        // eligible for rvq_slot_kernel (see fill_rvq_job)
    uint32_t full_tiles;    // tiles whose 128 vectors are all complete (< full_vecs, < nvec)
    uint32_t cta_begin;     // job-per-CTA schedule: first CTA of this job
    uint32_t cta_count;     // job-per-CTA schedule: CTAs of this job (copies: owning CTA in cta_begin)
};

struct LayerParams {
    Job jobs[RVQ_MAX_LAYER_JOBS];
    int njobs;
    uint32_t total_tiles;
    uint32_t per_cta_jobs;  // 1: every CTA works on one RVQ job; 0: contiguous tile ranges
};

__device__ unsigned int g_index_error;

// The kernels' dynamic shared memory (the staged codebook).
extern __shared__ uint4 g_dyn_smem[];

// ---------------------------------------------------------------------------
// Device pieces
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t load_code(const Job& job, int k, uint32_t n, bool& bad) {
    uint32_t c;
    size_t off = (size_t)k * job.stage_stride + n;
    if (job.index_bytes == 4) c = __ldg(reinterpret_cast<const uint8_t*>(job.idx) + (size_t)(n >> 2) * 16 + k * 4 + (n & 3));
    else if (job.index_bytes == 1) c = __ldg(reinterpret_cast<const uint8_t*>(job.idx) + off);
    else c = (uint16_t)__ldg(reinterpret_cast<const short*>(job.idx) + off);
    uint32_t nc = job.ncodes ? job.ncodes : 65536u;
    if (c >= nc) { bad = true; c = 0; }
    return c;
}

__device__ __forceinline__ float load_scale(const Job& job, uint32_t n) {
    uint32_t g = fastdiv(n, job.gv);
    return load_as_f32(job.scales, g, job.scale_kind);
}

// Store the 8 fp32 values of vector n (scale already applied).
__device__ __forceinline__ void store_vec(const Job& job, uint32_t n, const float (&v)[8]) {
    if (n < job.full_vecs && job.out_aligned) {
        if (job.out_kind == RVQ_F32) {
            float4* o = reinterpret_cast<float4*>(job.out) + (size_t)n * 2;
            o[0] = make_float4(v[0], v[1], v[2], v[3]);
            o[1] = make_float4(v[4], v[5], v[6], v[7]);
        } else {
            uint4 q;
            q.x = pack2(v[0], v[1], job.out_kind);
            q.y = pack2(v[2], v[3], job.out_kind);
            q.z = pack2(v[4], v[5], job.out_kind);
            q.w = pack2(v[6], v[7], job.out_kind);
            reinterpret_cast<uint4*>(job.out)[n] = q;
        }
        return;
    }
    uint64_t base = (uint64_t)n * 8;
#pragma unroll
    for (int t = 0; t < 8; ++t)
        if (base + t < job.trimmed) store_from_f32(job.out, (int64_t)(base + t), job.out_kind, v[t]);
}

// 16-byte slot of entry (k, c), copy p, in the fp16 staging (layouts above).
__device__ __forceinline__ uint32_t staged_slot(const Job& job, uint32_t k, uint32_t c, uint32_t p) {
    if (job.fast_ok) return ((k >> 1) << 12) | (c << 4) | ((k & 1) << 3) | p;
    const uint32_t nc = job.ncodes ? job.ncodes : 65536u;
    return ((k * nc + c) << job.copies_log2) + p;
}

// Stage job.cb into shared memory.  Returns the gather mode every thread of
// the CTA agrees on.  Must be called by all threads of the CTA.
__device__ int stage_codebook(const Job& job, uint4* smem) {
    const int n_entries = (int)job.stages * (job.ncodes ? (int)job.ncodes : 65536);
    const int copies = 1 << job.copies_log2;
    const int lane = threadIdx.x & 31;
    int inexact = 0;
    if (job.f16_fits) {
        for (int e = threadIdx.x; e < n_entries; e += blockDim.x) {
            uint4 q;
            if (job.cb_kind == RVQ_F16) {
                q = __ldg(reinterpret_cast<const uint4*>(job.cb) + e);
            } else {
                const float4* src = reinterpret_cast<const float4*>(job.cb) + (size_t)e * 2;
                float4 a = __ldg(src), b = __ldg(src + 1);
                float f[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
                uint32_t w[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    __half h0 = __float2half_rn(f[2 * i]), h1 = __float2half_rn(f[2 * i + 1]);
                    inexact |= (__float_as_uint(__half2float(h0)) != __float_as_uint(f[2 * i])) |
                               (__float_as_uint(__half2float(h1)) != __float_as_uint(f[2 * i + 1])) |
                               isnan(f[2 * i]) | isnan(f[2 * i + 1]);
                    w[i] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
                }
                q = make_uint4(w[0], w[1], w[2], w[3]);
            }
            // rotate the copy index with the lane so the 8 lanes of a phase
            // write 8 different bank quads
            const uint32_t nc = job.ncodes ? job.ncodes : 65536u;
            const uint32_t k = (uint32_t)e / nc, c = (uint32_t)e - k * nc;
            for (int i = 0; i < copies; ++i) {
                int cp = (i + lane) & (copies - 1);
                smem[staged_slot(job, k, c, (uint32_t)cp)] = q;
            }
        }
        inexact = __syncthreads_or(inexact);
        if (!inexact) return GATHER_SMEM_F16;
    }
    if (job.f32_fits && job.cb_kind == RVQ_F32) {
        if (job.f16_fits) __syncthreads();  // fp16 staging of this CTA is being replaced
        const uint4* src = reinterpret_cast<const uint4*>(job.cb);
        for (int e = threadIdx.x; e < n_entries * 2; e += blockDim.x) smem[e] = __ldg(src + e);
        __syncthreads();
        return GATHER_SMEM_F32;
    }
    __syncthreads();
    return GATHER_GLOBAL;
}

// Fast path: u8 indices over 256 codes, fp16 staging with 8 copies, K = 4
// stages (the compressor's default), 16-bit output (bf16 or fp16 fixed at
// compile time, so each pack is one conversion), a 32-byte aligned output,
// every vector of every tile complete.  Lane L owns vectors 4L .. 4L + 3 of
// the warp's tile: its index word of plane k holds their stage-k codes in
// bytes 0..3, and one prmt of that word with the lane's constant bits gives
// the byte offset of the staged entry (k / 2 << 16 | code << 8 | k % 2 << 7 |
// (L & 7) << 4).  The staged fp16 pairs are added into the fp32 accumulators
// with add.rn.f32.f16 on their register halves, the scale is applied with
// packed fp32x2 multiplies (same IEEE products), and vector pairs leave as
// 256-bit stores.  Each warp walks tiles ta + warp, ta + warp + 32, ... and
// loads the next tile's index words while it decodes the current one.
// SCALE4: group_vecs is a multiple of 4, so a lane's 4 vectors share a scale.
template <bool OUT_BF16, bool SCALE4>
__device__ __forceinline__ void run_fast(const Job& job, uint32_t ta, uint32_t tb, int warp, int lane,
                                         const char* smem) {
    // the few job fields the loop needs, read once from parameter space
    const uint32_t* idx32 = reinterpret_cast<const uint32_t*>(job.idx);
    const uint32_t plane32 = job.stage_stride >> 2;
    uint4* out = reinterpret_cast<uint4*>(job.out);
    const unsigned short* scales = reinterpret_cast<const unsigned short*>(job.scales);
    const FastDiv gv = job.gv;
    uint32_t lb[4];
#pragma unroll
    for (int k = 0; k < 4; ++k)
        lb[k] = ((uint32_t)(k & 1) << 7) | ((uint32_t)(lane & 7) << 4) | ((uint32_t)(k >> 1) << 16);
    uint32_t t = ta + warp;
    uint32_t w[4];
    // this lane's 4 code words of tile u (one word per plane)
    auto load_words = [&](uint32_t u, uint32_t (&o)[4]) {
#pragma unroll
        for (int k = 0; k < 4; ++k) o[k] = __ldg(idx32 + (size_t)k * plane32 + u * 32u + lane);
    };
    if (t < tb) load_words(t, w);
    for (; t < tb; t += kWarps) {
        uint32_t wn[4];
        if (t + kWarps < tb) load_words(t + kWarps, wn);
        const uint32_t n0 = t * kTileVecs + 4u * lane;
        float s4 = 0.f;
        if (SCALE4) s4 = __half2float(__ushort_as_half(__ldg(scales + fastdiv(n0, gv))));
        uint4 prev;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint4 q = *reinterpret_cast<const uint4*>(smem + __byte_perm(w[k], lb[k], 0x7604 | (i << 4)));
                add_f16x2_f32(acc[0], acc[1], q.x);
                add_f16x2_f32(acc[2], acc[3], q.y);
                add_f16x2_f32(acc[4], acc[5], q.z);
                add_f16x2_f32(acc[6], acc[7], q.w);
            }
            const float s = SCALE4 ? s4 : __half2float(__ushort_as_half(__ldg(scales + fastdiv(n0 + i, gv))));
            mul2_f32(acc[0], acc[1], s);
            mul2_f32(acc[2], acc[3], s);
            mul2_f32(acc[4], acc[5], s);
            mul2_f32(acc[6], acc[7], s);
            uint4 q;
            q.x = pack2(acc[0], acc[1], OUT_BF16 ? RVQ_BF16 : RVQ_F16);
            q.y = pack2(acc[2], acc[3], OUT_BF16 ? RVQ_BF16 : RVQ_F16);
            q.z = pack2(acc[4], acc[5], OUT_BF16 ? RVQ_BF16 : RVQ_F16);
            q.w = pack2(acc[6], acc[7], OUT_BF16 ? RVQ_BF16 : RVQ_F16);
            if (i & 1) store_v8_na(out + n0 + i - 1, prev, q);
            else prev = q;
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) w[k] = wn[k];
    }
}

// Generic tile: any stage count and gather mode.
__device__ void tile_generic(const Job& job, uint32_t tile, int lane, const uint4* smem, int mode) {
    const uint32_t v0 = tile * kTileVecs;
    const uint32_t cpy = lane & ((1u << job.copies_log2) - 1u);
    const uint32_t ncodes = job.ncodes ? job.ncodes : 65536u;
    bool bad = false;
    for (int j = 0; j < kJ; ++j) {
        uint32_t n = v0 + 32 * j + lane;
        if (n >= job.nvec) break;
        float acc[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) acc[t] = 0.0f;
        for (int k = 0; k < (int)job.stages; ++k) {
            uint32_t c = load_code(job, k, n, bad);
            uint32_t e = k * ncodes + c;
            float v[8];
            if (mode == GATHER_SMEM_F16) {
                uint4 q = smem[staged_slot(job, (uint32_t)k, c, cpy)];
                uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    v[2 * i] = __half2float(__ushort_as_half((uint16_t)(w[i] & 0xFFFFu)));
                    v[2 * i + 1] = __half2float(__ushort_as_half((uint16_t)(w[i] >> 16)));
                }
            } else if (mode == GATHER_SMEM_F32) {
                const float4* p = reinterpret_cast<const float4*>(smem) + (size_t)e * 2;
                float4 a = p[0], b = p[1];
                v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
                v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
            } else if (job.cb_kind == RVQ_F32) {
                const float4* p = reinterpret_cast<const float4*>(job.cb) + (size_t)e * 2;
                float4 a = __ldg(p), b = __ldg(p + 1);
                v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
                v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
            } else {
                uint4 q = __ldg(reinterpret_cast<const uint4*>(job.cb) + e);
                uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    v[2 * i] = __half2float(__ushort_as_half((uint16_t)(w[i] & 0xFFFFu)));
                    v[2 * i + 1] = __half2float(__ushort_as_half((uint16_t)(w[i] >> 16)));
                }
            }
#pragma unroll
            for (int t = 0; t < 8; ++t) acc[t] = __fadd_rn(acc[t], v[t]);
        }
        float s = load_scale(job, n);
#pragma unroll
        for (int t = 0; t < 8; ++t) acc[t] = __fmul_rn(acc[t], s);
        store_vec(job, n, acc);
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(&g_index_error, 1u);
}

__device__ void copy_tile(const Job& job, uint32_t tile, int lane) {
    const uint64_t begin = (uint64_t)tile * kCopyTileBytes;
    const uint64_t end = min((uint64_t)job.nvec, begin + kCopyTileBytes);
    const uint8_t* src = reinterpret_cast<const uint8_t*>(job.idx);
    uint8_t* dst = reinterpret_cast<uint8_t*>(job.out);
    bool aligned = ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0;
    if (aligned) {
        uint64_t vec_end = begin + ((end - begin) & ~15ull);
        for (uint64_t o = begin + 16ull * lane; o < vec_end; o += 16 * 32)
            *reinterpret_cast<uint4*>(dst + o) = __ldg(reinterpret_cast<const uint4*>(src + o));
        for (uint64_t o = vec_end + lane; o < end; o += 32) dst[o] = src[o];
    } else {
        for (uint64_t o = begin + lane; o < end; o += 32) dst[o] = src[o];
    }
}

__device__ void copy_tail(const Job& job) {
    for (uint32_t i = threadIdx.x; i < job.tail_numel; i += blockDim.x) {
        float v = load_as_f32(job.tail, i, job.tail_kind);
        store_from_f32(job.out, (int64_t)(job.trimmed + i), job.out_kind, v);
    }
}

// One warp tile (512 elements) of an int8_groupwise job: lane L owns elements
// 16 L .. 16 L + 15; out = cast(float(q) * float(scale)), the product one fp32
// multiply and the cast round-to-nearest-even (_decode_int8_into,
// infer_compressed_layerwise_single_slot.py:110-120).  fast_ok: q and out
// 16-byte aligned, 16-bit output and 16 | group_size (one scale per lane).
__device__ void int8_tile(const Job& job, uint32_t tile, int lane) {
    const uint32_t e0 = tile * kInt8TileElems + 16u * (uint32_t)lane;
    const int8_t* q = reinterpret_cast<const int8_t*>(job.idx);
    if (job.fast_ok && e0 + 16u <= job.nvec) {
        const int4 raw = __ldg(reinterpret_cast<const int4*>(q + e0));
        const float s = load_as_f32(job.scales, fastdiv(e0, job.gv), job.scale_kind);
        const uint32_t w[4] = {(uint32_t)raw.x, (uint32_t)raw.y, (uint32_t)raw.z, (uint32_t)raw.w};
        uint32_t o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float a = (float)(int8_t)(w[i >> 1] >> (16 * (i & 1)));
            const float b = (float)(int8_t)(w[i >> 1] >> (16 * (i & 1) + 8));
            o[i] = pack2(__fmul_rn(a, s), __fmul_rn(b, s), job.out_kind);
        }
        uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(job.out) + e0);
        dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
        dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
        return;
    }
    for (uint32_t i = 0; i < 16u; ++i) {
        const uint32_t e = e0 + i;
        if (e >= job.nvec) break;
        const float s = load_as_f32(job.scales, fastdiv(e, job.gv), job.scale_kind);
        store_from_f32(job.out, (int64_t)e, job.out_kind, __fmul_rn((float)q[e], s));
    }
}

// Tiles [a, e) (job-local) of one int8 job; `owner` copies the tail.
__device__ __forceinline__ void process_int8(const Job& job, uint32_t a, uint32_t e, bool owner, int warp,
                                             int lane) {
    if (owner) copy_tail(job);
    for (uint32_t t = a + warp; t < e; t += kWarps) int8_tile(job, t, lane);
}

// Decode tiles [a, e) (job-local) of one RVQ job; `owner` copies the tail.
// All threads of the CTA call it.
__device__ __forceinline__ void process_rvq(const Job& job, uint32_t a, uint32_t e, bool owner, int warp,
                                            int lane, uint4* smem, bool& staged_once) {
    if (job.nvec == 0) {                    // tail-only entry: nothing to stage
        if (owner) copy_tail(job);
        return;
    }
    if (staged_once) __syncthreads();       // readers of the previous codebook are done
    staged_once = true;
    const int mode = stage_codebook(job, smem);
    if (owner) copy_tail(job);
    uint32_t g = a;                         // first tile left for the generic path
    if (mode == GATHER_SMEM_F16 && job.fast_ok) {
        const uint32_t fe = min(e, job.full_tiles);
        if (a < fe) {
            const char* cs = reinterpret_cast<const char*>(smem);
            const bool s4 = (job.gv.d & 3u) == 0;
            if (job.out_kind == RVQ_BF16) {
                if (s4) run_fast<true, true>(job, a, fe, warp, lane, cs);
                else run_fast<true, false>(job, a, fe, warp, lane, cs);
            } else {
                if (s4) run_fast<false, true>(job, a, fe, warp, lane, cs);
                else run_fast<false, false>(job, a, fe, warp, lane, cs);
            }
            g = fe;
        }
    }
    for (uint32_t t = g + warp; t < e; t += kWarps) tile_generic(job, t, lane, smem, mode);
}

__global__ void __launch_bounds__(kThreads, 1) rvq_layer_kernel(const __grid_constant__ LayerParams p) {
    extern __shared__ uint4 smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t G = gridDim.x, b = blockIdx.x;
    bool staged_once = false;
    if (p.per_cta_jobs) {
        // raw copies first (each owned by one CTA), then this CTA's share of its RVQ job
        for (int j = 0; j < p.njobs; ++j) {
            const Job& job = p.jobs[j];
            if (job.kind == JOB_COPY && job.cta_begin == b)
                for (uint32_t t = warp; t < job.tile_count; t += kWarps) copy_tile(job, t, lane);
        }
        for (int j = 0; j < p.njobs; ++j) {
            const Job& job = p.jobs[j];
            if (job.kind == JOB_COPY || b < job.cta_begin || b >= job.cta_begin + job.cta_count) continue;
            const uint32_t r = b - job.cta_begin, cc = job.cta_count, tc = job.tile_count;
            const uint32_t a = (uint32_t)(((uint64_t)tc * r) / cc), e = (uint32_t)(((uint64_t)tc * (r + 1)) / cc);
            if (job.kind == JOB_INT8) process_int8(job, a, e, r == 0, warp, lane);
            else process_rvq(job, a, e, r == 0, warp, lane, smem, staged_once);
        }
        return;
    }
    const uint32_t T = p.total_tiles;
    const uint32_t t0 = (uint32_t)(((uint64_t)T * b) / G);
    const uint32_t t1 = (uint32_t)(((uint64_t)T * (b + 1)) / G);
    for (int j = 0; j < p.njobs; ++j) {
        const uint32_t jb = p.jobs[j].tile_begin, je = jb + p.jobs[j].tile_count;
        const uint32_t a = max(t0, jb), e = min(t1, je);
        if (a >= e) continue;
        const Job& job = p.jobs[j];
        if (job.kind == JOB_COPY) {
            for (uint32_t t = a + warp; t < e; t += kWarps) copy_tile(job, t - jb, lane);
            continue;
        }
        if (job.kind == JOB_INT8) {
            process_int8(job, a - jb, e - jb, a == jb, warp, lane);
            continue;
        }
        process_rvq(job, a - jb, e - jb, a == jb, warp, lane, smem, staged_once);
    }
}

// ---------------------------------------------------------------------------
// The slot kernel: a layer slot whose RVQ entries all have quad-layout codes,
// an fp16 codebook, fp16 scales and whole vectors, decoded into bf16 -- what a
// layer plan uploads, with a multiple of 4 vectors per scale -- plus its raw copies.  The same arithmetic and
// schedule as the fast path of rvq_layer_kernel, in a kernel that holds
// nothing else, so the hot loop keeps every value in registers.  Lane L owns
// vectors 4L .. 4L + 3 of a 128-vector tile and gets their 16 stage codes
// with one 16-byte load; the last tile of an entry may be partial (the quad
// buffer is zero-padded; stores and scale reads past nvec are skipped).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void slot_stage(const Job& job, char* smem) {
    const int lane = threadIdx.x & 31;
    for (int e = threadIdx.x; e < 4 * 256; e += blockDim.x) {
        const uint4 q = __ldg(reinterpret_cast<const uint4*>(job.cb) + e);
        char* base = smem + ((e >> 9) << 16) + ((e & 255) << 8) + (((e >> 8) & 1) << 7);
#pragma unroll
        for (int i = 0; i < 8; ++i) *reinterpret_cast<uint4*>(base + (((i + lane) & 7) << 4)) = q;
    }
}

__device__ __forceinline__ void slot_tiles(const Job& job, uint32_t ta, uint32_t tb, int warp, int lane) {
    const char* smem = reinterpret_cast<const char*>(g_dyn_smem);
    const uint4* quads = reinterpret_cast<const uint4*>(job.idx);
    uint4* out = reinterpret_cast<uint4*>(job.out);
    const unsigned short* scales = reinterpret_cast<const unsigned short*>(job.scales);
    const FastDiv gv = job.gv;
    const uint32_t nvec = job.nvec;
    uint32_t lb[4];
#pragma unroll
    for (int k = 0; k < 4; ++k)
        lb[k] = ((uint32_t)(k & 1) << 7) | ((uint32_t)(lane & 7) << 4) | ((uint32_t)(k >> 1) << 16);
    uint32_t t = ta + warp;
    uint4 w;
    if (t < tb) w = __ldg(quads + t * 32u + lane);
    for (; t < tb; t += kWarps) {
        uint4 wn;
        if (t + kWarps < tb) wn = __ldg(quads + (t + kWarps) * 32u + lane);
        const uint32_t n0 = t * kTileVecs + 4u * lane;
        const bool whole = n0 + 4u <= nvec;
        // group_vecs is a multiple of 4: the lane's 4 vectors share one scale
        const float s = n0 < nvec ? __half2float(__ushort_as_half(__ldg(scales + fastdiv(n0, gv)))) : 0.f;
        const uint32_t wk[4] = {w.x, w.y, w.z, w.w};
        uint4 prev;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint4 q = *reinterpret_cast<const uint4*>(smem + __byte_perm(wk[k], lb[k], 0x7604 | (i << 4)));
                add_f16x2_f32(acc[0], acc[1], q.x);
                add_f16x2_f32(acc[2], acc[3], q.y);
                add_f16x2_f32(acc[4], acc[5], q.z);
                add_f16x2_f32(acc[6], acc[7], q.w);
            }
            mul2_f32(acc[0], acc[1], s);
            mul2_f32(acc[2], acc[3], s);
            mul2_f32(acc[4], acc[5], s);
            mul2_f32(acc[6], acc[7], s);
            uint4 q;
            q.x = pack2(acc[0], acc[1], RVQ_BF16);
            q.y = pack2(acc[2], acc[3], RVQ_BF16);
            q.z = pack2(acc[4], acc[5], RVQ_BF16);
            q.w = pack2(acc[6], acc[7], RVQ_BF16);
            if (i & 1) {
                if (whole) store_v8_na(out + n0 + i - 1, prev, q);
                else {                                  // the partial last tile of the entry
                    if (n0 + i - 1 < nvec) out[n0 + i - 1] = prev;
                    if (n0 + i < nvec) out[n0 + i] = q;
                }
            } else {
                prev = q;
            }
        }
        w = wn;
    }
}

__global__ void __launch_bounds__(kThreads, 1) rvq_slot_kernel(const __grid_constant__ LayerParams p) {
    char* smem = reinterpret_cast<char*>(g_dyn_smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t b = blockIdx.x;
    // raw copies first (each owned by one CTA), then this CTA's share of its RVQ job
    for (int j = 0; j < p.njobs; ++j) {
        const Job& job = p.jobs[j];
        if (job.kind == JOB_COPY && job.cta_begin == b)
            for (uint32_t t = warp; t < job.tile_count; t += kWarps) copy_tile(job, t, lane);
    }
    for (int j = 0; j < p.njobs; ++j) {
        const Job& job = p.jobs[j];
        if (job.kind != JOB_RVQ || b < job.cta_begin || b >= job.cta_begin + job.cta_count) continue;
        const uint32_t r = b - job.cta_begin, cc = job.cta_count, tc = job.tile_count;
        const uint32_t a = (uint32_t)(((uint64_t)tc * r) / cc), e = (uint32_t)(((uint64_t)tc * (r + 1)) / cc);
        slot_stage(job, smem);
        __syncthreads();
        if (r == 0) copy_tail(job);
        slot_tiles(job, a, e, warp, lane);
        return;                                  // the job-per-CTA schedule gives a CTA one RVQ job
    }
}

// Quad layout: out[q] = the 4 stage words of vectors 4q .. 4q + 3 (byte 4 k + j
// = stage k's code of vector 4 q + j), zero past nvec up to a whole 128-vector
// tile (32 quads), so tile loads never leave the buffer.  One thread per quad.
__global__ void quad_codes_kernel(const uint8_t* __restrict__ planes, int64_t stride, int64_t nvec,
                                  uint4* __restrict__ out) {
    const int64_t quads = (nvec + kTileVecs - 1) / kTileVecs * (kTileVecs / 4);
    for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < quads; q += (int64_t)gridDim.x * blockDim.x) {
        uint32_t w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            uint32_t v = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int64_t n = 4 * q + j;
                if (n < nvec) v |= (uint32_t)planes[k * stride + n] << (8 * j);
            }
            w[k] = v;
        }
        out[q] = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

struct DeviceInfo {
    bool ready = false;
    bool ok = false;
    int sm_count = 0;
    int max_smem = 0;
};

static DeviceInfo g_devices[kMaxDevices];
static std::mutex g_dev_mutex;

static int cuda_fail(cudaError_t e) {
    last_cuda_error_slot() = (int)e;
    return RVQ_ERR_CUDA;
}

// Per-device set-up: SM count, opt-in shared memory, kernel attribute.
static int device_info(DeviceInfo** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) { last_cuda_error_slot() = (int)e; return RVQ_ERR_UNAVAILABLE; }
    if (dev < 0 || dev >= kMaxDevices) return RVQ_ERR_UNAVAILABLE;
    DeviceInfo& di = g_devices[dev];
    std::lock_guard<std::mutex> lock(g_dev_mutex);
    if (!di.ready) {
        di.ready = true;
        cudaDeviceProp prop;
        e = cudaGetDeviceProperties(&prop, dev);
        if (e != cudaSuccess || prop.major != 10) {
            if (e != cudaSuccess) last_cuda_error_slot() = (int)e;
            di.ok = false;
        } else {
            di.sm_count = prop.multiProcessorCount;
            cudaFuncAttributes fa;
            e = cudaFuncGetAttributes(&fa, rvq_layer_kernel);
            // dynamic shared memory may use what the kernel's static shared memory leaves
            di.max_smem = (int)prop.sharedMemPerBlockOptin - (e == cudaSuccess ? (int)fa.sharedSizeBytes : 0);
            if (e == cudaSuccess)
                e = cudaFuncSetAttribute(rvq_layer_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         di.max_smem);
            if (e == cudaSuccess)
                e = cudaFuncSetAttribute(rvq_slot_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         di.max_smem);
            di.ok = (e == cudaSuccess);
            if (e != cudaSuccess) last_cuda_error_slot() = (int)e;
        }
    }
    if (!di.ok) return RVQ_ERR_UNAVAILABLE;
    *out = &di;
    return RVQ_OK;
}

static bool is_float_kind(int k) { return k == RVQ_F16 || k == RVQ_BF16 || k == RVQ_F32; }

static int check_entry(const rvq_entry* e) {
    if (!e) return RVQ_ERR_INVALID;
    if (e->d != 8) return RVQ_ERR_UNSUPPORTED;
    if (!is_float_kind(e->out_kind)) return RVQ_ERR_UNSUPPORTED;
    if (e->index_kind != RVQ_U8 && e->index_kind != RVQ_I16 && e->index_kind != RVQ_U8X4) return RVQ_ERR_UNSUPPORTED;
    if (e->index_kind == RVQ_U8X4 && (e->stages != 4 || e->ncodes > 256 || ((uintptr_t)e->indices & 15)))
        return RVQ_ERR_INVALID;
    if (e->codebook_kind != RVQ_F16 && e->codebook_kind != RVQ_F32) return RVQ_ERR_UNSUPPORTED;
    if (!is_float_kind(e->scale_kind) || !is_float_kind(e->tail_kind)) return RVQ_ERR_UNSUPPORTED;
    if (e->stages < 1 || e->stages > 65535 || e->ncodes < 1 || e->ncodes > 65536) return RVQ_ERR_INVALID;
    if (e->index_kind == RVQ_U8 && e->ncodes > 256) return RVQ_ERR_INVALID;
    if (e->nvec < 0 || e->tail_numel < 0 || e->trimmed < 0 || e->group_vecs < 1) return RVQ_ERR_INVALID;
    if (e->nvec >= (1ll << 31) || e->group_vecs >= (1ll << 31) || e->tail_numel >= (1ll << 31))
        return RVQ_ERR_TOO_LARGE;
    if (e->stage_stride < e->nvec || (int64_t)e->stages * e->stage_stride >= (1ll << 40)) return RVQ_ERR_INVALID;
    if (e->trimmed > e->nvec * 8) return RVQ_ERR_INVALID;
    if (!e->out) return RVQ_ERR_INVALID;
    if (e->nvec > 0 && (!e->indices || !e->codebook || !e->scales)) return RVQ_ERR_INVALID;
    if (e->tail_numel > 0 && !e->tail) return RVQ_ERR_INVALID;
    if (e->codebook && ((uintptr_t)e->codebook & 15)) return RVQ_ERR_INVALID;
    return RVQ_OK;
}

static int check_int8_entry(const rvq_int8_entry* e) {
    if (!e) return RVQ_ERR_INVALID;
    if (!is_float_kind(e->out_kind) || !is_float_kind(e->scale_kind) || !is_float_kind(e->tail_kind))
        return RVQ_ERR_UNSUPPORTED;
    if (e->trimmed < 0 || e->tail_numel < 0 || e->group_size < 1) return RVQ_ERR_INVALID;
    if (e->trimmed % e->group_size != 0) return RVQ_ERR_INVALID;
    if (e->trimmed >= (1ll << 31) || e->tail_numel >= (1ll << 31) || e->group_size >= (1ll << 31))
        return RVQ_ERR_TOO_LARGE;
    if (!e->out) return RVQ_ERR_INVALID;
    if (e->trimmed > 0 && (!e->q || !e->scales)) return RVQ_ERR_INVALID;
    if (e->tail_numel > 0 && !e->tail) return RVQ_ERR_INVALID;
    return RVQ_OK;
}

static void fill_int8_job(const rvq_int8_entry* e, Job& j) {
    memset(&j, 0, sizeof(j));
    j.kind = JOB_INT8;
    j.idx = e->q;
    j.scales = e->scales;
    j.tail = e->tail;
    j.out = e->out;
    j.nvec = (uint32_t)e->trimmed;
    j.gv = make_fastdiv((uint32_t)e->group_size);
    j.trimmed = (uint64_t)e->trimmed;
    j.tail_numel = (uint32_t)e->tail_numel;
    j.scale_kind = (uint8_t)e->scale_kind;
    j.tail_kind = (uint8_t)e->tail_kind;
    j.out_kind = (uint8_t)e->out_kind;
    j.out_aligned = ((uintptr_t)e->out & 15) == 0;
    j.fast_ok = j.out_aligned && ((uintptr_t)e->q & 15) == 0 && e->group_size % 16 == 0 &&
                (e->out_kind == RVQ_BF16 || e->out_kind == RVQ_F16);
    uint32_t tiles = (uint32_t)((e->trimmed + kInt8TileElems - 1) / kInt8TileElems);
    if (tiles == 0 && e->tail_numel > 0) tiles = 1;
    j.tile_count = tiles;
}

static size_t stage_bytes_f16(int copies_log2, int64_t entries) { return (size_t)entries * 16u << copies_log2; }

static int fill_rvq_job(const rvq_entry* e, Job& j, size_t& smem_need) {
    memset(&j, 0, sizeof(j));
    j.kind = JOB_RVQ;
    j.idx = e->indices;
    j.cb = e->codebook;
    j.scales = e->scales;
    j.tail = e->tail;
    j.out = e->out;
    j.nvec = (uint32_t)e->nvec;
    j.stage_stride = (uint32_t)e->stage_stride;
    if (e->stage_stride >= (1ll << 32)) return RVQ_ERR_TOO_LARGE;
    j.gv = make_fastdiv((uint32_t)e->group_vecs);
    j.trimmed = (uint64_t)e->trimmed;
    j.full_vecs = (uint32_t)(e->trimmed / 8);
    j.tail_numel = (uint32_t)e->tail_numel;
    j.stages = (uint16_t)e->stages;
    j.ncodes = (uint16_t)(e->ncodes == 65536 ? 0 : e->ncodes);
    j.index_bytes = (uint8_t)(e->index_kind == RVQ_U8 ? 1 : (e->index_kind == RVQ_U8X4 ? 4 : 2));
    j.cb_kind = (uint8_t)e->codebook_kind;
    j.scale_kind = (uint8_t)e->scale_kind;
    j.tail_kind = (uint8_t)e->tail_kind;
    j.out_kind = (uint8_t)e->out_kind;
    j.out_aligned = ((uintptr_t)e->out & 15) == 0;
    const int64_t entries = (int64_t)e->stages * e->ncodes;
    int cl = 3;
    while (cl > 0 && stage_bytes_f16(cl, entries) > (size_t)kSmemBudget) --cl;
    j.copies_log2 = (uint8_t)cl;
    j.f16_fits = stage_bytes_f16(cl, entries) <= (size_t)kSmemBudget;
    j.f32_fits = (size_t)entries * 32u <= (size_t)kSmemBudget;
    size_t need = 0;
    if (j.f16_fits) need = stage_bytes_f16(cl, entries);
    if (j.cb_kind == RVQ_F32 && j.f32_fits) need = need > (size_t)entries * 32u ? need : (size_t)entries * 32u;
    if (need > smem_need) smem_need = need;
    uint32_t tiles = (uint32_t)((e->nvec + kTileVecs - 1) / kTileVecs);
    if (tiles == 0 && e->tail_numel > 0) tiles = 1;
    j.tile_count = tiles;
    const uint64_t complete = (uint64_t)(e->nvec < (int64_t)j.full_vecs ? e->nvec : j.full_vecs);
    j.full_tiles = (uint32_t)(complete / kTileVecs);
    const bool planes_ok = e->index_kind == RVQ_U8 && ((uintptr_t)e->indices & 3) == 0 && (e->stage_stride & 3) == 0 &&
                           (e->out_kind == RVQ_BF16 || e->out_kind == RVQ_F16);
    j.fast_ok = planes_ok && e->ncodes == 256 && e->stages == 4 && cl == 3 && ((uintptr_t)e->out & 31) == 0 &&
                e->scale_kind == RVQ_F16;
    // the slot kernel: quad codes, fp16 codebook (staged exactly), bf16 slot, whole vectors,
    // 4 | group_vecs
    j.slot_ok = e->index_kind == RVQ_U8X4 && e->ncodes == 256 && e->codebook_kind == RVQ_F16 &&
                e->out_kind == RVQ_BF16 && e->scale_kind == RVQ_F16 && ((uintptr_t)e->out & 31) == 0 &&
                e->trimmed == e->nvec * 8 && e->nvec > 0 && e->group_vecs % 4 == 0;
    return RVQ_OK;
}

// Job-per-CTA schedule: every RVQ job gets a number of CTAs proportional
// to its tiles (largest remainder, at least one), so no CTA restages a
// codebook or waits at a job boundary.  Returns the grid size, or 0 when
// the jobs do not fit that scheme (more RVQ jobs than half the SMs).
static uint32_t plan_per_cta(LayerParams& p, uint32_t sms) {
    uint32_t n_rvq = 0;
    uint64_t total = 0;
    for (int i = 0; i < p.njobs; ++i)
        if (p.jobs[i].kind != JOB_COPY && p.jobs[i].tile_count) { ++n_rvq; total += p.jobs[i].tile_count; }
    if (n_rvq == 0 || 2 * n_rvq > sms) return 0;
    double ideal[RVQ_MAX_LAYER_JOBS] = {0};
    uint32_t cnt[RVQ_MAX_LAYER_JOBS] = {0};
    uint32_t sum = 0;
    for (int i = 0; i < p.njobs; ++i) {
        const Job& j = p.jobs[i];
        if (j.kind == JOB_COPY || !j.tile_count) continue;
        ideal[i] = (double)sms * j.tile_count / (double)total;
        uint32_t c = (uint32_t)ideal[i];
        if (c < 1) c = 1;
        if (c > j.tile_count) c = j.tile_count;
        cnt[i] = c;
        sum += c;
    }
    while (sum > sms) {                     // at-least-one rounding overshot: take from the richest
        int best = -1;
        double bd = -1e30;
        for (int i = 0; i < p.njobs; ++i)
            if (cnt[i] > 1 && cnt[i] - ideal[i] > bd) { bd = cnt[i] - ideal[i]; best = i; }
        if (best < 0) return 0;
        --cnt[best];
        --sum;
    }
    while (sum < sms) {                     // hand out the rest by largest remainder
        int best = -1;
        double bd = -1e30;
        for (int i = 0; i < p.njobs; ++i)
            if (p.jobs[i].kind != JOB_COPY && cnt[i] && cnt[i] < p.jobs[i].tile_count && ideal[i] - cnt[i] > bd) {
                bd = ideal[i] - cnt[i];
                best = i;
            }
        if (best < 0) break;
        ++cnt[best];
        ++sum;
    }
    uint32_t begin = 0, copy_owner = 0;
    for (int i = 0; i < p.njobs; ++i) {
        Job& j = p.jobs[i];
        if (j.kind != JOB_COPY) {
            j.cta_begin = begin;
            j.cta_count = cnt[i];
            begin += cnt[i];
        }
    }
    for (int i = 0; i < p.njobs; ++i)
        if (p.jobs[i].kind == JOB_COPY) p.jobs[i].cta_begin = (copy_owner++) % (begin ? begin : 1);
    return begin;
}

static int launch_jobs(LayerParams& p, size_t smem_need, int max_ctas, void* stream) {
    DeviceInfo* di = nullptr;
    int rc = device_info(&di);
    if (rc != RVQ_OK) return rc;
    const uint32_t ctas = (max_ctas > 0 && max_ctas < di->sm_count) ? (uint32_t)max_ctas : (uint32_t)di->sm_count;
    uint32_t total = 0;
    for (int i = 0; i < p.njobs; ++i) {
        p.jobs[i].tile_begin = total;
        total += p.jobs[i].tile_count;
    }
    p.total_tiles = total;
    if (total == 0) return RVQ_OK;
    if (smem_need > (size_t)di->max_smem) return RVQ_ERR_TOO_LARGE;
    uint32_t grid = plan_per_cta(p, ctas);
    p.per_cta_jobs = grid ? 1u : 0u;
    bool slot = grid != 0;
    for (int i = 0; i < p.njobs && slot; ++i)
        if (p.jobs[i].kind == JOB_INT8 || (p.jobs[i].kind == JOB_RVQ && !p.jobs[i].slot_ok)) slot = false;
    if (!grid) {
        grid = ctas;
        if (grid > total) grid = total;
    }
    if (slot) rvq_slot_kernel<<<grid, kThreads, smem_need, (cudaStream_t)stream>>>(p);
    else rvq_layer_kernel<<<grid, kThreads, smem_need, (cudaStream_t)stream>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
    return RVQ_OK;
}

}  // namespace rvq

using namespace rvq;

extern "C" {

int rvq_available(void) {
    DeviceInfo* di = nullptr;
    return device_info(&di) == RVQ_OK ? 1 : 0;
}

int rvq_check_entry(const rvq_entry* e) { return check_entry(e); }

int rvq_decode(const rvq_entry* e, void* stream) {
    return rvq_decode_layer(e, 1, nullptr, 0, stream);
}

int rvq_decode_layer(const rvq_entry* entries, int n_entries, const rvq_copy* copies, int n_copies,
                     void* stream) {
    return rvq_decode_layer_mixed(entries, n_entries, nullptr, 0, copies, n_copies, stream);
}

int rvq_check_int8_entry(const rvq_int8_entry* e) { return check_int8_entry(e); }

int rvq_decode_int8(const rvq_int8_entry* e, void* stream) {
    return rvq_decode_layer_mixed(nullptr, 0, e, 1, nullptr, 0, stream);
}

int rvq_decode_layer_mixed(const rvq_entry* entries, int n_entries, const rvq_int8_entry* int8s, int n_int8,
                           const rvq_copy* copies, int n_copies, void* stream) {
    return rvq_decode_layer_ctas(entries, n_entries, int8s, n_int8, copies, n_copies, 0, stream);
}

int rvq_decode_layer_ctas(const rvq_entry* entries, int n_entries, const rvq_int8_entry* int8s, int n_int8,
                          const rvq_copy* copies, int n_copies, int max_ctas, void* stream) {
    if (max_ctas < 0) return RVQ_ERR_INVALID;
    if (n_entries < 0 || n_int8 < 0 || n_copies < 0 || n_entries + n_int8 + n_copies > RVQ_MAX_LAYER_JOBS)
        return RVQ_ERR_INVALID;
    if ((n_entries && !entries) || (n_int8 && !int8s) || (n_copies && !copies)) return RVQ_ERR_INVALID;
    LayerParams p;
    memset(&p, 0, sizeof(p));
    size_t smem = 0;
    for (int i = 0; i < n_entries; ++i) {
        int rc = check_entry(&entries[i]);
        if (rc != RVQ_OK) return rc;
        rc = fill_rvq_job(&entries[i], p.jobs[p.njobs], smem);
        if (rc != RVQ_OK) return rc;
        p.njobs++;
    }
    for (int i = 0; i < n_int8; ++i) {
        const int rc = check_int8_entry(&int8s[i]);
        if (rc != RVQ_OK) return rc;
        fill_int8_job(&int8s[i], p.jobs[p.njobs++]);
    }
    for (int i = 0; i < n_copies; ++i) {
        const rvq_copy& c = copies[i];
        if (c.nbytes < 0 || c.nbytes >= (1ll << 31)) return RVQ_ERR_INVALID;
        if (c.nbytes == 0) continue;
        if (!c.src || !c.dst) return RVQ_ERR_INVALID;
        Job& j = p.jobs[p.njobs++];
        memset(&j, 0, sizeof(j));
        j.kind = JOB_COPY;
        j.idx = c.src;
        j.out = c.dst;
        j.nvec = (uint32_t)c.nbytes;
        j.tile_count = (uint32_t)((c.nbytes + kCopyTileBytes - 1) / kCopyTileBytes);
    }
    return launch_jobs(p, smem, max_ctas, stream);
}

int64_t rvq_quad_codes_bytes(int64_t nvec) { return nvec < 1 ? 0 : (nvec + kTileVecs - 1) / kTileVecs * kTileVecs * 4; }

int rvq_quad_codes(const void* planes, int64_t stage_stride, int64_t nvec, void* out, void* stream) {
    if (!planes || !out || nvec < 1 || stage_stride < nvec || ((uintptr_t)out & 15)) return RVQ_ERR_INVALID;
    const int64_t quads = (nvec + kTileVecs - 1) / kTileVecs * (kTileVecs / 4);
    const int64_t blocks64 = (quads + 255) / 256;
    const unsigned blocks = (unsigned)(blocks64 < 148 * 32 ? blocks64 : 148 * 32);
    quad_codes_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(reinterpret_cast<const uint8_t*>(planes), stage_stride,
                                                               nvec, reinterpret_cast<uint4*>(out));
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
    return RVQ_OK;
}

int rvq_take_index_error(void) {
    unsigned int v = 0, zero = 0;
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) { last_cuda_error_slot() = (int)e; return -RVQ_ERR_CUDA; }
    e = cudaMemcpyFromSymbol(&v, g_index_error, sizeof(v));
    if (e != cudaSuccess) { last_cuda_error_slot() = (int)e; return -RVQ_ERR_CUDA; }
    e = cudaMemcpyToSymbol(g_index_error, &zero, sizeof(zero));
    if (e != cudaSuccess) { last_cuda_error_slot() = (int)e; return -RVQ_ERR_CUDA; }
    return v ? 1 : 0;
}

int rvq_last_cuda_error(void) { return last_cuda_error_slot(); }

const char* rvq_status_string(int status) {
    switch (status) {
        case RVQ_OK: return "ok";
        case RVQ_ERR_INVALID: return "invalid argument";
        case RVQ_ERR_UNSUPPORTED: return "unsupported entry";
        case RVQ_ERR_UNAVAILABLE: return "no usable sm_100 CUDA device";
        case RVQ_ERR_CUDA: return "CUDA runtime error";
        case RVQ_ERR_TOO_LARGE: return "size exceeds a limit";
        default: return "unknown status";
    }
}

int rvq_version(void) { return 100; }

// Host-side mirror of the device division, exported for CPU tests.
uint32_t rvq_test_fastdiv(uint32_t d, uint32_t n) {
    FastDiv f = make_fastdiv(d);
    return fastdiv(n, f);
}

}  // extern "C"
