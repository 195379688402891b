// Batch-1 table GEMV (rvq_gemv_tiles): constants, the job and launch
// parameters, the device-side unit (code-word ring, table build, row sums)
// and the host-side unit planner.  Included by rvq_gemv_tiles.cu (the plain
// launch) and rvq_persist.cu (the persistent decode step).
#pragma once

#include <string.h>

#include "rvq_common.cuh"

namespace rvq {
namespace tiles {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr int kGroups = 32;                                 // 8-element groups per tile
constexpr int kTileCols = kGroups * 8;                      // 256 columns
constexpr int kStages = 4;
constexpr int kCodes = 256;
constexpr int kPairs = kStages * kCodes;                    // (stage, code) codebook rows
constexpr int kLutWords = kCodes * (kStages / 2) * kGroups; // 16384 words (2 fp16 entries each), 64 KB
constexpr int kCbFloats = kPairs * 8;                       // codebook, fp32, 32 KB
constexpr int kBatchRows = 256;                             // rows per staged batch
constexpr int kRing = 4;                                    // ring slots
constexpr int kMaxJobs = 4;
constexpr int kMaxUnits = 1024;
constexpr int kMaxCtas = 160;
constexpr int kSwitchRows = 768;                            // starting a unit (table build, first batch) ~ 768 rows
constexpr long long kWaitLimit = 1ll << 22;                 // mbarrier polls before giving up
constexpr int kLineWords = 32;                              // code words per row of a tile (128 B)
// [table 64 KB][codebook 32 KB][ring slots 0..3][x slice][barriers]
constexpr size_t kSmemBytes =
    (size_t)(kLutWords + kCbFloats + kRing * kBatchRows * kGroups + kTileCols) * 4 + 64;
// operand partial tiles staged in the table's space before the table is built
constexpr int kMaxStagedTiles = kLutWords / kTileCols;

// sticky: a TMA wait gave up (one flag per translation unit that includes this file)
static __device__ int g_wait_timeout;

struct TJob {
    const uint32_t* codes;      // [ntiles][rows][32] code words (rvq_tile_codes)
    const void* cb;             // [4][256][8]
    const void* scales;
    rvq_vec x;                  // operand (or the "up" half when gate is set)
    rvq_vec gate;               // gate.ptr != null: operand = bf16(bf16(silu(gate)) * x)
    float* part;                // [ntiles][rows]
    int64_t cols;
    int32_t rows;
    int32_t G;                  // groups per row = cols / 8
    FastDiv gvdiv;              // vectors per scale
    FastDiv rpsdiv;             // rows per scale, when a scale never changes along a row
    int32_t row_scales;         // 1: scale index = row / rows_per_scale
    int32_t cb_kind;
    int32_t scale_kind;
};

struct TParams {
    TJob jobs[kMaxJobs];
    int32_t n_units;
    int32_t n_ctas;
    int32_t cta_first[kMaxCtas + 1];  // CTA c runs units [cta_first[c], cta_first[c + 1])
    uint32_t unit_jt[kMaxUnits];  // job << 24 | tile
    int32_t unit_r0[kMaxUnits];
    int32_t unit_r1[kMaxUnits];
};

__device__ __forceinline__ float bf16r(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// Operands are read through L2 (ld.global.cg): the persistent decode step
// reads vectors that other CTAs of the same launch wrote.
__device__ __forceinline__ float ldcg_as_f32(const void* p, int64_t i, int kind) {
    if (kind == RVQ_F32) return __ldcg(reinterpret_cast<const float*>(p) + i);
    const unsigned short u = __ldcg(reinterpret_cast<const unsigned short*>(p) + i);
    return kind == RVQ_F16 ? __half2float(__ushort_as_half(u)) : __bfloat162float(__ushort_as_bfloat16(u));
}

__device__ __forceinline__ float operand(const rvq_vec& v, int64_t i) {
    if (v.kind == RVQ_F32) {
        const float* p = reinterpret_cast<const float*>(v.ptr);
        float s = __ldcg(p + i);
        for (int t = 1; t < v.ntiles; ++t) s += __ldcg(p + (int64_t)t * v.n + i);
        return bf16r(s);
    }
    return ldcg_as_f32(v.ptr, i, v.kind);
}

// All ntiles x 256 partials of the tile's operand slice into dst[t][c] (zero
// past the matrix edge), 8 independent loads per thread in flight.
__device__ __forceinline__ void stage_partials(const rvq_vec& v, int tile, int64_t cols, float* dst) {
    const float* p = reinterpret_cast<const float*>(v.ptr);
    const int total = v.ntiles * kTileCols;
    for (int i0 = threadIdx.x; i0 < total; i0 += 8 * kThreads) {
        float r[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int i = i0 + k * kThreads;
            const int t = i >> 8;
            const int64_t col = (int64_t)tile * kTileCols + (i & (kTileCols - 1));
            r[k] = (i < total && col < cols) ? __ldcg(p + (int64_t)t * v.n + col) : 0.f;
        }
#pragma unroll
        for (int k = 0; k < 8; ++k)
            if (i0 + k * kThreads < total) dst[i0 + k * kThreads] = r[k];
    }
}

// The tile-ordered sum of staged partials for column c, rounded to bf16.
__device__ __forceinline__ float staged_value(const float* src, int ntiles, int c) {
    float s = src[c];
    for (int t = 1; t < ntiles; ++t) s += src[t * kTileCols + c];
    return bf16r(s);
}

// Byte offset in the table of the entry for the code in byte K of `w`;
// `lane_bits` = (K / 2) << 7 | lane << 2 | (K % 2) << 1.
template <int K>
__device__ __forceinline__ uint32_t lut_offset(uint32_t w, uint32_t lane_bits) {
    return __byte_perm(w, lane_bits, 0x7604 | (K << 4));
}

__device__ __forceinline__ unsigned short lut_entry(const uint32_t* lut, uint32_t byte_offset) {
    return *reinterpret_cast<const unsigned short*>(reinterpret_cast<const char*>(lut) + byte_offset);
}

// acc + entry, one fp32 round-to-nearest add of the fp16 entry.
__device__ __forceinline__ float add_entry(float acc, unsigned short h) {
    asm("add.rn.f32.f16 %0, %1, %0;" : "+f"(acc) : "h"(h));
    return acc;
}

// The four stage entries of one code word, summed in stage order.
__device__ __forceinline__ float lookup4(const uint32_t* lut, uint32_t w, uint32_t lb0, uint32_t lb1, uint32_t lb2,
                                         uint32_t lb3) {
    float s = __half2float(__ushort_as_half(lut_entry(lut, lut_offset<0>(w, lb0))));
    s = add_entry(s, lut_entry(lut, lut_offset<1>(w, lb1)));
    s = add_entry(s, lut_entry(lut, lut_offset<2>(w, lb2)));
    return add_entry(s, lut_entry(lut, lut_offset<3>(w, lb3)));
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }

template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

__device__ __forceinline__ void mbar_init(uint32_t bar) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: false (and the sticky flag set) if the phase never completed;
// then one more bounded wait, so that a late copy lands before the CTA moves on.
// After a false return the caller issues no further copies and waits for none:
// the launch's results are undefined apart from the flag, and a copy that never
// completed may still be in flight when the CTA exits.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    for (long long i = 0; i < kWaitLimit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    atomicExch(&g_wait_timeout, 1);
    for (long long i = 0; i < kWaitLimit; ++i)
        if (mbar_try_wait(bar, parity)) break;
    return false;
}

// `bytes` (a multiple of 16) of contiguous code words into shared memory,
// completing on the mbarrier.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    mbar_expect_tx(bar, bytes);
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

// Rows [r, r + n) of a tile's code lines into ring slot `dst`.
__device__ __forceinline__ void load_batch(uint32_t dst, const uint32_t* lines, int r, int n, uint32_t bar) {
    bulk_load(dst, lines + (int64_t)r * kLineWords, (uint32_t)n * kLineWords * 4, bar);
}

// ---------------------------------------------------------------------------
// The tile's table: word (c, pair, g) = fp16 pair (cb[2 pair][c] . x'_g,
// cb[2 pair + 1][c] . x'_g), x'_g = 2^-E x[8g : 8g + 8].
// ---------------------------------------------------------------------------

// FFMA (codebooks fp16 cannot hold exactly, staged in fp32): warp w builds
// words p = w + 32 j (p = 2 c + pair, word index 32 p + g); lane = group.  Two words' four codebook rows are loaded (broadcast) before
// any is stored; each store is one conflict-free 128-byte row of words.
__device__ __forceinline__ void build_lut_f16(uint32_t* __restrict__ lut, const float* __restrict__ cbs,
                                              const float* __restrict__ xs, float xscale) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float xr[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) xr[i] = xs[lane * 8 + i] * xscale;
    const float4* cb4 = reinterpret_cast<const float4*>(cbs);
#pragma unroll 1
    for (int p0 = warp; p0 < kCodes * 2; p0 += kWarps * 2) {
        float4 a[4], b[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {            // j = 2 * word + stage within the pair
            const int p = p0 + (j >> 1) * kWarps, c = p >> 1, k = ((p & 1) << 1) + (j & 1);
            a[j] = cb4[(k * kCodes + c) * 2];
            b[j] = cb4[(k * kCodes + c) * 2 + 1];
        }
        float acc[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float t = a[j].x * xr[0];
            t = fmaf(a[j].y, xr[1], t);
            t = fmaf(a[j].z, xr[2], t);
            t = fmaf(a[j].w, xr[3], t);
            t = fmaf(b[j].x, xr[4], t);
            t = fmaf(b[j].y, xr[5], t);
            t = fmaf(b[j].z, xr[6], t);
            t = fmaf(b[j].w, xr[7], t);
            acc[j] = t;
        }
#pragma unroll
        for (int w = 0; w < 2; ++w) {
            const __half2 h = __floats2half2_rn(acc[2 * w], acc[2 * w + 1]);    // low half: even stage
            lut[(p0 + w * kWarps) * kGroups + lane] = *reinterpret_cast<const uint32_t*>(&h);
        }
    }
}

// The same table by tensor-core MMAs: LUT[(k, c)][g] = sum_t cb_k[c][t] x'_g[t]
// is a [1024 x 8] x [8 x 32] product.  mma.sync m16n8k16 (fp16 operands, fp32
// accumulation; K padded from 8 to 16 with zeros): an m16 block holds codes
// 8 b .. 8 b + 7 at stage 2 p in rows 0-7 and at stage 2 p + 1 in rows 8-15,
// so each thread's accumulators (c0, c2) and (c1, c3) are the stage pair of
// one (code, group) and pack directly into the table's fp16-pair words.
// Warp w computes m16 blocks w and w + 32 (pairs 0 and 1) for the 4 n8
// blocks of groups: 8 MMAs.  Products of fp16 values are exact; only the
// fp32 summation order may differ from the FFMA build.
__device__ __forceinline__ void build_lut_mma(uint32_t* __restrict__ lut, const uint4* __restrict__ cbh,
                                              const float* __restrict__ xs, float xscale) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gid = lane >> 2, tig = lane & 3;
    // B fragments: x' of groups 8 nb + gid, elements 2 tig and 2 tig + 1 (rows 8..15 zero)
    uint32_t bx[4];
#pragma unroll
    for (int nb = 0; nb < 4; ++nb) {
        const int g = 8 * nb + gid;
        const __half2 h = __floats2half2_rn(xs[8 * g + 2 * tig] * xscale, xs[8 * g + 2 * tig + 1] * xscale);
        bx[nb] = *reinterpret_cast<const uint32_t*>(&h);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int mb = warp + 32 * h;              // m16 block: pair p = mb / 32, code block b = mb % 32
        const int p = mb >> 5, code = 8 * (mb & 31) + gid;
        // A fragment: word tig of the fp16 codebook rows (stage 2p, code) and (stage 2p + 1, code)
        const uint32_t a0 = reinterpret_cast<const uint32_t*>(cbh + (2 * p) * kCodes + code)[tig];
        const uint32_t a1 = reinterpret_cast<const uint32_t*>(cbh + (2 * p + 1) * kCodes + code)[tig];
#pragma unroll
        for (int nb = 0; nb < 4; ++nb) {
            float c0, c1, c2, c3;
            asm volatile(
                "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
                "{%10, %10, %10, %10};\n"
                : "=f"(c0), "=f"(c1), "=f"(c2), "=f"(c3)
                : "r"(a0), "r"(a1), "r"(0u), "r"(0u), "r"(bx[nb]), "r"(0u), "f"(0.f));
            const int g = 8 * nb + 2 * tig;
            const __half2 w0 = __floats2half2_rn(c0, c2), w1 = __floats2half2_rn(c1, c3);   // low half: even stage
            lut[(code * 2 + p) * kGroups + g] = *reinterpret_cast<const uint32_t*>(&w0);
            lut[(code * 2 + p) * kGroups + g + 1] = *reinterpret_cast<const uint32_t*>(&w1);
        }
    }
}

__device__ __forceinline__ uint32_t* ring_slot(uint32_t* ring, int slot) { return ring + slot * kBatchRows * kGroups; }

// Power-of-two scale 2^-E bringing max |x| = amax into [1, 2), and 2^E.
__device__ __forceinline__ void tile_scale(float amax, float& scale, float& unscale) {
    scale = unscale = 1.f;
    if (!(amax > 0.f) || !(amax <= 3.0e38f)) return;      // zero or non-finite: no scaling
    int e = (int)((__float_as_uint(amax) >> 23) & 0xffu) - 127;
    e = e < -126 ? -126 : (e > 126 ? 126 : e);
    scale = __uint_as_float((uint32_t)(127 - e) << 23);
    unscale = __uint_as_float((uint32_t)(127 + e) << 23);
}

// ---------------------------------------------------------------------------
// One unit (job, tile, row range): code words stream into the ring while the
// codebook and the operand slice are staged and the table is built; then the
// rows, batch by batch.  Shared by the plain GEMV launch and the persistent
// decode step.
// ---------------------------------------------------------------------------

// The dynamic shared memory: [table 64 KB][codebook 32 KB][ring][x slice][barriers],
// plus the CTA's small shared state.
struct TileSmem {
    uint32_t* lut;
    float* cbs;
    uint32_t* ring;
    float* xs;
    uint32_t bar0;
    int* slot_done;              // warps finished with a ring slot
    float* xmax;                 // per-warp max |x| of the tile
    // set when a ring wait gave up twice: from then on the CTA issues no copies and
    // waits for none (its partial sums are invalid; the sticky flag tells the host)
    volatile int* aborted;
};

__device__ __forceinline__ TileSmem tile_smem(float* smem, int* slot_done, float* xmax, volatile int* aborted) {
    TileSmem S;
    S.lut = reinterpret_cast<uint32_t*>(smem);
    S.cbs = smem + kLutWords;
    S.ring = reinterpret_cast<uint32_t*>(S.cbs + kCbFloats);
    S.xs = reinterpret_cast<float*>(S.ring + kRing * kBatchRows * kGroups);
    S.bar0 = smem_u32(reinterpret_cast<uint64_t*>(S.xs + kTileCols));
    S.slot_done = slot_done;
    S.xmax = xmax;
    S.aborted = aborted;
    return S;
}

// Called by every thread once, before the first unit.
__device__ __forceinline__ void tile_smem_init(const TileSmem& S) {
    const int tid = threadIdx.x;
    if (tid < kRing) S.slot_done[tid] = 0;
    if (tid == 0) {
        *S.aborted = 0;
        for (int s = 0; s < kRing; ++s) mbar_init(S.bar0 + 8 * s);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    __syncthreads();
}

// What a CTA carries from one unit to the next.
struct UnitState {
    uint32_t phase_bits = 0;     // bit s: parity of ring slot s's next phase
    const void* cb = nullptr;    // codebook now in shared memory
    int cb_kind = -1;
    bool cb_half = false;        // ... staged as fp16 (else fp32)
};

// Thread 0 starts the copies of the unit's first ring batches.
__device__ __forceinline__ void issue_unit_loads(const TJob& J, int tile, int r0, int r1, const TileSmem& S) {
    if (threadIdx.x != 0 || *S.aborted) return;
    const uint32_t* lines = J.codes + (int64_t)tile * J.rows * kLineWords;
    const int nb = (r1 - r0 + kBatchRows - 1) / kBatchRows;
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    for (int b = 0; b < kRing && b < nb; ++b) {
        const int rb = r0 + b * kBatchRows;
        load_batch(smem_u32(ring_slot(S.ring, b)), lines, rb, min(r1 - rb, kBatchRows), S.bar0 + 8 * b);
    }
}

// The tile's operand slice into S.xs (zero past the matrix edge) and the
// per-warp maxima of |x| into S.xmax, from J.x (and J.gate).  Partial-sum
// operands are staged in the table's space, then summed in tile order.
__device__ __forceinline__ void stage_operand(const TJob& J, int tile, const TileSmem& S) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float* staged = reinterpret_cast<float*>(S.lut);
    const bool has_gate = J.gate.ptr != nullptr;
    const bool stage_x = J.x.kind == RVQ_F32 && J.x.ntiles > 1 &&
                         J.x.ntiles + (has_gate ? J.gate.ntiles : 0) <= kMaxStagedTiles;
    const bool stage_g = has_gate && stage_x && J.gate.kind == RVQ_F32 && J.gate.ntiles > 1;
    if (stage_x) stage_partials(J.x, tile, J.cols, staged);
    if (stage_g) stage_partials(J.gate, tile, J.cols, staged + J.x.ntiles * kTileCols);
    if (stage_x) __syncthreads();
    if (tid < kTileCols) {
        const int64_t col = (int64_t)tile * kTileCols + tid;
        float xv = 0.f;
        if (col < J.cols) {
            xv = stage_x ? staged_value(staged, J.x.ntiles, tid) : operand(J.x, col);
            if (has_gate) {
                const float g = stage_g ? staged_value(staged + J.x.ntiles * kTileCols, J.gate.ntiles, tid)
                                        : operand(J.gate, col);
                xv = bf16r(bf16r(g / (1.0f + expf(-g))) * xv);
            }
        }
        S.xs[tid] = xv;
        float m = fabsf(xv);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) S.xmax[warp] = m;
    }
}

// One unit.  Every thread calls it (shared memory free: the caller synchronised
// after the previous unit).  `issue` false: issue_unit_loads already ran for it.
// `stage()` fills S.xs and S.xmax (stage_operand, or the caller's own); it runs
// after the codebook copies start, so it may first wait for its inputs.
template <class Stage>
__device__ __forceinline__ void run_unit(const TJob& J, int tile, int r0, int r1, const TileSmem& S,
                                         UnitState& st, bool issue, Stage&& stage) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // per-stage table address bits of this lane (see lut_offset)
    const uint32_t lb0 = (uint32_t)lane << 2, lb1 = lb0 | 2u, lb2 = lb0 | 128u, lb3 = lb0 | 130u;
    uint32_t* __restrict__ lut = S.lut;
    float* __restrict__ cbs = S.cbs;
    const int G = J.G;
    const int gt = min(kGroups, G - tile * kGroups);
    const int nb = (r1 - r0 + kBatchRows - 1) / kBatchRows;
    const uint32_t* lines = J.codes + (int64_t)tile * J.rows * kLineWords;   // this tile's code lines

    // 1. code words of the first four batches start streaming in
    if (issue) issue_unit_loads(J, tile, r0, r1, S);

    // 2. codebook, then the tile's operand slice
    if (J.cb != st.cb || J.cb_kind != st.cb_kind) {
        // fp16 when every codebook value is an fp16 number (the artifact's
        // codebooks are fp16), else fp32
        st.cb = J.cb;
        st.cb_kind = J.cb_kind;
        uint4* cbh = reinterpret_cast<uint4*>(cbs);
        int inexact = 0;
        if (J.cb_kind == RVQ_F16) {
            const uint4* src = reinterpret_cast<const uint4*>(J.cb);
            for (int i = tid; i < kPairs; i += kThreads) cp_async16(cbh + i, src + i);
            cp_async_commit();
        } else {
            for (int i = tid; i < kPairs; i += kThreads) {
                uint32_t w[4];
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const float f0 = load_as_f32(J.cb, (int64_t)i * 8 + 2 * t, J.cb_kind);
                    const float f1 = load_as_f32(J.cb, (int64_t)i * 8 + 2 * t + 1, J.cb_kind);
                    const __half2 h = __floats2half2_rn(f0, f1);
                    inexact |= (__low2float(h) != f0) | (__high2float(h) != f1);
                    w[t] = *reinterpret_cast<const uint32_t*>(&h);
                }
                cbh[i] = make_uint4(w[0], w[1], w[2], w[3]);
            }
        }
        st.cb_half = !__syncthreads_or(inexact);
        if (!st.cb_half) {
            for (int i = tid; i < kCbFloats; i += kThreads) cbs[i] = load_as_f32(J.cb, i, J.cb_kind);
        }
    }
    stage();
    cp_async_wait<0>();          // the codebook
    __syncthreads();

    // 3. the tile's table (shared-memory bound: the codebook rows are broadcast
    //    loads, the table 64 KB of conflict-free stores), from 2^-E x
    float amax = S.xmax[0];
#pragma unroll
    for (int w = 1; w < kTileCols / 32; ++w) amax = fmaxf(amax, S.xmax[w]);
    float xscale, xunscale;
    tile_scale(amax, xscale, xunscale);
    if (st.cb_half) build_lut_mma(lut, reinterpret_cast<const uint4*>(cbs), S.xs, xscale);
    else build_lut_f16(lut, cbs, S.xs, xscale);
    __syncthreads();

    // 4. rows, batch by batch, three batches streaming in while one is processed.
    //    Every warp waits on the slot's barrier itself, and the last warp to
    //    finish a slot issues its refill: no CTA-wide barrier per batch.
    //    Lanes past the matrix edge read zero code words and table columns
    //    built from x = 0 (exact zeros); rows past the batch (stale words) only
    //    reach outputs that are not stored.
    const uint32_t g_global = (uint32_t)tile * kGroups + lane;
    float* part = J.part + (int64_t)tile * J.rows;
    // this lane's output row scale, fetched two batches ahead of its use
    // (lanes 4i..4i+3 share the row i of each 8-row group; one row group
    // per warp and batch)
    const int orow_in = warp * 8 + ((lane >> 2) & 7);
    const bool scale_lane = J.row_scales && (lane & 3) == 0;
    auto row_scale = [&](int b) -> float {
        const int r = r0 + b * kBatchRows + orow_in;
        return (scale_lane && b < nb && r < r1)
                   ? load_as_f32(J.scales, fastdiv((uint32_t)r, J.rpsdiv), J.scale_kind) : 1.f;
    };
    float sc_next = row_scale(0), sc_next2 = row_scale(1);
    for (int b = 0; b < nb; ++b) {
        const float oscale_b = sc_next;
        sc_next = sc_next2;
        sc_next2 = row_scale(b + 2);
        const int slot = b % kRing;
        if (!*S.aborted && !mbar_wait(S.bar0 + 8 * slot, (st.phase_bits >> slot) & 1u)) *S.aborted = 1;
        st.phase_bits ^= 1u << slot;
        const int rb0 = r0 + b * kBatchRows;
        const int nrows = min(r1, rb0 + kBatchRows) - rb0;
        const uint32_t* cs = ring_slot(S.ring, slot) + lane;
        static_assert(kWarps * 8 == kBatchRows, "one 8-row group per warp and batch");
        {
            const int rb = warp * 8;
            const int orow = rb + ((lane >> 2) & 7);
            const float oscale = oscale_b;
            float v[8];
            if (J.row_scales) {
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] = lookup4(lut, cs[(rb + i) * kGroups], lb0, lb1, lb2, lb3);
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float s = lookup4(lut, cs[(rb + i) * kGroups], lb0, lb1, lb2, lb3);
                    // per-vector scales: only rows and groups inside the matrix have one
                    const bool valid = rb + i < nrows && lane < gt;
                    v[i] = valid ? s * load_as_f32(J.scales,
                                                   fastdiv((uint32_t)(rb0 + rb + i) * (uint32_t)G + g_global,
                                                           J.gvdiv),
                                                   J.scale_kind)
                                 : 0.f;
                }
            }
            const float tot = reduce8(v);
            if ((lane & 3) == 0 && orow < nrows) part[rb0 + orow] = (tot * xunscale) * oscale;
        }
        if (b + kRing < nb) {
            const int nb0 = r0 + (b + kRing) * kBatchRows;
            uint32_t* buf = ring_slot(S.ring, slot);
            __syncwarp();
            if (lane == 0) {
                __threadfence_block();
                const int done = atomicAdd(&S.slot_done[slot], 1);
                if (done == kWarps - 1) {               // every warp has left this slot
                    S.slot_done[slot] = 0;
                    __threadfence_block();
                    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
                    if (!*S.aborted)
                        load_batch(smem_u32(buf), lines, nb0, min(r1 - nb0, kBatchRows), S.bar0 + 8 * slot);
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------

// The kernel-side job of a checked rvq_gemv_tile_job.
inline TJob make_tjob(const rvq_gemv_tile_job& g) {
    TJob J;
    memset(&J, 0, sizeof(J));
    J.codes = reinterpret_cast<const uint32_t*>(g.weight.indices);
    J.cb = g.weight.codebook;
    J.scales = g.weight.scales;
    J.x = g.x;
    J.gate = g.gate;
    J.part = g.partials;
    J.cols = g.cols;
    J.rows = (int32_t)g.rows;
    J.G = (int32_t)(g.cols / 8);
    const uint32_t gv = (uint32_t)g.weight.group_vecs;
    J.gvdiv = make_fastdiv(gv);
    J.row_scales = gv % (uint32_t)J.G == 0;
    J.rpsdiv = make_fastdiv(J.row_scales ? gv / (uint32_t)J.G : 1u);
    J.cb_kind = g.weight.codebook_kind;
    J.scale_kind = g.weight.scale_kind;
    return J;
}

// Units.  Two plans are costed, a unit costing its rows plus kSwitchRows, and
// the one whose most loaded CTA costs less is taken:
//  * one unit per CTA: tile t gets c_t CTAs with equal row ranges, the c_t
//    chosen (binary search on the cost bound) to minimise the largest unit;
//  * runs: the (job, tile, row) work in job and tile order is cut into
//    contiguous runs of equal cost, one run per CTA (a run that crosses a tile
//    boundary builds two tables).
// Row ranges are cut at multiples of 8 rows.

inline int plan(const rvq_gemv_tile_job* jobs, int n, int sms, TParams& p, int switch_rows = kSwitchRows) {
    int ntiles = 0;
    int64_t rows_total = 0;
    for (int j = 0; j < n; ++j) {
        const int64_t nt = (jobs[j].cols / 8 + kGroups - 1) / kGroups;
        ntiles += (int)nt;
        rows_total += nt * jobs[j].rows;
    }
    if (ntiles > kMaxUnits) return RVQ_ERR_TOO_LARGE;
    const int ctas = sms < kMaxCtas ? sms : kMaxCtas;

    // plan A: one unit per CTA
    auto ctas_for = [&](int64_t bound_rows, int j) -> int64_t {   // CTAs per tile of job j
        const int64_t R = jobs[j].rows;
        int64_t c = (R + bound_rows - 1) / bound_rows;
        const int64_t cmax = (R + 7) / 8;
        return c < 1 ? 1 : (c > cmax ? cmax : c);
    };
    auto total_ctas = [&](int64_t bound_rows) -> int64_t {
        int64_t t = 0;
        for (int j = 0; j < n; ++j) t += ctas_for(bound_rows, j) * ((jobs[j].cols / 8 + kGroups - 1) / kGroups);
        return t;
    };
    int64_t lo = 8, hi = 8;
    for (int j = 0; j < n; ++j) hi = hi > jobs[j].rows ? hi : jobs[j].rows;
    hi = (hi + 7) & ~7ll;
    if (total_ctas(hi) > ctas) {
        lo = hi = -1;                                       // more tiles than CTAs: plan A impossible
    } else {
        while (lo < hi) {                                   // smallest bound whose CTA count fits
            const int64_t mid = ((lo + hi) / 2 + 7) & ~7ll;
            if (mid >= hi) break;
            if (total_ctas(mid) <= ctas) hi = mid; else lo = mid + 8;
        }
    }
    double cost_a = 1e30;
    int64_t bound = hi;
    if (bound > 0) {
        cost_a = 0;
        for (int j = 0; j < n; ++j) {
            const int64_t R = jobs[j].rows, c = ctas_for(bound, j);
            const int64_t longest = ((R + c - 1) / c + 7) & ~7ll;
            cost_a = cost_a > switch_rows + longest ? cost_a : (double)(switch_rows + longest);
        }
    }

    // plan B: contiguous runs of equal cost
    const double target = (double)(rows_total + (int64_t)switch_rows * (ntiles + ctas)) / ctas;
    const double cost_b = target + switch_rows;             // the run that ends mid-tile pays one more table

    int u = 0, c = 0;
    p.cta_first[0] = 0;
    if (cost_a <= cost_b) {
        for (int j = 0; j < n; ++j) {
            const int nt = (int)((jobs[j].cols / 8 + kGroups - 1) / kGroups);
            const int64_t R = jobs[j].rows, cj = ctas_for(bound, j);
            for (int t = 0; t < nt; ++t) {
                for (int64_t k = 0; k < cj; ++k) {
                    const int64_t a = (R * k / cj) & ~7ll, b = k + 1 == cj ? R : (R * (k + 1) / cj) & ~7ll;
                    if (b <= a) continue;
                    if (u >= kMaxUnits || c >= kMaxCtas) return RVQ_ERR_TOO_LARGE;
                    p.unit_jt[u] = ((uint32_t)j << 24) | (uint32_t)t;
                    p.unit_r0[u] = (int32_t)a;
                    p.unit_r1[u] = (int32_t)b;
                    ++u;
                    p.cta_first[++c] = u;
                }
            }
        }
        p.n_ctas = c;
        p.n_units = u;
        return RVQ_OK;
    }
    double cost = 0;
    for (int j = 0; j < n; ++j) {
        const int nt = (int)((jobs[j].cols / 8 + kGroups - 1) / kGroups);
        const int R = (int)jobs[j].rows;
        for (int t = 0; t < nt; ++t) {
            int r = 0;
            while (r < R) {
                const double room = target - cost - switch_rows;      // rows this run can still take
                if (cost > 0 && room < 64 && c + 1 < ctas) {           // close this run, open the next
                    p.cta_first[++c] = u;
                    cost = 0;
                    continue;
                }
                int take = R - r;
                if (c + 1 < ctas && room < take) {
                    take = (int)room;
                    take = take < 64 ? 64 : (take + 7) & ~7;
                    if (take > R - r) take = R - r;
                }
                if (u >= kMaxUnits) return RVQ_ERR_TOO_LARGE;
                p.unit_jt[u] = ((uint32_t)j << 24) | (uint32_t)t;
                p.unit_r0[u] = r;
                p.unit_r1[u] = r + take;
                ++u;
                cost += switch_rows + take;
                r += take;
            }
        }
    }
    p.cta_first[c + 1] = u;
    p.n_ctas = c + 1;
    p.n_units = u;
    return RVQ_OK;
}

}  // namespace tiles
}  // namespace rvq
