// Batch-1 RVQ dequant-GEMV writing per-tile partial sums (sm_100a).
//
//   part[t][r] = sum over the 8-column groups g of tile t (256 columns) of
//                scale(r, g) * sum_k LUT_k[code_k(r, g)][g],
//   LUT_k[c][g] = codebook_k[c] . x[8g : 8g + 8]
//
// i.e. y = W x without reconstructing W: per 8 weights, 4 table lookups and
// 3 adds.  The reference has no fused path (it reconstructs W into the slot
// and calls F.linear, infer_compressed_layerwise_triton.py:290-292).
//
// A unit is one (job, tile, row range).  Its rows' code words (one
// 32-bit word per vector, stored tile-major by rvq_tile_codes so that a tile's
// rows are contiguous 128-byte lines) stream into a four-slot shared-memory
// ring, 256 rows (32 KB, one contiguous range) per bulk copy (cp.async.bulk),
// while the CTA builds the tile's 64 KB table (4 stages x 256 codes x 32
// groups, fp16).  Each CTA owns a contiguous run of (job, tile, row range)
// units sized so that every CTA has the same work, counting a table build as
// kSwitchRows rows; the codebook stays in shared memory across units of one
// job.
//
// Table: x is first scaled by a power of two 2^-E so that max |x| over the
// tile lies in [1, 2) (exact), every entry is rounded once to fp16 (relative
// error <= 2^-11, below the 2^-8 of a bf16 weight), and each row's tile sum
// is multiplied back by 2^E.  Entries are accumulated in fp32 (add.rn.f32.f16).
// Layout [code][stage / 2][group][stage % 2]: the 32-bit word (code, pair,
// group) holds the entries of stages 2 pair and 2 pair + 1, lane g always reads
// bank g (conflict-free random-code lookups), and the byte offset of an entry,
// code << 8 | (stage / 2) << 7 | g << 2 | (stage % 2) << 1, takes one byte
// permute (prmt) of the code word.
//
// Rows are reduced 8 at a time with a warp reduce-scatter.  Nothing is shared
// between CTAs: partial sums go to [ntiles][rows] and the consumer adds them in
// tile order, so the result is deterministic and needs no cross-CTA sync.

#include <mutex>
#include <string.h>

#include "rvq_common.cuh"
#include "rvq_vecdecode.cuh"

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

__device__ int g_wait_timeout;                              // sticky: a TMA wait gave up

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

__device__ __forceinline__ float operand(const rvq_vec& v, int64_t i) {
    if (v.kind == RVQ_F32) {
        const float* p = reinterpret_cast<const float*>(v.ptr);
        float s = __ldg(p + i);
        for (int t = 1; t < v.ntiles; ++t) s += __ldg(p + (int64_t)t * v.n + i);
        return bf16r(s);
    }
    return load_as_f32(v.ptr, i, v.kind);
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
            r[k] = (i < total && col < cols) ? __ldg(p + (int64_t)t * v.n + col) : 0.f;
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

__global__ void __launch_bounds__(kThreads, 1) rvq_gemv_tiles_kernel(const __grid_constant__ TParams p) {
    extern __shared__ __align__(128) float smem[];
    uint32_t* __restrict__ lut = reinterpret_cast<uint32_t*>(smem);
    float* __restrict__ cbs = smem + kLutWords;
    uint32_t* ring = reinterpret_cast<uint32_t*>(cbs + kCbFloats);
    float* xs = reinterpret_cast<float*>(ring + kRing * kBatchRows * kGroups);
    uint64_t* bars = reinterpret_cast<uint64_t*>(xs + kTileCols);
    float* staged = smem;                                // operand partials, before the table is built
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t bar0 = smem_u32(bars);
    // per-stage table address bits of this lane (see lut_offset)
    const uint32_t lb0 = (uint32_t)lane << 2, lb1 = lb0 | 2u, lb2 = lb0 | 128u, lb3 = lb0 | 130u;

    __shared__ int slot_done[kRing];                     // warps finished with a ring slot
    __shared__ float xmax[kTileCols / 32];               // per-warp max |x| of the tile
    // set when a ring wait gave up twice: from then on the CTA issues no copies and
    // waits for none (its partial sums are invalid; the sticky flag tells the host)
    __shared__ volatile int aborted;
    if (tid < kRing) slot_done[tid] = 0;
    if (tid == 0) aborted = 0;
    pdl_launch_dependents();
    if (tid == 0) {
        for (int s = 0; s < kRing; ++s) mbar_init(bar0 + 8 * s);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    __syncthreads();
    uint32_t phase_bits = 0;                             // bit s: parity of ring slot s's next phase

    const int u_first = p.cta_first[blockIdx.x], u_last = p.cta_first[blockIdx.x + 1];
    int cb_job = -1;                                     // job whose codebook is in shared memory
    bool cb_half = false;                                // ... staged as fp16 (else fp32)
    for (int u = u_first; u < u_last; ++u) {
        const uint32_t jt = p.unit_jt[u];
        const int ji = (int)(jt >> 24);
        const TJob& J = p.jobs[ji];
        const int tile = (int)(jt & 0xffffffu);
        const int r0 = p.unit_r0[u], r1 = p.unit_r1[u];
        const int G = J.G;
        const int gt = min(kGroups, G - tile * kGroups);
        const int nb = (r1 - r0 + kBatchRows - 1) / kBatchRows;
        const uint32_t* lines = J.codes + (int64_t)tile * J.rows * kLineWords;   // this tile's code lines
        if (u != u_first) __syncthreads();              // the previous unit is done with shared memory

        // 1. code words of the first four batches start streaming in
        if (tid == 0 && !aborted) {
            asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
            for (int b = 0; b < kRing && b < nb; ++b) {
                const int rb = r0 + b * kBatchRows;
                load_batch(smem_u32(ring_slot(ring, b)), lines, rb, min(r1 - rb, kBatchRows), bar0 + 8 * b);
            }
        }

        // 2. codebook (fp32) and the tile's operand slice; partial-sum operands
        //    are staged in the table's space, then summed in tile order
        if (ji != cb_job) {
            // fp16 when every codebook value is an fp16 number (the artifact's
            // codebooks are fp16), else fp32
            cb_job = ji;
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
            cb_half = !__syncthreads_or(inexact);
            if (!cb_half) {
                for (int i = tid; i < kCbFloats; i += kThreads) cbs[i] = load_as_f32(J.cb, i, J.cb_kind);
            }
        }
        if (u == u_first) pdl_wait();                    // x comes from the previous kernel
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
            xs[tid] = xv;
            float m = fabsf(xv);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            if (lane == 0) xmax[warp] = m;
        }
        cp_async_wait<0>();          // the codebook
        __syncthreads();

        // 3. the tile's table (shared-memory bound: the codebook rows are broadcast
        //    loads, the table 64 KB of conflict-free stores), from 2^-E x
        float amax = xmax[0];
#pragma unroll
        for (int w = 1; w < kTileCols / 32; ++w) amax = fmaxf(amax, xmax[w]);
        float xscale, xunscale;
        tile_scale(amax, xscale, xunscale);
        if (cb_half) build_lut_mma(lut, reinterpret_cast<const uint4*>(cbs), xs, xscale);
        else build_lut_f16(lut, cbs, xs, xscale);
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
            if (!aborted && !mbar_wait(bar0 + 8 * slot, (phase_bits >> slot) & 1u)) aborted = 1;
            phase_bits ^= 1u << slot;
            const int rb0 = r0 + b * kBatchRows;
            const int nrows = min(r1, rb0 + kBatchRows) - rb0;
            const uint32_t* cs = ring_slot(ring, slot) + lane;
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
                uint32_t* buf = ring_slot(ring, slot);
                __syncwarp();
                if (lane == 0) {
                    __threadfence_block();
                    const int done = atomicAdd(&slot_done[slot], 1);
                    if (done == kWarps - 1) {               // every warp has left this slot
                        slot_done[slot] = 0;
                        __threadfence_block();
                        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
                        if (!aborted)
                            load_batch(smem_u32(buf), lines, nb0, min(r1 - nb0, kBatchRows), bar0 + 8 * slot);
                    }
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Exact-weight variant (rvq_gemv_tiles_exact).  Every weight is rebuilt
// bit-identically to rvq_decode -- fp32 sum of the stage codewords in stage
// order starting from +0, times the fp32 scale, rounded to nearest even bf16
// -- and multiplied by the bf16 operand in fp32 (exact products, an fma chain
// over the vector's 8 columns), so the products are those F.linear forms on
// the decoded bf16 slot and only the fp32 summation order differs.  No tables:
// lane g of a warp owns group g of the tile, and a warp takes 8 rows per
// batch, reduced over the lanes with reduce8.
//
// The codebook sits in shared memory as fp16 with 8 copies per entry
// (rvq_vecdecode.cuh); a codebook that fp16 cannot hold exactly is read from
// global memory in fp32 instead.
// Code words are loaded straight from the tile-major lines, one batch ahead.
// ---------------------------------------------------------------------------
namespace exact {
constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr int kBatchRows = kWarps * 8;                       // 8 rows per warp and batch
constexpr int kCbBytes = vdec::kCbBytes;                     // 128 KB
constexpr int kMaxStagedTiles = 64;                          // operand partial tiles staged (64 KB)
constexpr size_t kSmemBytes = (size_t)kCbBytes + (size_t)(kMaxStagedTiles + 1) * kTileCols * 4;
constexpr int kSwitchRows = 256;                             // starting a unit ~ 256 rows
}  // namespace exact

// sum over t of w[t] * x[t] in fp32, t = 0..7 in order (bf16 x bf16 products are exact)
__device__ __forceinline__ float dot8_bf16(const uint4& w, const uint32_t (&xh)[4]) {
    float acc;
    asm("{\n .reg .b16 w0, w1, w2, w3, w4, w5, w6, w7, x0, x1, x2, x3, x4, x5, x6, x7;\n"
        " mov.b32 {w0, w1}, %1;\n mov.b32 {w2, w3}, %2;\n mov.b32 {w4, w5}, %3;\n mov.b32 {w6, w7}, %4;\n"
        " mov.b32 {x0, x1}, %5;\n mov.b32 {x2, x3}, %6;\n mov.b32 {x4, x5}, %7;\n mov.b32 {x6, x7}, %8;\n"
        " fma.rn.f32.bf16 %0, w0, x0, 0f00000000;\n fma.rn.f32.bf16 %0, w1, x1, %0;\n"
        " fma.rn.f32.bf16 %0, w2, x2, %0;\n fma.rn.f32.bf16 %0, w3, x3, %0;\n"
        " fma.rn.f32.bf16 %0, w4, x4, %0;\n fma.rn.f32.bf16 %0, w5, x5, %0;\n"
        " fma.rn.f32.bf16 %0, w6, x6, %0;\n fma.rn.f32.bf16 %0, w7, x7, %0;\n}\n"
        : "=f"(acc)
        : "r"(w.x), "r"(w.y), "r"(w.z), "r"(w.w), "r"(xh[0]), "r"(xh[1]), "r"(xh[2]), "r"(xh[3]));
    return acc;
}

template <bool SMEM>
__device__ __forceinline__ void exact_rows(const TJob& J, const char* cbs, int tile, int r0, int r1, int gt,
                                           const uint32_t (&xh)[4], const uint32_t (&lb)[4]) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t* lines = J.codes + (int64_t)tile * J.rows * kLineWords;
    float* part = J.part + (int64_t)tile * J.rows;
    const uint32_t g_global = (uint32_t)tile * kGroups + lane;
    const int nb = (r1 - r0 + exact::kBatchRows - 1) / exact::kBatchRows;
    const int orow = warp * 8 + ((lane >> 2) & 7);
    // this warp's 8 code words of batch b (zero past the unit's rows), and with
    // per-row scales, lane l's copy of the scale of the warp's row l & 7
    auto fetch = [&](int b, uint32_t (&w)[8], float& rs) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int r = r0 + b * exact::kBatchRows + warp * 8 + i;
            w[i] = (b < nb && r < r1) ? __ldg(lines + (int64_t)r * kLineWords + lane) : 0u;
        }
        const int r = r0 + b * exact::kBatchRows + warp * 8 + (lane & 7);
        rs = (J.row_scales && b < nb && r < r1) ? load_as_f32(J.scales, fastdiv((uint32_t)r, J.rpsdiv), J.scale_kind)
                                               : 0.f;
    };
    uint32_t wn[8];
    float rsn;
    fetch(0, wn, rsn);
    for (int b = 0; b < nb; ++b) {
        uint32_t wc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) wc[i] = wn[i];
        const float rsc = rsn;
        fetch(b + 1, wn, rsn);
        const int rb = r0 + b * exact::kBatchRows + warp * 8;
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int r = rb + i;
            float s;
            if (J.row_scales) {
                s = __shfl_sync(0xffffffffu, rsc, i);          // zero past the unit's rows
            } else {
                s = (r < r1 && lane < gt)
                        ? load_as_f32(J.scales, fastdiv((uint32_t)r * (uint32_t)J.G + g_global, J.gvdiv),
                                      J.scale_kind)
                        : 0.f;
            }
            v[i] = dot8_bf16(vdec::weights_bf16<SMEM>(cbs, J.cb, J.cb_kind, wc[i], lb, s), xh);
        }
        const float tot = reduce8(v);
        const int r = r0 + b * exact::kBatchRows + orow;
        if ((lane & 3) == 0 && r < r1) part[r] = tot;
    }
}

__global__ void __launch_bounds__(exact::kThreads, 1) rvq_gemv_exact_kernel(const __grid_constant__ TParams p) {
    extern __shared__ __align__(128) float smem[];
    char* cbs = reinterpret_cast<char*>(smem);
    float* staged = smem + exact::kCbBytes / 4;                  // operand partials [tiles][256]
    float* xs = staged + exact::kMaxStagedTiles * kTileCols;     // the tile's operand slice
    const int tid = threadIdx.x, lane = tid & 31;
    uint32_t lb[4];
    vdec::lane_bits(lane, lb);
    pdl_launch_dependents();
    const int u_first = p.cta_first[blockIdx.x], u_last = p.cta_first[blockIdx.x + 1];
    int cb_job = -1;
    bool cb_smem = false;
    for (int u = u_first; u < u_last; ++u) {
        const uint32_t jt = p.unit_jt[u];
        const int ji = (int)(jt >> 24);
        const TJob& J = p.jobs[ji];
        const int tile = (int)(jt & 0xffffffu);
        const int r0 = p.unit_r0[u], r1 = p.unit_r1[u];
        const int gt = min(kGroups, J.G - tile * kGroups);
        if (u != u_first) __syncthreads();                       // the previous unit is done with shared memory
        if (ji != cb_job) {
            cb_job = ji;
            cb_smem = vdec::stage_cb8(J.cb, J.cb_kind, cbs, tid, exact::kThreads);
        }
        if (u == u_first) pdl_wait();                            // the operand comes from the previous kernel
        const bool has_gate = J.gate.ptr != nullptr;
        const bool stage_x = J.x.kind == RVQ_F32 && J.x.ntiles > 1 &&
                             J.x.ntiles + (has_gate ? J.gate.ntiles : 0) <= exact::kMaxStagedTiles;
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
            xs[tid] = xv;                                        // a bf16 value (operand kinds are bf16 or partials)
        }
        __syncthreads();
        uint32_t xh[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) xh[i] = pack2(xs[lane * 8 + 2 * i], xs[lane * 8 + 2 * i + 1], RVQ_BF16);
        if (cb_smem) exact_rows<true>(J, cbs, tile, r0, r1, gt, xh, lb);
        else exact_rows<false>(J, cbs, tile, r0, r1, gt, xh, lb);
    }
}

// ---------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------
struct DevInfo {
    bool ready = false, ok = false;
    int sms = 0;
};
DevInfo g_dev[64];
std::mutex g_mu;

int dev_info(DevInfo** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64) {
        last_cuda_error_slot() = (int)e;
        return RVQ_ERR_UNAVAILABLE;
    }
    std::lock_guard<std::mutex> lock(g_mu);
    DevInfo& d = g_dev[dev];
    if (!d.ready) {
        d.ready = true;
        cudaDeviceProp prop;
        e = cudaGetDeviceProperties(&prop, dev);
        if (e == cudaSuccess && prop.major == 10 && prop.sharedMemPerBlockOptin >= kSmemBytes &&
            prop.sharedMemPerBlockOptin >= exact::kSmemBytes) {
            d.sms = prop.multiProcessorCount;
            e = cudaFuncSetAttribute(rvq_gemv_tiles_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kSmemBytes);
            if (e == cudaSuccess)
                e = cudaFuncSetAttribute(rvq_gemv_exact_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)exact::kSmemBytes);
            d.ok = e == cudaSuccess;
        }
        if (e != cudaSuccess) last_cuda_error_slot() = (int)e;
    }
    if (!d.ok) return RVQ_ERR_UNAVAILABLE;
    *out = &d;
    return RVQ_OK;
}

bool operand_ok(const rvq_vec& v, int64_t n) {
    if (v.ptr == nullptr || v.n != n || v.ntiles < 1) return false;
    if (v.kind == RVQ_F32) return true;
    return (v.kind == RVQ_BF16 || v.kind == RVQ_F16) && v.ntiles == 1;
}

int check_job(const rvq_gemv_tile_job& g) {
    const rvq_entry& w = g.weight;
    const int rc = rvq_check_entry(&w);
    if (rc != RVQ_OK) return rc;
    if (w.stages != kStages || w.ncodes != kCodes || w.index_kind != RVQ_U8 || w.d != 8)
        return RVQ_ERR_UNSUPPORTED;
    if (g.rows < 1 || g.cols < 8 || g.cols % 8) return RVQ_ERR_UNSUPPORTED;
    if (g.rows * (g.cols / 8) != w.nvec || w.trimmed != w.nvec * 8 || w.tail_numel != 0)
        return RVQ_ERR_UNSUPPORTED;
    if ((uintptr_t)w.indices & 15) return RVQ_ERR_INVALID;      // bulk copies start on 16 bytes
    if (w.nvec >= (1ll << 32) || g.rows >= (1ll << 31) || (g.cols + kTileCols - 1) / kTileCols >= (1 << 24))
        return RVQ_ERR_TOO_LARGE;
    if (w.codebook_kind != RVQ_F32 && w.codebook_kind != RVQ_F16 && w.codebook_kind != RVQ_BF16)
        return RVQ_ERR_UNSUPPORTED;
    if (w.codebook_kind == RVQ_F32 && ((uintptr_t)w.codebook & 15)) return RVQ_ERR_INVALID;
    if (!operand_ok(g.x, g.cols) || (g.gate.ptr != nullptr && !operand_ok(g.gate, g.cols))) return RVQ_ERR_INVALID;
    if (g.partials == nullptr) return RVQ_ERR_INVALID;
    return RVQ_OK;
}

// Units.  Two plans are costed, a unit costing its rows plus kSwitchRows, and
// the one whose most loaded CTA costs less is taken:
//  * one unit per CTA: tile t gets c_t CTAs with equal row ranges, the c_t
//    chosen (binary search on the cost bound) to minimise the largest unit;
//  * runs: the (job, tile, row) work in job and tile order is cut into
//    contiguous runs of equal cost, one run per CTA (a run that crosses a tile
//    boundary builds two tables).
// Row ranges are cut at multiples of 8 rows.

int plan(const rvq_gemv_tile_job* jobs, int n, int sms, TParams& p, int switch_rows = kSwitchRows) {
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

// Tile-major code lines: out[t][r][w] = the code word of vector (r, 32 t + w),
// zero past the last group.  One thread per output word.
__global__ void tile_codes_kernel(const uint8_t* __restrict__ planes, int64_t stage_stride, int64_t rows,
                                  int64_t G, int64_t ntiles, uint32_t* __restrict__ out) {
    const int64_t total = ntiles * rows * kLineWords;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t w = i % kLineWords, tr = i / kLineWords;
        const int64_t r = tr % rows, t = tr / rows;
        const int64_t g = t * kLineWords + w;
        uint32_t word = 0;
        if (g < G) {
            const int64_t v = r * G + g;
            word = (uint32_t)planes[v] | ((uint32_t)planes[stage_stride + v] << 8) |
                   ((uint32_t)planes[2 * stage_stride + v] << 16) | ((uint32_t)planes[3 * stage_stride + v] << 24);
        }
        out[i] = word;
    }
}

}  // namespace tiles
}  // namespace rvq

using namespace rvq;
using namespace rvq::tiles;

extern "C" {

int64_t rvq_gemv_tiles_count(int64_t cols) { return cols < 1 ? 0 : (cols + kTileCols - 1) / kTileCols; }

int64_t rvq_tile_codes_bytes(int64_t rows, int64_t cols) {
    if (rows < 1 || cols < 8 || cols % 8) return 0;
    return rvq_gemv_tiles_count(cols) * rows * kLineWords * 4;
}

int rvq_tile_codes(const void* planes, int64_t stage_stride, int64_t rows, int64_t cols, void* out, void* stream) {
    if (planes == nullptr || out == nullptr || rows < 1 || cols < 8 || cols % 8) return RVQ_ERR_INVALID;
    const int64_t G = cols / 8;
    if (stage_stride < rows * G || ((uintptr_t)out & 15)) return RVQ_ERR_INVALID;
    const int64_t ntiles = rvq_gemv_tiles_count(cols);
    const int64_t total = ntiles * rows * kLineWords;
    const int64_t blocks64 = (total + 255) / 256;
    const int blocks = (int)(blocks64 < 148 * 16 ? blocks64 : 148 * 16);
    tile_codes_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(reinterpret_cast<const uint8_t*>(planes),
                                                                stage_stride, rows, G, ntiles,
                                                                reinterpret_cast<uint32_t*>(out));
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        last_cuda_error_slot() = (int)e;
        return RVQ_ERR_CUDA;
    }
    return RVQ_OK;
}

static int launch_tiles(const rvq_gemv_tile_job* jobs, int n_jobs, void* stream, bool exact_weights) {
    if (jobs == nullptr || n_jobs < 1 || n_jobs > kMaxJobs) return RVQ_ERR_INVALID;
    for (int i = 0; i < n_jobs; ++i) {
        const int rc = check_job(jobs[i]);
        if (rc != RVQ_OK) return rc;
        // exact weights are multiplied as bf16 x bf16: the operands must be bf16 values
        if (exact_weights && (jobs[i].x.kind == RVQ_F16 || (jobs[i].gate.ptr && jobs[i].gate.kind == RVQ_F16)))
            return RVQ_ERR_UNSUPPORTED;
    }
    DevInfo* d = nullptr;
    int rc = dev_info(&d);
    if (rc != RVQ_OK) return rc;
    static thread_local TParams p;
    memset(&p, 0, sizeof(p));
    for (int i = 0; i < n_jobs; ++i) {
        const rvq_gemv_tile_job& g = jobs[i];
        TJob& J = p.jobs[i];
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
    }
    rc = plan(jobs, n_jobs, d->sms, p, exact_weights ? exact::kSwitchRows : kSwitchRows);
    if (rc != RVQ_OK) return rc;
    const int grid = p.n_ctas;
    cudaError_t e =
        exact_weights
            ? launch_pdl(rvq_gemv_exact_kernel, dim3(grid), dim3(exact::kThreads), exact::kSmemBytes,
                         (cudaStream_t)stream, p)
            : launch_pdl(rvq_gemv_tiles_kernel, dim3(grid), dim3(kThreads), kSmemBytes, (cudaStream_t)stream, p);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) {
        last_cuda_error_slot() = (int)e;
        return RVQ_ERR_CUDA;
    }
    return RVQ_OK;
}

int rvq_gemv_tiles(const rvq_gemv_tile_job* jobs, int n_jobs, void* stream) {
    return launch_tiles(jobs, n_jobs, stream, false);
}

int rvq_gemv_tiles_exact(const rvq_gemv_tile_job* jobs, int n_jobs, void* stream) {
    return launch_tiles(jobs, n_jobs, stream, true);
}

int rvq_take_wait_timeout(void) {
    int v = 0;
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&v, g_wait_timeout, sizeof(int));
    const int zero = 0;
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_wait_timeout, &zero, sizeof(int));
    if (e != cudaSuccess) {
        last_cuda_error_slot() = (int)e;
        return -RVQ_ERR_CUDA;
    }
    return v;
}

}  // extern "C"
