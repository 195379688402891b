// Fused dequant-GEMM on the tensor cores for small batches and prompts (sm_100a):
//
//   y[t][r] = bf16( sum_c x[t][c] * W[r][c] ),  t < T tokens, W an RVQ entry
//
// The reference materialises W into the slot and calls F.linear
// (infer_compressed_layerwise_triton.py:290-292).  Here W never reaches HBM
// or shared memory: it is the A operand of tcgen05.mma read from tensor
// memory.  A CTA owns 128-row tiles of W and ranges of 64-column chunks
// ("segments").  For every chunk, 16 decoder warps rebuild the 128 x 64
// weights bit-identically to the slot's bf16 values (rvq_vecdecode.cuh; the
// codebook is the only large shared-memory table) and store them into a TMEM
// weight stage with tcgen05.st: warp w owns TMEM lanes 32 (w % 4) .. + 31, one
// weight row per thread, and two of the chunk's 8 vectors.  Their code words
// and scales are loaded kPrefetch chunks ahead, so HBM latency is not paid per
// chunk.  The issuer warp loads x[block][chunk] by TMA (rows past T read as
// zero) and issues four tcgen05.mma (kind::f16, A = the TMEM stage, B = x in
// shared memory, M = 128 weight rows, N = a block of up to 192 tokens, K = 16),
// accumulating in TMEM.  Four epilogue warps read each finished segment with
// tcgen05.ld; two accumulators alternate, so the next segment's MMAs run while
// the previous one is read out.  A prompt of more than 192 tokens runs as
// equal token blocks: each weight chunk is decoded once per block.
//
// Work split: the (row tile, token block, chunk) units in that order are cut
// into one contiguous range per SM, so every CTA decodes the same number of
// chunks.  Each CTA derives its segments (the (tile, block) pairs its range
// touches), their piece numbers and workspace slots from the split formula
// itself, so the launch carries no table.  A (tile, block) cut into several
// pieces writes fp32 partial sums to the workspace -- slot 2c for the first
// segment of CTA c, 2c + 1 for its last (a middle segment is never cut); the
// CTA that finishes its last piece (ticket counter) adds the pieces in piece
// order and writes y, so results do not depend on timing.  Units held by one
// CTA write y directly.
//
// Only the codes (0.5 B per weight), the scales and x are read from HBM.
//
// exact = 0 decodes the weights with fp16 stage sums (weights_bf16_fast)
// instead of the bit-exact fp32 chain.

#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <string.h>
#include <type_traits>

#include "rvq_common.cuh"
#include "rvq_sm100.cuh"
#include "rvq_vecdecode.cuh"

namespace rvq {
namespace batch {

using namespace sm100;

constexpr int kDecodeWarps = 16;
constexpr int kEpiWarps = 4;
constexpr int kIssuer = kDecodeWarps + kEpiWarps;           // warp index of the MMA issuer
constexpr int kProducer = kIssuer + 1;                       // warp index of the x loader
constexpr int kThreads = (kProducer + 1) * 32;               // 704
// Named barrier 2 + s hands TMEM/x stage s to the issuer: decoder warps and the
// x loader arrive, the issuer waits (no shared-memory polling on that path).
constexpr int kStageBarThreads = (kDecodeWarps + 2) * 32;
constexpr int kRedTokens = 16;                               // tokens per step of the split-K reduction
constexpr int kRedPieces = 1;                                // pieces loaded per round of the reduction
constexpr int kTileRows = 128;                               // MMA M: weight rows per tile
constexpr int kChunk = 64;                                   // columns per chunk (one 128-byte swizzle row)
constexpr int kChunkVecs = kChunk / 8;
constexpr int kMaxStages = 4;
constexpr int kPrefetch = 2;                                 // chunks of codes and scales in flight per decoder
constexpr int kBlockTokens = 192;                            // MMA N per token block (max)
constexpr int kMaxTokens = 65536;
constexpr long long kWaitLimit = 1ll << 24;
constexpr int kBudget = 226 * 1024;                          // dynamic shared memory limit used per CTA

__device__ int g_batch_timeout;

struct BParams {
    CUtensorMap xmap;         // x [T][K] bf16, box {64, npad}, 128-byte swizzle
    const uint32_t* codes;    // tile-major code lines [ceil(K/256)][R][32]
    const void* cb;
    const void* scales;
    __nv_bfloat16* y;         // [T][R]
    float* part;              // workspace: [2 n_ctas][npad][128] fp32
    uint32_t* tickets;        // workspace: [tiles * blocks]
    int64_t U;                // (tile, token block, chunk) units
    int32_t R, G, T, npad, blocks, KC, stages, n_ctas;
    int32_t cb_kind, scale_kind, row_scales;
    int32_t exact;            // 1: bit-exact bf16 weights, 0: fp16 stage sums
    FastDiv gvdiv, rpsdiv;
};

// CTA c owns units [range_begin(c), range_begin(c + 1)).
__device__ __forceinline__ int64_t range_begin(const BParams& p, int c) { return p.U * c / p.n_ctas; }
// The CTA whose range holds unit u.
__device__ __forceinline__ int cta_of(const BParams& p, int64_t u) { return (int)(((u + 1) * p.n_ctas - 1) / p.U); }

// The segment that starts at unit u of a range ending at u1: its (tile, block)
// index and chunk range [kc0, kc1).
struct Seg {
    int unit, kc0, kc1;
};
__device__ __forceinline__ Seg seg_at(const BParams& p, int64_t u, int64_t u1) {
    Seg s;
    s.unit = (int)(u / p.KC);
    const int64_t base = (int64_t)s.unit * p.KC;
    s.kc0 = (int)(u - base);
    s.kc1 = (int)(u1 - base < p.KC ? u1 - base : p.KC);
    return s;
}

// TMEM columns: accumulators at 0 and npad, each read 32 columns at a time
// (up to column npad + round32(npad) - 1), then weight stages of 32 columns
// from a_base_of(npad).
__host__ __device__ __forceinline__ int a_base_of(int npad) {
    return (npad + (npad + 31) / 32 * 32 + 31) / 32 * 32;
}
__host__ __device__ __forceinline__ uint32_t tmem_cols_of(int npad, int stages) {
    const int need = a_base_of(npad) + 32 * stages;
    return need <= 32 ? 32u : (need <= 64 ? 64u : (need <= 128 ? 128u : (need <= 256 ? 256u : 512u)));
}

__device__ __forceinline__ float load_scale_at(const BParams& p, int row, int g) {
    if (p.row_scales) return load_as_f32(p.scales, fastdiv((uint32_t)row, p.rpsdiv), p.scale_kind);
    if (g >= p.G) return 0.f;
    return load_as_f32(p.scales, fastdiv((uint32_t)row * (uint32_t)p.G + (uint32_t)g, p.gvdiv), p.scale_kind);
}

__global__ void __launch_bounds__(kThreads, 1) rvq_gemv_batch_kernel(const __grid_constant__ BParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    char* cbs = reinterpret_cast<char*>(base);                               // 128 KB codebook
    const int xstage_bytes = p.npad * 128;
    uint8_t* xs = base + vdec::kCbBytes;                                     // x stages
    uint64_t* bars = reinterpret_cast<uint64_t*>(xs + p.stages * xstage_bytes);
    // x_full[S] | done[S] | acc_full[2] | acc_free[2]
    const uint32_t bar_x = smem_addr(bars), bar_done = bar_x + 8 * kMaxStages;
    const uint32_t bar_accf = bar_done + 8 * kMaxStages, bar_acce = bar_accf + 16;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kMaxStages + 4);
    __shared__ int last_piece;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int S = p.stages;
    const int cta = blockIdx.x;
    const int64_t u_first = range_begin(p, cta), u_last = range_begin(p, cta + 1);
    const int n_chunks = (int)(u_last - u_first);
    // the CTA's first chunk: (tile, token block) unit and column chunk
    const int unit0 = (int)(u_first / p.KC), kc_first = (int)(u_first - (int64_t)unit0 * p.KC);
    // TMEM: two accumulators of npad columns (the epilogue reads 32 columns at a
    // time), then S weight stages of 32 columns (128 rows x 64 bf16)
    const uint32_t a_base = (uint32_t)a_base_of(p.npad);
    const uint32_t tmem_cols = tmem_cols_of(p.npad, S);

    if (tid == 0) {
        for (int s = 0; s < kMaxStages; ++s) {
            mbar_init(bar_x + 8 * s, 1);
            mbar_init(bar_done + 8 * s, 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(bar_accf + 8 * a, 1);
            mbar_init(bar_acce + 8 * a, kEpiWarps);
        }
        mbar_init_fence();
    }
    if (warp == 0) tmem_alloc(smem_addr(tmem_slot), tmem_cols);
    tc_fence_before();
    __syncthreads();                                                         // barriers initialised

    // ---- x loader: chunk g's x into stage g % S (for g >= S once the MMAs of
    // chunk g - S are done); once it has landed, arrive on the stage barrier
    int x_st = 0, x_ph = 0, x_blk = unit0 % p.blocks, x_kc = kc_first;
    auto load_x = [&](int st) {
        mbar_expect_tx(bar_x + 8 * st, (uint32_t)xstage_bytes);
        tma_load_2d(smem_addr(xs + st * xstage_bytes), &p.xmap, x_kc * kChunk, x_blk * p.npad, bar_x + 8 * st);
        if (++x_kc == p.KC) {
            x_kc = 0;
            if (++x_blk == p.blocks) x_blk = 0;
        }
    };
    if (warp == kProducer && lane == 0)
        for (int g = 0; g < S && g < n_chunks; ++g) load_x(g);

    // ---- decoders: warp w owns TMEM lanes 32 (w % 4) .. + 31 (tile rows) and
    // vectors 2 (w / 4), 2 (w / 4) + 1 of every chunk; thread = one row.  Code
    // words and scales are fetched kPrefetch chunks ahead (the first ones
    // before the codebook is staged); a per-row scale is read once per tile.
    const int quarter = warp & 3, vp = (warp >> 2) & 3;
    const int r = 32 * quarter + lane;
    int f_tile = unit0 / p.blocks, f_blk = unit0 % p.blocks, f_kc = kc_first;
    int s_tile = -1;
    float s_row = 0.f;
    uint2 cw[kPrefetch];
    float cs0[kPrefetch], cs1[kPrefetch];
    auto fetch = [&](uint2& w, float& s0, float& s1) {
        const int row = f_tile * kTileRows + r;
        w = make_uint2(0u, 0u);
        s0 = s1 = 0.f;
        if (row < p.R) {
            const uint32_t* line = p.codes + ((int64_t)(f_kc >> 2) * p.R + row) * 32 + (f_kc & 3) * kChunkVecs;
            w = __ldg(reinterpret_cast<const uint2*>(line) + vp);
            if (p.row_scales) {
                if (f_tile != s_tile) {
                    s_tile = f_tile;
                    s_row = load_as_f32(p.scales, fastdiv((uint32_t)row, p.rpsdiv), p.scale_kind);
                }
                s0 = s1 = s_row;
            } else {
                s0 = load_scale_at(p, row, f_kc * kChunkVecs + 2 * vp);
                s1 = load_scale_at(p, row, f_kc * kChunkVecs + 2 * vp + 1);
            }
        }
        if (++f_kc == p.KC) {
            f_kc = 0;
            if (++f_blk == p.blocks) {
                f_blk = 0;
                ++f_tile;
            }
        }
    };
    if (warp < kDecodeWarps) {
#pragma unroll
        for (int i = 0; i < kPrefetch; ++i)
            if (i < n_chunks) fetch(cw[i], cs0[i], cs1[i]);
    }

    const bool cb_smem = vdec::stage_cb8(p.cb, p.cb_kind, cbs, tid, kThreads);   // ends with a barrier
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp < kDecodeWarps) {
        // Each chunk: decode into registers, wait until the MMAs of chunk g - S
        // have left TMEM stage g % S, store, arrive on the stage barrier.  One
        // loop per codebook source (shared memory, or global for a codebook
        // fp16 cannot hold), so the hot loop holds a single decode path.
        uint32_t lb[4];
        vdec::lane_bits(lane, lb);
        const uint32_t t_lane = tmem + ((uint32_t)(32 * quarter) << 16) + a_base + 8u * (uint32_t)vp;
        auto decode_loop = [&](auto mode_tag) {
            constexpr int kMode = decltype(mode_tag)::value;     // 0 fast, 1 exact, 2 exact from global
            auto decode = [&](uint32_t w, float s) -> uint4 {
                if (kMode == 0) return vdec::weights_bf16_fast(cbs, w, lb, s);
                return vdec::weights_bf16<kMode == 1>(cbs, p.cb, p.cb_kind, w, lb, s);
            };
            int st = 0, ph = 0;
            for (int g0 = 0; g0 < n_chunks; g0 += kPrefetch) {
#pragma unroll
                for (int i = 0; i < kPrefetch; ++i) {
                    const int g = g0 + i;
                    if (g >= n_chunks) break;
                    const uint4 q0 = decode(cw[i].x, cs0[i]);
                    const uint4 q1 = decode(cw[i].y, cs1[i]);
                    if (g + kPrefetch < n_chunks) fetch(cw[i], cs0[i], cs1[i]);
                    if (g >= S) {                                  // the MMAs of chunk g - S left stage st
                        if (lane == 0) mbar_wait(bar_done + 8 * st, ph ^ 1, kWaitLimit, &g_batch_timeout);
                        __syncwarp();
                    }
                    tmem_st8(t_lane + 32u * (uint32_t)st, q0, q1);
                    tmem_st_wait();
                    tc_fence_before();
                    named_arrive(2 + st, kStageBarThreads);
                    if (++st == S) {
                        st = 0;
                        ph ^= 1;
                    }
                }
            }
        };
        if (!cb_smem) decode_loop(std::integral_constant<int, 2>{});
        else if (p.exact) decode_loop(std::integral_constant<int, 1>{});
        else decode_loop(std::integral_constant<int, 0>{});
    } else if (warp == kIssuer) {
        // ---- MMA issuer: once stage g % S holds chunk g's weights and x, four
        // MMAs into the segment's accumulator, committed to done[g % S]
        const uint32_t idesc = instr_desc_bf16(kTileRows, p.npad);
        int st = 0, n_seg = 0;
        for (int64_t u = u_first; u < u_last; ++n_seg) {
            const Seg sg = seg_at(p, u, u_last);
            u += sg.kc1 - sg.kc0;
            const int acc = n_seg & 1;
            if (n_seg >= 2) {                                      // the epilogue has read this accumulator
                if (lane == 0) mbar_wait(bar_acce + 8 * acc, ((n_seg >> 1) - 1) & 1, kWaitLimit, &g_batch_timeout);
                __syncwarp();
            }
            const uint32_t d = tmem + (uint32_t)(acc * p.npad);
            for (int kc = sg.kc0; kc < sg.kc1; ++kc) {
                named_sync(2 + st, kStageBarThreads);
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t wa = tmem + a_base + 32u * (uint32_t)st, xa = smem_addr(xs + st * xstage_bytes);
#pragma unroll
                    for (int ks = 0; ks < kChunk / 16; ++ks)
                        mma_bf16_ts(d, wa + 8u * (uint32_t)ks, sw128_desc(xa + 32 * ks), idesc, kc > sg.kc0 || ks > 0);
                    mma_commit(bar_done + 8 * st);
                    if (kc + 1 == sg.kc1) mma_commit(bar_accf + 8 * acc);
                }
                __syncwarp();
                if (++st == S) st = 0;
            }
        }
    } else if (warp == kProducer) {
        for (int g = 0; g < n_chunks; ++g) {
            if (lane == 0) {
                if (g >= S) {                                      // stage free: the MMAs of chunk g - S are done
                    mbar_wait(bar_done + 8 * x_st, x_ph ^ 1, kWaitLimit, &g_batch_timeout);
                    load_x(x_st);
                }
                mbar_wait(bar_x + 8 * x_st, x_ph, kWaitLimit, &g_batch_timeout);
            }
            __syncwarp();
            named_arrive(2 + x_st, kStageBarThreads);
            if (++x_st == S) {
                x_st = 0;
                x_ph ^= 1;
            }
        }
    } else {
        // ---- epilogue warps: warp e reads TMEM lanes 32 e .. 32 e + 31 (tile rows)
        const int e = warp - kDecodeWarps;
        const int r = 32 * e + lane;
        int n_seg = 0;
        for (int64_t u = u_first; u < u_last; ++n_seg) {
            const Seg sg = seg_at(p, u, u_last);
            u += sg.kc1 - sg.kc0;
            const int acc = n_seg & 1;
            const int tile = sg.unit / p.blocks;
            const int t0 = (sg.unit % p.blocks) * p.npad, nt = min(p.npad, p.T - t0);
            // the CTAs whose ranges hold this unit's chunks: pieces cf .. cl, this CTA's is cta - cf
            const int64_t ubase = (int64_t)sg.unit * p.KC;
            const int cf = cta_of(p, ubase), np = cta_of(p, ubase + p.KC - 1) - cf + 1;
            const int row = tile * kTileRows + r;
            if (lane == 0) mbar_wait_sleep(bar_accf + 8 * acc, (n_seg >> 1) & 1, kWaitLimit, &g_batch_timeout);
            __syncwarp();
            tc_fence_after();
            // partials: [slot][128 rows][npad] fp32, a row's tokens contiguous
            float* part = p.part + ((int64_t)(2 * cta + (n_seg ? 1 : 0)) * kTileRows + r) * p.npad;
            for (int c0 = 0; c0 < p.npad; c0 += 32) {
                uint32_t vals[32];
                tmem_ld32(tmem + ((uint32_t)(32 * e) << 16) + (uint32_t)(acc * p.npad + c0), vals);
                tmem_ld_wait();
                if (np == 1) {
                    const int tn = min(32, nt - c0);
                    if (row < p.R) {
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            if (i < tn)
                                p.y[(int64_t)(t0 + c0 + i) * p.R + row] = __float2bfloat16_rn(__uint_as_float(vals[i]));
                    }
                } else {
                    const int nw = min(32, p.npad - c0);                 // a multiple of 16
#pragma unroll
                    for (int i = 0; i < 32; i += 4)
                        if (i < nw)
                            __stcg(reinterpret_cast<float4*>(part + c0 + i),
                                   make_float4(__uint_as_float(vals[i]), __uint_as_float(vals[i + 1]),
                                               __uint_as_float(vals[i + 2]), __uint_as_float(vals[i + 3])));
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_acce + 8 * acc);
            if (np > 1) {
                // the CTA that finishes the unit's last piece adds the pieces in piece order
                __threadfence();
                asm volatile("bar.sync 1, %0;\n" ::"n"(kEpiWarps * 32) : "memory");
                if (e == 0 && lane == 0) last_piece = atomicAdd(&p.tickets[sg.unit], 1u) == (uint32_t)(np - 1);
                asm volatile("bar.sync 1, %0;\n" ::"n"(kEpiWarps * 32) : "memory");
                if (last_piece) {
                    __threadfence();
                    // piece 0 is CTA cf's last segment unless cf's range starts at this unit;
                    // piece q > 0 is the first segment of CTA cf + q
                    const int slot0 = 2 * cf + (range_begin(p, cf) == ubase ? 0 : 1);
                    if (row < p.R) {
                        for (int tb = 0; tb < nt; tb += kRedTokens) {
                            // kRedTokens tokens of kRedPieces pieces in flight at once
                            float4 sum[kRedTokens / 4];
                            const float4* s0 = reinterpret_cast<const float4*>(
                                p.part + ((int64_t)slot0 * kTileRows + r) * p.npad + tb);
#pragma unroll
                            for (int j = 0; j < kRedTokens / 4; ++j) sum[j] = __ldcg(s0 + j);
                            for (int q0 = 1; q0 < np; q0 += kRedPieces) {
                                float4 v[kRedPieces][kRedTokens / 4];
#pragma unroll
                                for (int qq = 0; qq < kRedPieces; ++qq) {
                                    if (q0 + qq < np) {
                                        const float4* sq = reinterpret_cast<const float4*>(
                                            p.part + ((int64_t)(2 * (cf + q0 + qq)) * kTileRows + r) * p.npad + tb);
#pragma unroll
                                        for (int j = 0; j < kRedTokens / 4; ++j) v[qq][j] = __ldcg(sq + j);
                                    }
                                }
#pragma unroll
                                for (int qq = 0; qq < kRedPieces; ++qq) {
                                    if (q0 + qq < np) {
#pragma unroll
                                        for (int j = 0; j < kRedTokens / 4; ++j) {
                                            sum[j].x += v[qq][j].x;
                                            sum[j].y += v[qq][j].y;
                                            sum[j].z += v[qq][j].z;
                                            sum[j].w += v[qq][j].w;
                                        }
                                    }
                                }
                            }
#pragma unroll
                            for (int j = 0; j < kRedTokens / 4; ++j) {
                                const float f[4] = {sum[j].x, sum[j].y, sum[j].z, sum[j].w};
#pragma unroll
                                for (int k = 0; k < 4; ++k) {
                                    const int t = tb + 4 * j + k;
                                    if (t < nt) p.y[(int64_t)(t0 + t) * p.R + row] = __float2bfloat16_rn(f[k]);
                                }
                            }
                        }
                    }
                    if (e == 0 && lane == 0) p.tickets[sg.unit] = 0u;  // ready for the next launch
                }
                asm volatile("bar.sync 1, %0;\n" ::"n"(kEpiWarps * 32) : "memory");
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem, tmem_cols);
}

// ---------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------
std::mutex g_mu;
bool g_ready[64] = {}, g_ok[64] = {};
int g_sms[64] = {};
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int prepare(int* sms) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64) {
        last_cuda_error_slot() = (int)e;
        return RVQ_ERR_UNAVAILABLE;
    }
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_ready[dev]) {
        g_ready[dev] = true;
        cudaDeviceProp prop;
        e = cudaGetDeviceProperties(&prop, dev);
        if (e == cudaSuccess && prop.major == 10 && prop.sharedMemPerBlockOptin >= (size_t)kBudget) {
            g_sms[dev] = prop.multiProcessorCount;
            e = cudaFuncSetAttribute(rvq_gemv_batch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kBudget);
            if (e == cudaSuccess && g_encode == nullptr) {
                void* fn = nullptr;
                cudaDriverEntryPointQueryResult q;
                e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
                if (e == cudaSuccess && q == cudaDriverEntryPointSuccess)
                    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
            }
            g_ok[dev] = e == cudaSuccess && g_encode != nullptr;
        }
        if (e != cudaSuccess) last_cuda_error_slot() = (int)e;
    }
    *sms = g_sms[dev];
    return g_ok[dev] ? RVQ_OK : RVQ_ERR_UNAVAILABLE;
}

// Tokens per block (the MMA N, a multiple of 16): all of them up to
// kBlockTokens, else the prompt cut into equal blocks of at most kBlockTokens.
int npad_of(int64_t T) {
    const int64_t nb = (T + kBlockTokens - 1) / kBlockTokens;
    const int64_t per = (T + nb - 1) / nb;
    return (int)((per + 15) / 16 * 16);
}

int stages_for(int npad) {
    int s = (kBudget - 1024 - vdec::kCbBytes - 256) / (npad * 128);
    s = s > kMaxStages ? kMaxStages : s;
    while (s > 1 && a_base_of(npad) + 32 * s > 512) --s;
    return s;
}

// The balanced split's sizes.  Returns the workspace bytes it needs (two
// partial slots per CTA, then one ticket per (tile, token block) unit) or a
// negative status.
int64_t plan(const rvq_gemv_batch_job& j, int sms, BParams* p) {
    const int64_t R = j.rows, G = j.cols / 8, T = j.tokens;
    const int64_t KC = (G + kChunkVecs - 1) / kChunkVecs;
    const int64_t NT = (R + kTileRows - 1) / kTileRows;
    const int64_t npad = npad_of(T), NB = (T + npad - 1) / npad;
    const int64_t NU = NT * NB;                                   // (tile, token block) units
    const int64_t U = NU * KC;
    if (U >= (1ll << 31)) return -RVQ_ERR_TOO_LARGE;
    const int64_t ctas = sms < U ? sms : U;
    if (p) {
        p->U = U;
        p->KC = (int32_t)KC;
        p->n_ctas = (int32_t)ctas;
        p->npad = (int32_t)npad;
        p->blocks = (int32_t)NB;
    }
    const int64_t part_bytes = (2 * ctas * npad * kTileRows * 4 + 255) / 256 * 256;
    return part_bytes + NU * 4;
}

int check_job(const rvq_gemv_batch_job* j) {
    if (j == nullptr || j->x == nullptr || j->y == nullptr) return RVQ_ERR_INVALID;
    const rvq_entry& w = j->weight;
    int rc = rvq_check_entry(&w);
    if (rc != RVQ_OK) return rc;
    if (w.stages != 4 || w.ncodes != 256 || w.index_kind != RVQ_U8 || w.d != 8) return RVQ_ERR_UNSUPPORTED;
    if (j->rows < 1 || j->cols < 8 || j->cols % 8 || j->tokens < 1 || j->tokens > kMaxTokens)
        return RVQ_ERR_UNSUPPORTED;
    if (j->rows * (j->cols / 8) != w.nvec || w.trimmed != w.nvec * 8 || w.tail_numel != 0) return RVQ_ERR_UNSUPPORTED;
    if (j->x_kind != RVQ_BF16 || j->y_kind != RVQ_BF16) return RVQ_ERR_UNSUPPORTED;
    if (w.codebook_kind != RVQ_F32 && w.codebook_kind != RVQ_F16 && w.codebook_kind != RVQ_BF16)
        return RVQ_ERR_UNSUPPORTED;
    if (((uintptr_t)w.indices & 15) || ((uintptr_t)j->x & 15) || ((j->cols * 2) & 15)) return RVQ_ERR_INVALID;
    if (w.nvec >= (1ll << 32) || j->rows >= (1ll << 24) || (j->cols / kChunk) >= (1 << 16)) return RVQ_ERR_TOO_LARGE;
    return RVQ_OK;
}

}  // namespace batch
}  // namespace rvq

using namespace rvq;
using namespace rvq::batch;

extern "C" {

size_t rvq_gemv_batch_workspace_size(const rvq_gemv_batch_job* job) {
    if (check_job(job) != RVQ_OK) return 0;
    int sms = 0;
    if (prepare(&sms) != RVQ_OK) return 0;
    const int64_t b = plan(*job, sms, nullptr);
    return b < 0 ? 0 : (size_t)b;
}

int rvq_gemv_batch(const rvq_gemv_batch_job* job, void* workspace, size_t workspace_bytes, void* stream) {
    int rc = check_job(job);
    if (rc != RVQ_OK) return rc;
    int sms = 0;
    rc = prepare(&sms);
    if (rc != RVQ_OK) return rc;
    BParams p;
    memset(&p, 0, sizeof(p));
    const int64_t need = plan(*job, sms, &p);
    if (need < 0) return (int)-need;
    if (workspace == nullptr || workspace_bytes < (size_t)need || ((uintptr_t)workspace & 255)) return RVQ_ERR_INVALID;
    const rvq_entry& w = job->weight;
    p.stages = stages_for(p.npad);
    const cuuint64_t dims[2] = {(cuuint64_t)job->cols, (cuuint64_t)job->tokens};
    const cuuint64_t strides[1] = {(cuuint64_t)job->cols * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kChunk, (cuuint32_t)p.npad};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult cr = g_encode(&p.xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(job->x), dims, strides,
                                 box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return RVQ_ERR_INVALID;
    const int64_t NU = (job->rows + kTileRows - 1) / kTileRows * p.blocks;
    p.codes = reinterpret_cast<const uint32_t*>(w.indices);
    p.cb = w.codebook;
    p.scales = w.scales;
    p.y = reinterpret_cast<__nv_bfloat16*>(job->y);
    p.part = reinterpret_cast<float*>(workspace);
    p.tickets = reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(workspace) + (size_t)need - (size_t)NU * 4);
    p.R = (int32_t)job->rows;
    p.G = (int32_t)(job->cols / 8);
    p.T = (int32_t)job->tokens;
    p.cb_kind = w.codebook_kind;
    p.scale_kind = w.scale_kind;
    p.exact = job->exact ? 1 : 0;
    const uint32_t gv = (uint32_t)w.group_vecs;
    p.gvdiv = make_fastdiv(gv);
    p.row_scales = gv % (uint32_t)p.G == 0;
    p.rpsdiv = make_fastdiv(p.row_scales ? gv / (uint32_t)p.G : 1u);
    const size_t smem = 1024 + (size_t)vdec::kCbBytes + (size_t)p.stages * p.npad * 128 + 256;
    rvq_gemv_batch_kernel<<<p.n_ctas, kThreads, smem, (cudaStream_t)stream>>>(p);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        last_cuda_error_slot() = (int)e;
        return RVQ_ERR_CUDA;
    }
    return RVQ_OK;
}

int rvq_take_batch_timeout(void) {
    int v = 0;
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&v, g_batch_timeout, sizeof(int));
    const int zero = 0;
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_batch_timeout, &zero, sizeof(int));
    if (e != cudaSuccess) {
        last_cuda_error_slot() = (int)e;
        return -RVQ_ERR_CUDA;
    }
    return v;
}

}  // extern "C"
