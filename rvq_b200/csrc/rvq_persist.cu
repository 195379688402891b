// Persistent batch-1 decode step (sm_100a): ONE cooperative launch, one CTA
// of 1024 threads per SM, runs every layer of a Qwen3 decoder for one token.
// It replaces the seven launches per layer of the plain step (rvq_step_norm,
// rvq_gemv_tiles x 4, rvq_step_attention, rvq_step_norm), i.e. the per-layer
// module calls of the reference's _layerwise_logits
// (infer_compressed_layerwise_triton.py:271-292) with the weights never
// materialised.
//
// Per layer l the CTAs go through
//   norm1  CTAs 0..7: h += down partials (layer 0: h = embed row), each CTA
//          one eighth of h and its sum of squares (the 8 ranks of
//          rvq_step_norm's cluster);
//   qkv    every CTA: its table-GEMV units (rvq_tiles.cuh), the operand
//          x = ln1 * bf16(h * inv) computed per 256-column tile;
//   attn   CTAs G - n_kv .. G - 1: one kv head each, the 8 key ranges of
//          rvq_step_attention's cluster handled in turn inside the CTA;
//   o      every CTA, operand attn_out;
//   norm2  CTAs 0..7: h += o partials;
//   gu     every CTA, operand ln2 * bf16(h * inv);
//   down   every CTA, operand bf16(silu(gate)) * up from the partials;
// and after the last layer the final norm writes x_final.
//
// Every phase repeats, in the same order, the fp32 arithmetic of the kernel it
// replaces (the norm's per-rank sums of squares added in rank order, the
// attention's per-range maxima, sums and P V partial sums combined in range
// order), so h, x_final and the KV cache are bit-identical to the plain step.
//
// Hand-over between phases: monotonic counters in global memory (norm
// arrivals, GEMV-phase arrivals spread over 16 counters, attention arrivals,
// exit), each on a 128-byte line of its own.  A producer CTA synchronises,
// then its thread 0 adds 1 with a release reduction; a consumer polls with
// relaxed loads spaced by 100 ns and issues one acquire fence once the count
// for this layer is reached (about one second at most, then a sticky error
// flag and no further waits).  Every CTA passes the
// phase's wait before it arrives, even one without work in the phase, so no
// CTA arrives at phase k + 1 before all have arrived at phase k, and a count
// of k x (arrivals per phase) therefore means phases 1..k are complete.  A CTA
// starts the code-word copies of its next GEMV unit and stages the codebook
// before it waits for the operand.  The last CTA to leave resets the
// counters, so every step starts from zero.  All CTAs are co-resident
// (cooperative launch), and every wait is on an earlier phase, so no wait can
// depend on a CTA that waits for it.
//
// Data written inside the launch and read by other CTAs (h, the partials,
// attn_out, the norm sums) is read through L2 (ld.global.cg), never through
// the read-only path.

#include <memory>
#include <mutex>
#include <string.h>
#include <vector>

#include "rvq_common.cuh"
#include "rvq_stepops.cuh"
#include "rvq_tiles.cuh"

namespace rvq {
namespace tiles {
int check_job(const rvq_gemv_tile_job& g);      // rvq_gemv_tiles.cu
}  // namespace tiles

namespace persist {

using namespace stepops;
using tiles::TileSmem;
using tiles::TJob;
using tiles::UnitState;
using tiles::kTileCols;

constexpr int kThreads = tiles::kThreads;          // 1024
constexpr int kWarps = kThreads / 32;
constexpr int kRanks = 8;                          // norm slices / attention key ranges
constexpr int kHD = 128;
constexpr int kE = kHD / 32;
constexpr int kMaxRep = 8;
constexpr int kNormMaxSlice = 2048;                // two elements per thread
// attention scratch: the table, codebook and ring space (floats); the P V
// partial of every (range, warp) for 4 heads sits in its last 128 KB
constexpr int kScratch = tiles::kLutWords + tiles::kCbFloats + tiles::kRing * tiles::kBatchRows * tiles::kGroups;
constexpr int kAttnFixed = 8592;
constexpr int kMaxScores = 15360;                  // rep * max_len
constexpr int kPvOffset = tiles::kLutWords + tiles::kCbFloats;
constexpr int kPvFloats = kRanks * 8 * 4 * 128;    // [range][warp][head of 4][HD]
static_assert(kAttnFixed + kMaxScores <= kPvOffset && kPvOffset + kPvFloats <= kScratch, "attention scratch");
constexpr int kPhases = 4;                         // GEMV phases per layer

// sync words: each counter and the norm sums on a 128-byte line of its own
// (the counters are polled by every CTA; the sums are read by one thread per
// CTA).  GEMV-phase arrivals are spread over kSub counters (CTA c adds to
// counter c % kSub), so that 148 CTAs finishing together do not queue on one
// address.
constexpr int kSub = 16;
enum { kCtrNorm = 0, kCtrAttn = 32, kCtrExit = 64, kSsWord = 96, kCtrGemv = 128 };
static_assert(kCtrGemv + 32 * kSub <= RVQ_PERSIST_SYNC_WORDS, "sync words");

static __device__ int g_persist_error;             // sticky: a phase wait gave up, or a bad grid

struct PPhase {
    TJob jobs[3];
    int32_t n_jobs;
    int32_t cta_first;                             // offset of this phase's [n_ctas + 1] unit bounds
};

struct PLayer {
    const void* ln1;
    const void* ln2;
    const void* q_norm;
    const void* k_norm;
    void* k_cache;
    void* v_cache;
    PPhase ph[kPhases];
};

struct PHead {
    rvq_persist_model m;
    int32_t n_ctas;
    int32_t hid_tiles;                             // tiles of a hidden-wide operand
    int32_t o_tiles;                               // tiles of the o projection's columns
    int32_t inter_tiles;                           // tiles of the down projection's columns
    int64_t layers_off;                            // byte offsets from the plan's start
    int64_t cta_first_off;
    int64_t unit_jt_off;
    int64_t unit_r0_off;
    int64_t unit_r1_off;
};

template <typename T>
__device__ __forceinline__ const T* at(const PHead* P, int64_t off) {
    return reinterpret_cast<const T*>(reinterpret_cast<const char*>(P) + off);
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t ld_relaxed(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Every thread: returns once *ctr >= target (thread 0 polls with relaxed
// loads, spaced out so that a hundred waiting CTAs do not crowd the counter's
// L2 line, then one acquire fence), or after about a second without it (then
// the sticky flag is set and this CTA waits no more).
__device__ __forceinline__ void wait_count(const uint32_t* ctr, uint32_t target, volatile int* failed) {
    if (threadIdx.x == 0 && !*failed) {
        const uint64_t t0 = globaltimer_ns();
        bool ok = false;
        for (uint32_t i = 0; i < (1u << 24); ++i) {
            if ((int32_t)(ld_relaxed(ctr) - target) >= 0) {
                ok = true;
                break;
            }
            __nanosleep(100);
            if ((i & 63) == 0 && globaltimer_ns() - t0 > 1000000000ull) break;
        }
        if (ok) {
            asm volatile("fence.acq_rel.gpu;\n" ::: "memory");
        } else {
            atomicExch(&g_persist_error, 1);
            *failed = 1;
        }
    }
    __syncthreads();
}

// Every thread: returns once every CTA has arrived at `phases` GEMV phases
// (lane k < kSub of warp 0 polls counter k against its share of the CTAs).
__device__ __forceinline__ void wait_gemv(const uint32_t* ctr, int G, uint32_t phases, volatile int* failed) {
    const int k = threadIdx.x;
    if (k < kSub && !*failed) {
        const uint32_t target = (uint32_t)(G / kSub + (k < G % kSub ? 1 : 0)) * phases;
        const uint32_t* p = ctr + kCtrGemv + 32 * k;
        const uint64_t t0 = globaltimer_ns();
        bool ok = false;
        for (uint32_t i = 0; i < (1u << 24); ++i) {
            if ((int32_t)(ld_relaxed(p) - target) >= 0) {
                ok = true;
                break;
            }
            __nanosleep(100);
            if ((i & 63) == 0 && globaltimer_ns() - t0 > 1000000000ull) break;
        }
        if (ok) {
            asm volatile("fence.acq_rel.gpu;\n" ::: "memory");
        } else {
            atomicExch(&g_persist_error, 1);
            *failed = 1;
        }
    }
    __syncthreads();
}

// Every thread: this CTA's writes so far are published (the barrier, then a
// release add by thread 0), and the counter advances.
__device__ __forceinline__ void arrive(uint32_t* ctr) {
    __syncthreads();
    if (threadIdx.x == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;\n" ::"l"(ctr) : "memory");
}

// ---------------------------------------------------------------------------
// RMSNorm (rvq_step_norm's rank `rank` of 8)
// ---------------------------------------------------------------------------

// h[slice] <- embed row (first) or h + add, kept in keep0 / keep1 (elements
// lo + tid and lo + tid + 1024); the slice's sum of squares to ss[rank].
__device__ __noinline__ void norm_slice(const PHead* P, int rank, const rvq_vec* add, bool first, float& keep0,
                                        float& keep1, float* warp_ss) {
    const rvq_persist_model& m = P->m;
    const int H = m.hidden;
    const int slice = (H + kRanks - 1) / kRanks;
    const int lo = rank * slice, hi = min(H, lo + slice);
    const int tid = threadIdx.x;
    float ss = 0.f;
    int64_t row = 0;
    if (first) {
        const int64_t tok = *m.token;
        row = (tok >= 0 && tok < m.vocab ? tok : 0) * (int64_t)H;
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const int i = lo + tid + k * kThreads;
        if (i < hi) {
            float hv;
            if (first) {
                hv = bf16_at(m.embed, row + i);
            } else {
                hv = ldcg_f32(m.h, i, RVQ_BF16);
                hv = bf16r(hv + vec_value_deep<true>(*add, i));
            }
            put_bf16(m.h, i, hv);
            if (k == 0) keep0 = hv;
            else keep1 = hv;
            ss = fmaf(hv, hv, ss);
        }
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) warp_ss[tid >> 5] = ss;
    __syncthreads();
    if (tid == 0) {
        float t = 0.f;
        for (int w = 0; w < kWarps; ++w) t += warp_ss[w];
        __stcg(reinterpret_cast<float*>(m.sync + kSsWord) + rank, t);
    }
}

// rsqrt(mean(h^2) + eps) from the 8 slices' sums, added in rank order; thread
// 0 reads them, the others get the result through shared memory.
__device__ __forceinline__ float norm_inv(const PHead* P, float* inv_sh) {
    if (threadIdx.x == 0) {
        const float* ss = reinterpret_cast<const float*>(P->m.sync + kSsWord);
        float v[kRanks];
#pragma unroll
        for (int r = 0; r < kRanks; ++r) v[r] = __ldcg(ss + r);
        float total = 0.f;
#pragma unroll
        for (int r = 0; r < kRanks; ++r) total += v[r];
        *inv_sh = rsqrtf(total / (float)P->m.hidden + P->m.eps);
    }
    __syncthreads();
    return *inv_sh;
}

// The GEMV operand of a normed phase: x = bf16(w * bf16(h * inv)) over the tile.
__device__ __forceinline__ void stage_normed(const PHead* P, const TJob& J, int tile, const void* w, float inv,
                                             const TileSmem& S) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid < kTileCols) {
        const int64_t col = (int64_t)tile * kTileCols + tid;
        float xv = 0.f;
        if (col < J.cols) xv = bf16r(bf16_at(w, col) * bf16r(ldcg_f32(P->m.h, col, RVQ_BF16) * inv));
        S.xs[tid] = xv;
        float mx = fabsf(xv);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) S.xmax[warp] = mx;
    }
}

// ---------------------------------------------------------------------------
// Decode attention of kv head `kv` (rvq_step_attention's 8-CTA cluster, the
// ranges handled inside one CTA): scratch `sm` is the table + codebook space.
// ---------------------------------------------------------------------------
__device__ __noinline__ void attend(const PHead* P, const PLayer& Ly, int kv, float* sm) {
    const rvq_persist_model& m = P->m;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int rep = m.n_heads / m.n_kv;
    const int max_len = m.max_len;
    const int64_t out0 = (int64_t)kv * rep * kHD;
    const int64_t pos = *m.pos;
    if (pos < 0 || pos >= max_len) {
        for (int i = tid; i < rep * kHD; i += kThreads) put_bf16(m.attn_out, out0 + i, 0.f);
        return;
    }
    const int L = (int)pos + 1;
    const int kpc = (L + kRanks - 1) / kRanks;     // keys per range
    float* raw = sm;                               // [rep + 2][HD]: q heads, k, v
    float* qs = sm + 1280;                         // [rep][HD] after norm + rope
    float* knew = sm + 2304;
    float* vnew = knew + kHD;
    float* wsm = sm + 2560;                        // q_norm, k_norm, cos[pos], sin[pos]
    float* pw = sm + kPvOffset;                    // [range][warp][4 heads][HD] P V partials
    float* oacc = sm + 7168;                       // [rep * HD]: the ranges' sum
    float* mloc = sm + 8192;                       // [range][head] maxima
    float* sloc = sm + 8256;                       // [range][head] sums
    float* red = sm + 8320;                        // [4 ranges][head][warp]
    float* gmax = sm + 8576;
    float* gsum = sm + 8584;
    float* sc = sm + kAttnFixed;                   // [rep][max_len] scores, then probabilities
    const __nv_bfloat16* kc = reinterpret_cast<const __nv_bfloat16*>(Ly.k_cache) + (int64_t)kv * max_len * kHD;
    const __nv_bfloat16* vc = reinterpret_cast<const __nv_bfloat16*>(Ly.v_cache) + (int64_t)kv * max_len * kHD;
    const rvq_vec qv = {m.q_part, (int64_t)m.n_heads * kHD, P->hid_tiles, RVQ_F32};
    const rvq_vec kvv = {m.k_part, (int64_t)m.n_kv * kHD, P->hid_tiles, RVQ_F32};
    const rvq_vec vv = {m.v_part, (int64_t)m.n_kv * kHD, P->hid_tiles, RVQ_F32};

    // 1. operands (tile sums of the q / k / v partials) and this position's tables
    for (int i = tid; i < 4 * kHD; i += kThreads) {
        const int which = i / kHD, d = i - which * kHD;
        const void* src = which == 0 ? Ly.q_norm : which == 1 ? Ly.k_norm : which == 2 ? m.cos : m.sin;
        wsm[i] = bf16_at(src, (which >= 2 ? pos * kHD : 0) + d);
    }
    for (int i = tid; i < (rep + 2) * kHD; i += kThreads) {
        const int r = i / kHD, d = i - r * kHD;
        raw[i] = r < rep ? vec_value<true>(qv, ((int64_t)kv * rep + r) * kHD + d)
               : r == rep ? vec_value<true>(kvv, (int64_t)kv * kHD + d)
                          : vec_value<true>(vv, (int64_t)kv * kHD + d);
    }
    __syncthreads();

    // 2. norm + rope (warp per head), the new k and v appended to the cache
    const int64_t cache_row = ((int64_t)kv * max_len + pos) * kHD;
    for (int hh = warp; hh <= rep; hh += kWarps) {
        float o[kE];
        const bool is_k = hh == rep;
        norm_rope_head<kHD>(raw + hh * kHD, wsm + (is_k ? kHD : 0), m.eps, wsm + 2 * kHD, wsm + 3 * kHD, o);
#pragma unroll
        for (int j = 0; j < kE; ++j) {
            const int d = lane + 32 * j;
            if (!is_k) {
                qs[hh * kHD + d] = o[j];
            } else {
                knew[d] = o[j];
                vnew[d] = raw[(rep + 1) * kHD + d];
                put_bf16(Ly.k_cache, cache_row + d, o[j]);
                put_bf16(Ly.v_cache, cache_row + d, vnew[d]);
            }
        }
    }
    __syncthreads();

    // 3. scores: warp per key (4 keys' rows loaded first), lane quad q ends up
    //    with head q of the reduce-scatter
    const int d0 = lane * kE;
    const int hq = (lane >> 2) & 7;
    for (int jb = warp; jb < L; jb += kWarps * 4) {
        float kd[4][kE];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int j = jb + c * kWarps;
            if (j == pos || j >= L) {
#pragma unroll
                for (int e = 0; e < kE; ++e) kd[c][e] = knew[d0 + e];
            } else {
                load_row_slice<kE>(kc + (int64_t)j * kHD + d0, kd[c]);
            }
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int j = jb + c * kWarps;
            if (j >= L) break;                     // warp-uniform
            float pr[8];
#pragma unroll
            for (int r = 0; r < 8; ++r) {
                float t = 0.f;
                if (r < rep) {
#pragma unroll
                    for (int e = 0; e < kE; ++e) t = fmaf(qs[r * kHD + d0 + e], kd[c][e], t);
                }
                pr[r] = t;
            }
            const float t = reduce8(pr);
            if ((lane & 3) == 0 && hq < rep) sc[hq * max_len + j] = bf16r(bf16r(bf16r(t) * m.scaling) + m.valid_bias);
        }
    }
    __syncthreads();

    // 4. softmax: each range's max and sum of exp(s - its max) (the sum as the
    //    cluster CTA forms it: thread t of 256 over keys j0 + t + 256 i, lane
    //    reduce-scatter, warps in order); then the ranges combined in order
    for (int q = warp; q < kRanks * rep; q += kWarps) {
        const int r = q / rep, h = q - r * rep;
        const int j0 = r * kpc, j1 = min(L, j0 + kpc);
        float mx = -INFINITY;
        for (int j = j0 + lane; j < j1; j += 32) mx = fmaxf(mx, sc[h * max_len + j]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) mloc[r * 8 + h] = mx;
    }
    __syncthreads();
    for (int p = 0; p < 2; ++p) {
        const int q = tid >> 8, t = tid & 255, r = 4 * p + q;
        const int j0 = r * kpc, j1 = min(L, j0 + kpc);
        float s8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) s8[i] = 0.f;
        for (int j = j0 + t; j < j1; j += 256) {
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (i < rep) s8[i] += expf(sc[i * max_len + j] - mloc[r * 8 + i]);
        }
        const float tot = reduce8(s8);
        if ((lane & 3) == 0 && hq < rep) red[q * 64 + hq * 8 + (t >> 5)] = tot;
        __syncthreads();
        if (tid < 4 * rep) {
            const int qq = tid / rep, h = tid - qq * rep;
            float a = 0.f;
            for (int w = 0; w < 8; ++w) a += red[qq * 64 + h * 8 + w];
            sloc[(4 * p + qq) * 8 + h] = a;
        }
        __syncthreads();
    }
    if (tid < rep) {
        float mx = -INFINITY;
        for (int c = 0; c < kRanks; ++c) mx = fmaxf(mx, mloc[c * 8 + tid]);
        float t = 0.f;
        for (int c = 0; c < kRanks; ++c) {
            const float s = sloc[c * 8 + tid];
            if (s > 0.f) t += s * expf(mloc[c * 8 + tid] - mx);
        }
        gmax[tid] = mx;
        gsum[tid] = t;
    }
    __syncthreads();
    for (int i = tid; i < rep * L; i += kThreads) {
        const int h = i / L, j = i - h * L;
        float* s = sc + h * max_len + j;
        *s = bf16r(expf(*s - gmax[h]) / gsum[h]);
    }
    __syncthreads();

    // 5. P V: warp w of range r takes keys j0 + w + 8 i (in increasing order),
    //    4 heads at a time, and stores its partial; then each output element
    //    adds a range's 8 warps in warp order and the ranges in range order
    for (int hg = 0; hg < rep; hg += 4) {
        for (int p = 0; p < 2; ++p) {
            const int w = warp & 7, r = 4 * p + (warp >> 3);
            const int j0 = r * kpc, j1 = min(L, j0 + kpc);
            float acc[4][kE];
#pragma unroll
            for (int h = 0; h < 4; ++h)
#pragma unroll
                for (int e = 0; e < kE; ++e) acc[h][e] = 0.f;
            for (int jb = j0 + w; jb < j1; jb += 8 * 4) {
                float vd[4][kE];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const int j = jb + c * 8;
                    if (j == pos || j >= j1) {
#pragma unroll
                        for (int e = 0; e < kE; ++e) vd[c][e] = vnew[d0 + e];
                    } else {
                        load_row_slice<kE>(vc + (int64_t)j * kHD + d0, vd[c]);
                    }
                }
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const int j = jb + c * 8;
                    if (j >= j1) break;
#pragma unroll
                    for (int h = 0; h < 4; ++h) {
                        if (hg + h < rep) {
                            const float pv = sc[(hg + h) * max_len + j];
#pragma unroll
                            for (int e = 0; e < kE; ++e) acc[h][e] = fmaf(pv, vd[c][e], acc[h][e]);
                        }
                    }
                }
            }
#pragma unroll
            for (int h = 0; h < 4; ++h)
#pragma unroll
                for (int e = 0; e < kE; ++e) pw[((r * 8 + w) * 4 + h) * kHD + d0 + e] = acc[h][e];
        }
        __syncthreads();
        const int nh = min(4, rep - hg);
        for (int i = tid; i < nh * kHD; i += kThreads) {
            float t = 0.f;
            for (int r = 0; r < kRanks; ++r) {
                const float* q = pw + (r * 8 * 4) * kHD + i;     // warp 0 of range r, head i / HD
                float u = q[0];
#pragma unroll
                for (int w = 1; w < 8; ++w) u += q[w * 4 * kHD];
                t += u;
            }
            oacc[hg * kHD + i] = t;
        }
        __syncthreads();
    }
    for (int i = tid; i < rep * kHD; i += kThreads) put_bf16(m.attn_out, out0 + i, oacc[i]);
}

// ---------------------------------------------------------------------------
// GEMV phases
// ---------------------------------------------------------------------------

// Thread 0 starts the copies of this CTA's first unit of the phase (false:
// the CTA has no unit in it).  The ring must be idle.
__device__ __forceinline__ bool prefetch_phase(const PHead* P, const PPhase& ph, const TileSmem& S) {
    const int32_t* cf = at<int32_t>(P, P->cta_first_off) + ph.cta_first;
    const int u0 = cf[blockIdx.x];
    if (u0 >= cf[blockIdx.x + 1]) return false;
    const uint32_t jt = at<uint32_t>(P, P->unit_jt_off)[u0];
    tiles::issue_unit_loads(ph.jobs[jt >> 24], (int)(jt & 0xffffffu), at<int32_t>(P, P->unit_r0_off)[u0],
                            at<int32_t>(P, P->unit_r1_off)[u0], S);
    return true;
}

// This CTA's units of the phase.  `wait()` runs once, before the first
// operand is staged; `stage(J, tile)` fills the tile's operand.
template <class Wait, class Stage>
__device__ __forceinline__ void gemv_phase(const PHead* P, const PPhase& ph, TJob* sjobs, const TileSmem& S,
                                           UnitState& st, bool prefetched, Wait&& wait, Stage&& stage) {
    const int32_t* cf = at<int32_t>(P, P->cta_first_off) + ph.cta_first;
    const int u0 = cf[blockIdx.x], u1 = cf[blockIdx.x + 1];
    if (u0 >= u1) {                                  // no units: still wait, so that this CTA's
        wait();                                      // arrival cannot run ahead of the phase before
        return;
    }
    {   // the phase's jobs into shared memory (read on every row batch)
        constexpr int kWords = (int)(sizeof(TJob) / 4);
        static_assert(sizeof(TJob) % 4 == 0, "TJob words");
        const uint32_t* src = reinterpret_cast<const uint32_t*>(ph.jobs);
        uint32_t* dst = reinterpret_cast<uint32_t*>(sjobs);
        for (int i = threadIdx.x; i < ph.n_jobs * kWords; i += kThreads) dst[i] = src[i];
        __syncthreads();
    }
    const uint32_t* ujt = at<uint32_t>(P, P->unit_jt_off);
    const int32_t* ur0 = at<int32_t>(P, P->unit_r0_off);
    const int32_t* ur1 = at<int32_t>(P, P->unit_r1_off);
    for (int u = u0; u < u1; ++u) {
        const uint32_t jt = ujt[u];
        const TJob& J = sjobs[jt >> 24];
        const int tile = (int)(jt & 0xffffffu);
        if (u != u0) __syncthreads();                // the previous unit is done with shared memory
        tiles::run_unit(J, tile, ur0[u], ur1[u], S, st, !(prefetched && u == u0), [&] {
            if (u == u0) wait();
            stage(J, tile);
        });
    }
}

__global__ void __launch_bounds__(kThreads, 1) rvq_persist_kernel(const PHead* __restrict__ P) {
    extern __shared__ __align__(128) float smem[];
    __shared__ int slot_done[tiles::kRing];
    __shared__ float xmax[kTileCols / 32];
    __shared__ volatile int aborted;
    __shared__ volatile int failed;
    __shared__ float warp_ss[kWarps];
    __shared__ float inv_sh;
    __shared__ TJob sjobs[3];
    const TileSmem S = tiles::tile_smem(smem, slot_done, xmax, &aborted);
    if (threadIdx.x == 0) failed = 0;
    tiles::tile_smem_init(S);
    if ((int)gridDim.x != P->n_ctas) {               // the same decision in every CTA
        if (threadIdx.x == 0) atomicExch(&g_persist_error, 2);
        return;
    }
    const rvq_persist_model& m = P->m;
    const int G = (int)gridDim.x, c = (int)blockIdx.x, L = m.n_layers;
    const PLayer* layers = at<PLayer>(P, P->layers_off);
    uint32_t* ctr = m.sync;
    uint32_t* gemv_ctr = ctr + kCtrGemv + 32 * (c % kSub);
    const bool norm_cta = c < kRanks;
    const int kv = c - (G - m.n_kv);                 // >= 0: this CTA attends for kv head kv
    const rvq_vec down_v = {m.down_part, m.hidden, P->inter_tiles, RVQ_F32};
    const rvq_vec o_v = {m.o_part, m.hidden, P->o_tiles, RVQ_F32};
    UnitState st;
    float keep0 = 0.f, keep1 = 0.f, inv = 0.f;
    const uint32_t G32 = (uint32_t)G;
    auto stage_op = [&](const TJob& J, int tile) { tiles::stage_operand(J, tile, S); };

    for (int l = 0; l < L; ++l) {
        const PLayer& Ly = layers[l];
        const uint32_t l32 = (uint32_t)l;
        bool pre = false;
        if (norm_cta) {                              // norm 1
            pre = prefetch_phase(P, Ly.ph[0], S);
            if (l > 0) wait_gemv(ctr, G, 4 * l32, &failed);
            norm_slice(P, c, &down_v, l == 0, keep0, keep1, warp_ss);
            arrive(ctr + kCtrNorm);
        }
        gemv_phase(P, Ly.ph[0], sjobs, S, st, pre,
                   [&] {
                       wait_count(ctr + kCtrNorm, kRanks * (2 * l32 + 1), &failed);
                       inv = norm_inv(P, &inv_sh);
                   },
                   [&](const TJob& J, int tile) { stage_normed(P, J, tile, Ly.ln1, inv, S); });
        arrive(gemv_ctr);

        pre = false;
        if (kv >= 0) {                               // attention (its scratch takes the ring too)
            wait_gemv(ctr, G, 4 * l32 + 1, &failed);
            attend(P, Ly, kv, reinterpret_cast<float*>(S.lut));
            st.cb = nullptr;                         // the codebook space was scratch
            arrive(ctr + kCtrAttn);
        }
        gemv_phase(P, Ly.ph[1], sjobs, S, st, pre,
                   [&] { wait_count(ctr + kCtrAttn, (uint32_t)m.n_kv * (l32 + 1), &failed); }, stage_op);
        arrive(gemv_ctr);

        pre = false;
        if (norm_cta) {                              // norm 2
            pre = prefetch_phase(P, Ly.ph[2], S);
            wait_gemv(ctr, G, 4 * l32 + 2, &failed);
            norm_slice(P, c, &o_v, false, keep0, keep1, warp_ss);
            arrive(ctr + kCtrNorm);
        }
        gemv_phase(P, Ly.ph[2], sjobs, S, st, pre,
                   [&] {
                       wait_count(ctr + kCtrNorm, kRanks * (2 * l32 + 2), &failed);
                       inv = norm_inv(P, &inv_sh);
                   },
                   [&](const TJob& J, int tile) { stage_normed(P, J, tile, Ly.ln2, inv, S); });
        arrive(gemv_ctr);

        gemv_phase(P, Ly.ph[3], sjobs, S, st, false,
                   [&] { wait_gemv(ctr, G, 4 * l32 + 3, &failed); }, stage_op);
        arrive(gemv_ctr);
    }

    if (norm_cta) {                                  // final norm
        const uint32_t L32 = (uint32_t)L;
        wait_gemv(ctr, G, 4 * L32, &failed);
        norm_slice(P, c, &down_v, false, keep0, keep1, warp_ss);
        arrive(ctr + kCtrNorm);
        wait_count(ctr + kCtrNorm, kRanks * (2 * L32 + 1), &failed);
        inv = norm_inv(P, &inv_sh);
        const int H = m.hidden;
        const int slice = (H + kRanks - 1) / kRanks;
        const int lo = c * slice, hi = min(H, lo + slice);
        const int i0 = lo + (int)threadIdx.x, i1 = i0 + kThreads;
        if (i0 < hi) put_bf16(m.x_final, i0, bf16_at(m.final_norm, i0) * bf16r(keep0 * inv));
        if (i1 < hi) put_bf16(m.x_final, i1, bf16_at(m.final_norm, i1) * bf16r(keep1 * inv));
    }

    __syncthreads();                                 // leave; the last CTA out resets the counters
    if (threadIdx.x == 0) {
        __threadfence();
        const uint32_t old = atomicAdd(ctr + kCtrExit, 1u);
        if (old == G32 - 1) {
            atomicExch(ctr + kCtrNorm, 0u);
            atomicExch(ctr + kCtrAttn, 0u);
            for (int k = 0; k < kSub; ++k) atomicExch(ctr + kCtrGemv + 32 * k, 0u);
            atomicExch(ctr + kCtrExit, 0u);
            __threadfence();
        }
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
        if (e == cudaSuccess && prop.major == 10 && prop.cooperativeLaunch &&
            prop.sharedMemPerBlockOptin >= tiles::kSmemBytes) {
            e = cudaFuncSetAttribute(rvq_persist_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)tiles::kSmemBytes);
            int per_sm = 0;
            if (e == cudaSuccess)
                e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, rvq_persist_kernel, kThreads,
                                                                  tiles::kSmemBytes);
            d.sms = prop.multiProcessorCount;
            d.ok = e == cudaSuccess && per_sm >= 1 && d.sms >= 2 * kRanks && d.sms <= tiles::kMaxCtas;
        }
        if (e != cudaSuccess) last_cuda_error_slot() = (int)e;
    }
    if (!d.ok) return RVQ_ERR_UNAVAILABLE;
    *out = &d;
    return RVQ_OK;
}

int64_t tiles_of(int64_t cols) { return (cols + kTileCols - 1) / kTileCols; }

int64_t align16(int64_t v) { return (v + 15) & ~15ll; }

int check_model(const rvq_persist_model& m, int sms) {
    if (m.n_layers < 1 || m.hidden < 8 || m.hidden % 8 || m.intermediate < 8 || m.intermediate % 8 || m.vocab < 1 ||
        m.max_len < 1 || m.n_kv < 1 || m.n_heads < m.n_kv || m.n_heads % m.n_kv)
        return RVQ_ERR_INVALID;
    if (m.head_dim != kHD || m.n_heads / m.n_kv > kMaxRep || m.hidden > kRanks * kNormMaxSlice ||
        m.n_kv > sms - kRanks || m.reserved != 0)
        return RVQ_ERR_UNSUPPORTED;
    if ((int64_t)(m.n_heads / m.n_kv) * m.max_len > kMaxScores) return RVQ_ERR_TOO_LARGE;
    if (!m.embed || !m.final_norm || !m.cos || !m.sin || !m.token || !m.pos || !m.h || !m.x_final || !m.attn_out ||
        !m.q_part || !m.k_part || !m.v_part || !m.o_part || !m.gate_part || !m.up_part || !m.down_part || !m.sync)
        return RVQ_ERR_INVALID;
    if ((uintptr_t)m.sync & 15) return RVQ_ERR_INVALID;
    return RVQ_OK;
}

// Builds the plan for `sms` CTAs into `out` (when not null, `cap` bytes);
// *bytes = its size.
int build_plan(const rvq_persist_model* m, const rvq_persist_layer* layers, int sms, char* out, int64_t cap,
               int64_t* bytes) {
    if (m == nullptr || layers == nullptr) return RVQ_ERR_INVALID;
    int rc = check_model(*m, sms);
    if (rc != RVQ_OK) return rc;
    const int L = m->n_layers;
    const int64_t H = m->hidden, I = m->intermediate, QD = (int64_t)m->n_heads * kHD, KD = (int64_t)m->n_kv * kHD;
    const int32_t ht = (int32_t)tiles_of(H), it = (int32_t)tiles_of(I);
    std::unique_ptr<tiles::TParams> tp(new tiles::TParams);
    std::vector<PLayer> pl((size_t)L);
    std::vector<int32_t> cta_first;
    std::vector<uint32_t> ujt;
    std::vector<int32_t> ur0, ur1;
    const rvq_vec hvec = {m->h, H, 1, RVQ_BF16};                 // stands for the normed operand
    const rvq_vec avec = {m->attn_out, QD, 1, RVQ_BF16};
    const rvq_vec upv = {m->up_part, I, ht, RVQ_F32};
    const rvq_vec gatev = {m->gate_part, I, ht, RVQ_F32};
    const rvq_vec none = {nullptr, 0, 0, 0};
    for (int l = 0; l < L; ++l) {
        const rvq_persist_layer& Y = layers[l];
        if (!Y.input_norm || !Y.post_norm || !Y.q_norm || !Y.k_norm || !Y.k_cache || !Y.v_cache)
            return RVQ_ERR_INVALID;
        rvq_gemv_tile_job jobs[kPhases][3];
        const int nj[kPhases] = {3, 1, 2, 1};
        memset(jobs, 0, sizeof(jobs));
        auto job = [&](rvq_gemv_tile_job& j, int p, rvq_vec x, rvq_vec g, float* part, int64_t rows, int64_t cols) {
            j.weight = Y.proj[p];
            j.x = x;
            j.gate = g;
            j.partials = part;
            j.rows = rows;
            j.cols = cols;
        };
        job(jobs[0][0], 0, hvec, none, m->q_part, QD, H);
        job(jobs[0][1], 1, hvec, none, m->k_part, KD, H);
        job(jobs[0][2], 2, hvec, none, m->v_part, KD, H);
        job(jobs[1][0], 3, avec, none, m->o_part, H, QD);
        job(jobs[2][0], 4, hvec, none, m->gate_part, I, H);
        job(jobs[2][1], 5, hvec, none, m->up_part, I, H);
        job(jobs[3][0], 6, upv, gatev, m->down_part, H, I);
        PLayer& P = pl[(size_t)l];
        memset(&P, 0, sizeof(P));
        P.ln1 = Y.input_norm;
        P.ln2 = Y.post_norm;
        P.q_norm = Y.q_norm;
        P.k_norm = Y.k_norm;
        P.k_cache = Y.k_cache;
        P.v_cache = Y.v_cache;
        for (int p = 0; p < kPhases; ++p) {
            for (int j = 0; j < nj[p]; ++j) {
                rc = tiles::check_job(jobs[p][j]);
                if (rc != RVQ_OK) return rc;
                P.ph[p].jobs[j] = tiles::make_tjob(jobs[p][j]);
            }
            P.ph[p].n_jobs = nj[p];
            memset(tp.get(), 0, sizeof(tiles::TParams));
            rc = tiles::plan(jobs[p], nj[p], sms, *tp);
            if (rc != RVQ_OK) return rc;
            P.ph[p].cta_first = (int32_t)cta_first.size();
            const int32_t base = (int32_t)ujt.size();
            for (int c = 0; c <= sms; ++c)
                cta_first.push_back(base + tp->cta_first[c < tp->n_ctas ? c : tp->n_ctas]);
            for (int u = 0; u < tp->n_units; ++u) {
                ujt.push_back(tp->unit_jt[u]);
                ur0.push_back(tp->unit_r0[u]);
                ur1.push_back(tp->unit_r1[u]);
            }
        }
    }
    PHead head;
    memset(&head, 0, sizeof(head));
    head.m = *m;
    head.n_ctas = sms;
    head.hid_tiles = ht;
    head.o_tiles = (int32_t)tiles_of(QD);
    head.inter_tiles = it;
    int64_t off = align16(sizeof(PHead));
    head.layers_off = off;
    off = align16(off + (int64_t)sizeof(PLayer) * L);
    head.cta_first_off = off;
    off = align16(off + 4 * (int64_t)cta_first.size());
    head.unit_jt_off = off;
    off = align16(off + 4 * (int64_t)ujt.size());
    head.unit_r0_off = off;
    off = align16(off + 4 * (int64_t)ur0.size());
    head.unit_r1_off = off;
    off = align16(off + 4 * (int64_t)ur1.size());
    *bytes = off;
    if (out == nullptr) return RVQ_OK;
    if (cap < off) return RVQ_ERR_INVALID;
    memset(out, 0, (size_t)off);
    memcpy(out, &head, sizeof(head));
    memcpy(out + head.layers_off, pl.data(), sizeof(PLayer) * (size_t)L);
    memcpy(out + head.cta_first_off, cta_first.data(), 4 * cta_first.size());
    memcpy(out + head.unit_jt_off, ujt.data(), 4 * ujt.size());
    memcpy(out + head.unit_r0_off, ur0.data(), 4 * ur0.size());
    memcpy(out + head.unit_r1_off, ur1.data(), 4 * ur1.size());
    return RVQ_OK;
}

}  // namespace persist
}  // namespace rvq

using namespace rvq;
using namespace rvq::persist;

extern "C" {

int64_t rvq_persist_plan_bytes(const rvq_persist_model* m, const rvq_persist_layer* layers) {
    DevInfo* d = nullptr;
    if (dev_info(&d) != RVQ_OK) return 0;
    int64_t bytes = 0;
    return build_plan(m, layers, d->sms, nullptr, 0, &bytes) == RVQ_OK ? bytes : 0;
}

int rvq_persist_plan(const rvq_persist_model* m, const rvq_persist_layer* layers, void* plan, int64_t bytes) {
    if (plan == nullptr || bytes < 1) return RVQ_ERR_INVALID;
    DevInfo* d = nullptr;
    const int rc = dev_info(&d);
    if (rc != RVQ_OK) return rc;
    int64_t need = 0;
    return build_plan(m, layers, d->sms, reinterpret_cast<char*>(plan), bytes, &need);
}

int64_t rvq_persist_plan_for(const rvq_persist_model* m, const rvq_persist_layer* layers, int32_t n_ctas, void* plan,
                             int64_t bytes) {
    if (n_ctas < 2 * kRanks || n_ctas > tiles::kMaxCtas) return -RVQ_ERR_INVALID;
    int64_t need = 0;
    int rc = build_plan(m, layers, n_ctas, nullptr, 0, &need);
    if (rc != RVQ_OK) return -rc;
    if (plan == nullptr) return need;
    rc = build_plan(m, layers, n_ctas, reinterpret_cast<char*>(plan), bytes, &need);
    return rc == RVQ_OK ? need : -rc;
}

int rvq_persist_step(const void* plan_dev, void* stream) {
    if (plan_dev == nullptr || ((uintptr_t)plan_dev & 15)) return RVQ_ERR_INVALID;
    DevInfo* d = nullptr;
    const int rc = dev_info(&d);
    if (rc != RVQ_OK) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)d->sms);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = tiles::kSmemBytes;
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, rvq_persist_kernel, reinterpret_cast<const PHead*>(plan_dev));
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) {
        last_cuda_error_slot() = (int)e;
        return RVQ_ERR_CUDA;
    }
    return RVQ_OK;
}

int rvq_persist_take_error(void) {
    int v = 0, w = 0;
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&v, g_persist_error, sizeof(int));
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&w, tiles::g_wait_timeout, sizeof(int));
    const int zero = 0;
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_persist_error, &zero, sizeof(int));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(tiles::g_wait_timeout, &zero, sizeof(int));
    if (e != cudaSuccess) {
        last_cuda_error_slot() = (int)e;
        return -RVQ_ERR_CUDA;
    }
    return (v || w) ? 1 : 0;
}

}  // extern "C"
