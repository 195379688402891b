// Batch-1 decode-step operations of a Qwen3 decoder layer (sm_100a):
// residual add + RMSNorm, GQA decode attention over a static KV cache, and
// SiLU-gated product.  They replace the small PyTorch kernels that the HF
// modules launch per layer (modeling_qwen3: Qwen3RMSNorm, eager_attention_
// forward, Qwen3MLP), rounding to bf16 where those modules round.
//
// Operands that are projection outputs arrive either as bf16 vectors or as
// fp32 per-tile partial sums ([ntiles][n], summed in tile order then rounded
// to bf16), so the GEMV that produced them needs no reduction pass of its own.

#include <cooperative_groups.h>
#include <string.h>
#include <type_traits>

#include "rvq_common.cuh"
#include "rvq_stepops.cuh"

namespace cg = cooperative_groups;

namespace rvq {
namespace {

using namespace stepops;


__device__ int g_tp_timeout;                 // sticky: a landing-buffer wait gave up

// Operand read through L2 (a landing buffer that peers write over NVLink:
// no stale L1 lines).  fp32 rows summed in row order, then rounded to bf16.
__device__ __forceinline__ float vec_value_l2(const rvq_vec& v, int64_t i) {
    const float* p = reinterpret_cast<const float*>(v.ptr) + i;
    float s = __ldcg(p);
    for (int t = 1; t < v.ntiles; ++t) s += __ldcg(p + (int64_t)t * v.n);
    return bf16r(s);
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Wait until *arrivals has reached `target` (wrap-around safe).  Gives up
// after about one second (or 2^24 polls), sets the sticky timeout flag and
// returns false; the caller then goes on with whatever the buffer holds.
__device__ __forceinline__ bool wait_arrivals(const uint32_t* arrivals, uint32_t target) {
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 0; i < (1u << 24); ++i) {
        if ((int32_t)(ld_acquire_sys(arrivals) - target) >= 0) return true;
        if (i > 64) __nanosleep(128);
        if ((i & 63) == 0 && globaltimer_ns() - t0 > 1000000000ull) break;
    }
    atomicExch(&g_tp_timeout, 1);
    return false;
}

// ---------------------------------------------------------------------------
// Residual add + RMSNorm.  8 CTAs in one cluster each own a slice of the
// hidden vector; the sum of squares is combined through distributed shared
// memory in rank order (deterministic).
// ---------------------------------------------------------------------------
constexpr int kNormCtas = 8;
constexpr int kNormThreads = 1024;
constexpr int kNormMaxSlice = 2048;     // hidden <= 16384

__global__ void __cluster_dims__(kNormCtas, 1, 1) __launch_bounds__(kNormThreads)
step_norm_kernel(rvq_norm_args a) {
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    __shared__ float hbuf[kNormMaxSlice];
    __shared__ float wbuf[kNormMaxSlice];
    __shared__ float warp_ss[kNormThreads / 32];
    __shared__ float cta_ss;
    const int64_t H = a.hidden;
    const int64_t slice = (H + kNormCtas - 1) / kNormCtas;
    const int64_t lo = rank * slice;
    const int64_t hi = lo + slice < H ? lo + slice : H;
    const int tid = threadIdx.x;

    pdl_launch_dependents();
    for (int64_t i = lo + tid; i < hi; i += kNormThreads) wbuf[i - lo] = bf16_at(a.weight, i);
    pdl_wait();
    const bool landing = a.arrivals != nullptr && a.token == nullptr && a.add.ptr != nullptr;
    uint32_t target = 0;
    if (landing) {                              // every rank's push has arrived
        target = __ldcg(a.consumed) + a.arrivals_per_use;
        if (tid == 0) wait_arrivals(a.arrivals, target);
        __syncthreads();
    }
    float ss = 0.f;
    if (a.token != nullptr) {
        const int64_t tok = *a.token;
        const int64_t row = (tok >= 0 && tok < a.vocab ? tok : 0) * H;
        for (int64_t i = lo + tid; i < hi; i += kNormThreads) {
            const float hv = bf16_at(a.embed, row + i);
            hbuf[i - lo] = hv;
            ss = fmaf(hv, hv, ss);
        }
    } else {
        for (int64_t i = lo + tid; i < hi; i += kNormThreads) {
            float hv = bf16_at(a.h, i);
            if (a.add.ptr != nullptr) hv = bf16r(hv + (landing ? vec_value_l2(a.add, i) : vec_value_deep(a.add, i)));
            hbuf[i - lo] = hv;
            ss = fmaf(hv, hv, ss);
        }
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) warp_ss[tid >> 5] = ss;
    __syncthreads();
    if (tid == 0) {
        float t = 0.f;
        for (int w = 0; w < kNormThreads / 32; ++w) t += warp_ss[w];
        cta_ss = t;
    }
    cluster.sync();
    float total = 0.f;
    for (int r = 0; r < kNormCtas; ++r) total += *cluster.map_shared_rank(&cta_ss, r);
    const float inv = rsqrtf(total / (float)H + a.eps);
    for (int64_t i = lo + tid; i < hi; i += kNormThreads) {
        const float hv = hbuf[i - lo];
        put_bf16(a.h, i, hv);
        put_bf16(a.x, i, wbuf[i - lo] * bf16r(hv * inv));
    }
    cluster.sync();       // no CTA leaves while another may still read its cta_ss
    if (landing && rank == 0 && tid == 0) *a.consumed = target;
}

// ---------------------------------------------------------------------------
// Decode attention.  A cluster of kAttnCtas CTAs per kv head splits the keys
// 0..pos into contiguous ranges; every CTA normalises and rotates q (the kv
// head's `rep` query heads) and the new k itself.  Within a CTA each warp
// takes keys w, w + 8, ...: its lanes hold head_dim / 32 consecutive
// elements, so a key's K and V rows are read with one coalesced load per warp
// and a score is a warp sum.  Softmax max and sum, and the P V partial
// products, are combined through distributed shared memory in rank order, so
// the result does not depend on scheduling.
// ---------------------------------------------------------------------------
constexpr int kAttnCtas = 8;
constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kMaxRep = 16;
constexpr int kKeyChunk = 4;          // keys whose rows a warp loads before using them

// Shared-memory floats of one CTA (host sizes the dynamic allocation with it).
__host__ __device__ constexpr int attn_smem_floats(int hd, int rep, int keys_per_cta) {
    return (rep + 2) * hd                  // raw operands: q heads, k, v
         + rep * hd                        // q after norm + rope
         + 2 * hd                          // new k (rotated), new v
         + kAttnWarps * rep * hd           // P V partial of each warp
         + rep * hd                        // P V partial of this CTA
         + rep * keys_per_cta              // scores, then probabilities
         + 2 * kMaxRep                     // local max, local sum
         + 4 * hd;                         // q_norm, k_norm, cos and sin rows of pos
}

template <int HD>
__global__ void __cluster_dims__(kAttnCtas, 1, 1) __launch_bounds__(kAttnThreads, 1)
step_attn_kernel(rvq_attn_args a) {
    constexpr int E = HD / 32;                 // elements per lane in the key loops
    constexpr int RG = 32 / E < kMaxRep ? 32 / E : kMaxRep;   // heads per P V register group
    extern __shared__ __align__(16) float smem[];
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int kv = blockIdx.y;
    const int rep = a.n_heads / a.n_kv;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    pdl_launch_dependents();
    const int64_t pos = *a.pos;
    if (pos < 0 || pos >= a.max_len) {               // same decision in every CTA of the cluster
        pdl_wait();
        for (int i = rank * kAttnThreads + tid; i < rep * HD; i += kAttnCtas * kAttnThreads)
            put_bf16(a.out, (int64_t)kv * rep * HD + i, 0.f);
        return;
    }
    const int L = (int)pos + 1;
    const int kpc_max = (a.max_len + kAttnCtas - 1) / kAttnCtas;
    const int kpc = (L + kAttnCtas - 1) / kAttnCtas;
    const int j0 = rank * kpc;
    const int j1 = min(L, j0 + kpc);
    float* raw = smem;
    float* qs = raw + (rep + 2) * HD;
    float* knew = qs + rep * HD;
    float* vnew = knew + HD;
    float* pw = vnew + HD;
    float* pout = pw + kAttnWarps * rep * HD;
    float* sc = pout + rep * HD;
    float* mloc = sc + rep * kpc_max;
    float* sloc = mloc + kMaxRep;
    float* wsm = sloc + kMaxRep;                // [4][HD]: q_norm, k_norm, cos[pos], sin[pos]
    __shared__ float red[kMaxRep][kAttnWarps];
    __shared__ float gmax[kMaxRep], gsum[kMaxRep];

    // 1. everything that does not depend on q, k, v is requested first: this warp's
    //    first kKeyChunk K and V rows, the norm weights and this position's cos / sin;
    //    then the operands (6 per thread in flight before their stores)
    const int d0 = lane * E;
    const __nv_bfloat16* kc = reinterpret_cast<const __nv_bfloat16*>(a.k_cache) + (int64_t)kv * a.max_len * HD;
    const __nv_bfloat16* vc = reinterpret_cast<const __nv_bfloat16*>(a.v_cache) + (int64_t)kv * a.max_len * HD;
    float kd0[kKeyChunk][E], vd0[kKeyChunk][E];
#pragma unroll
    for (int c = 0; c < kKeyChunk; ++c) {
        const int j = j0 + warp + c * kAttnWarps;
        if (j < j1 && j != pos) {
            load_row_slice<E>(kc + (int64_t)j * HD + d0, kd0[c]);
            load_row_slice<E>(vc + (int64_t)j * HD + d0, vd0[c]);
        }
    }
    for (int i = tid; i < 4 * HD; i += kAttnThreads) {
        const int which = i / HD, d = i - which * HD;
        const void* src = which == 0 ? a.q_norm : which == 1 ? a.k_norm : which == 2 ? a.cos : a.sin;
        wsm[i] = bf16_at(src, (which >= 2 ? pos * HD : 0) + d);
    }
    pdl_wait();                                      // q, k, v come from the previous kernel
    // the operands' tile sums are split over the cluster (CTA `rank` sums
    // elements [rank * och, (rank + 1) * och), all tile loads of an element in
    // flight), then every CTA gathers the other ranges over DSMEM
    const int nel = (rep + 2) * HD;
    const int och = (nel + kAttnCtas - 1) / kAttnCtas;
    for (int i = rank * och + tid; i < min(nel, (rank + 1) * och); i += kAttnThreads) {
        const int r = i / HD, d = i - r * HD;
        raw[i] = r < rep ? vec_value_deep(a.q, ((int64_t)kv * rep + r) * HD + d)
               : r == rep ? vec_value_deep(a.k, (int64_t)kv * HD + d)
                          : vec_value_deep(a.v, (int64_t)kv * HD + d);
    }
    cluster.sync();
    for (int base = 0; base < nel; base += 6 * kAttnThreads) {   // 6 DSMEM loads in flight, then the stores
        float val[6];
#pragma unroll
        for (int m = 0; m < 6; ++m) {
            const int i = min(base + tid + m * kAttnThreads, nel - 1);
            val[m] = cluster.map_shared_rank(raw, i / och)[i];
        }
#pragma unroll
        for (int m = 0; m < 6; ++m) {
            const int i = base + tid + m * kAttnThreads;
            if (i < nel && i / och != rank) raw[i] = val[m];
        }
    }
    __syncthreads();

    // 2. norm + rope (warp per head); the CTA whose range holds pos appends to the cache
    const bool owner = j0 <= pos && pos < j1;
    const int64_t cache_row = ((int64_t)kv * a.max_len + pos) * HD;
    for (int hh = warp; hh <= rep; hh += kAttnWarps) {
        float o[HD / 32];
        const bool is_k = hh == rep;
        norm_rope_head<HD>(raw + hh * HD, wsm + (is_k ? HD : 0), a.eps, wsm + 2 * HD, wsm + 3 * HD, o);
#pragma unroll
        for (int j = 0; j < HD / 32; ++j) {
            const int d = lane + 32 * j;
            if (!is_k) {
                qs[hh * HD + d] = o[j];
            } else {
                knew[d] = o[j];
                vnew[d] = raw[(rep + 1) * HD + d];
                if (owner) {
                    put_bf16(a.k_cache, cache_row + d, o[j]);
                    put_bf16(a.v_cache, cache_row + d, vnew[d]);
                }
            }
        }
    }
    __syncthreads();

    // 3. scores: warp per key, lanes over head_dim; rows of kKeyChunk keys loaded
    //    first; the rep heads' lane partials are reduced 8 heads at a time by one
    //    reduce-scatter (lane quad q ends up with head 8 g + q)
    constexpr int kGroupsMax = kMaxRep / 8;
    const int hq = (lane >> 2) & 7;                   // this lane quad's head within a group of 8
    float mx[kGroupsMax];
#pragma unroll
    for (int g = 0; g < kGroupsMax; ++g) mx[g] = -INFINITY;
    for (int jb = j0 + warp; jb < j1; jb += kAttnWarps * kKeyChunk) {
        float kd[kKeyChunk][E];
#pragma unroll
        for (int c = 0; c < kKeyChunk; ++c) {
            const int j = jb + c * kAttnWarps;
            if (j == pos || j >= j1) {
#pragma unroll
                for (int e = 0; e < E; ++e) kd[c][e] = knew[d0 + e];
            } else if (jb == j0 + warp) {
#pragma unroll
                for (int e = 0; e < E; ++e) kd[c][e] = kd0[c][e];
            } else {
                load_row_slice<E>(kc + (int64_t)j * HD + d0, kd[c]);
            }
        }
#pragma unroll
        for (int c = 0; c < kKeyChunk; ++c) {
            const int j = jb + c * kAttnWarps;
            if (j >= j1) break;                               // warp-uniform
#pragma unroll
            for (int g = 0; g < kGroupsMax; ++g) {
                if (8 * g < rep) {
                    float pr[8];
#pragma unroll
                    for (int r = 0; r < 8; ++r) {
                        float t = 0.f;
                        if (8 * g + r < rep) {
#pragma unroll
                            for (int e = 0; e < E; ++e) t = fmaf(qs[(8 * g + r) * HD + d0 + e], kd[c][e], t);
                        }
                        pr[r] = t;
                    }
                    const float t = reduce8(pr);
                    const int r = 8 * g + hq;
                    if (r < rep) {
                        const float sv = bf16r(bf16r(bf16r(t) * a.scaling) + a.valid_bias);
                        if ((lane & 3) == 0) sc[r * kpc_max + (j - j0)] = sv;
                        mx[g] = fmaxf(mx[g], sv);
                    }
                }
            }
        }
    }
    if ((lane & 3) == 0) {
#pragma unroll
        for (int g = 0; g < kGroupsMax; ++g)
            if (8 * g + hq < rep) red[8 * g + hq][warp] = mx[g];
    }
    __syncthreads();
    if (tid < rep) {
        float m = red[tid][0];
        for (int w = 1; w < kAttnWarps; ++w) m = fmaxf(m, red[tid][w]);
        mloc[tid] = m;
    }
    __syncthreads();

    // 4. softmax with one cluster exchange: each CTA sums exp(s - its own max);
    //    the global sum rescales those by exp(local max - global max), in rank
    //    order; probabilities are exp(s - global max) / sum, rounded to bf16
    float sm[kMaxRep];
#pragma unroll
    for (int r = 0; r < kMaxRep; ++r) sm[r] = 0.f;
    for (int j = j0 + tid; j < j1; j += kAttnThreads) {
#pragma unroll
        for (int r = 0; r < kMaxRep; ++r)
            if (r < rep) sm[r] += expf(sc[r * kpc_max + (j - j0)] - mloc[r]);
    }
#pragma unroll
    for (int g = 0; g < kGroupsMax; ++g) {
        if (8 * g < rep) {
            float pr[8];
#pragma unroll
            for (int r = 0; r < 8; ++r) pr[r] = sm[8 * g + r];
            const float t = reduce8(pr);
            if ((lane & 3) == 0 && 8 * g + hq < rep) red[8 * g + hq][warp] = t;
        }
    }
    __syncthreads();
    if (tid < rep) {
        float t = 0.f;
        for (int w = 0; w < kAttnWarps; ++w) t += red[tid][w];
        sloc[tid] = t;
    }
    cluster.sync();
    if (tid < rep) {
        float mcs[kAttnCtas], scs[kAttnCtas];                 // every CTA's max and sum, one round trip
#pragma unroll
        for (int c = 0; c < kAttnCtas; ++c) {
            mcs[c] = cluster.map_shared_rank(mloc, c)[tid];
            scs[c] = cluster.map_shared_rank(sloc, c)[tid];
        }
        float m = -INFINITY;
#pragma unroll
        for (int c = 0; c < kAttnCtas; ++c) m = fmaxf(m, mcs[c]);
        float t = 0.f;
#pragma unroll
        for (int c = 0; c < kAttnCtas; ++c)
            if (scs[c] > 0.f) t += scs[c] * expf(mcs[c] - m);
        gmax[tid] = m;
        gsum[tid] = t;
    }
    __syncthreads();
    for (int j = j0 + tid; j < j1; j += kAttnThreads) {
#pragma unroll
        for (int r = 0; r < kMaxRep; ++r)
            if (r < rep) sc[r * kpc_max + (j - j0)] = bf16r(expf(sc[r * kpc_max + (j - j0)] - gmax[r]) / gsum[r]);
    }
    __syncthreads();

    // 5. P V: warp per key again; RG heads' accumulators per register pass
    for (int rg = 0; rg < rep; rg += RG) {
        float acc[RG][E];
#pragma unroll
        for (int r = 0; r < RG; ++r)
#pragma unroll
            for (int e = 0; e < E; ++e) acc[r][e] = 0.f;
        for (int jb = j0 + warp; jb < j1; jb += kAttnWarps * kKeyChunk) {
            float vd[kKeyChunk][E];
#pragma unroll
            for (int c = 0; c < kKeyChunk; ++c) {
                const int j = jb + c * kAttnWarps;
                if (j == pos || j >= j1) {
#pragma unroll
                    for (int e = 0; e < E; ++e) vd[c][e] = vnew[d0 + e];
                } else if (jb == j0 + warp) {
#pragma unroll
                    for (int e = 0; e < E; ++e) vd[c][e] = vd0[c][e];
                } else {
                    load_row_slice<E>(vc + (int64_t)j * HD + d0, vd[c]);
                }
            }
#pragma unroll
            for (int c = 0; c < kKeyChunk; ++c) {
                const int j = jb + c * kAttnWarps;
                if (j >= j1) break;
#pragma unroll
                for (int r = 0; r < RG; ++r) {
                    if (rg + r < rep) {
                        const float pr = sc[(rg + r) * kpc_max + (j - j0)];
#pragma unroll
                        for (int e = 0; e < E; ++e) acc[r][e] = fmaf(pr, vd[c][e], acc[r][e]);
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < RG; ++r)
            if (rg + r < rep)
#pragma unroll
                for (int e = 0; e < E; ++e) pw[(warp * rep + rg + r) * HD + d0 + e] = acc[r][e];
    }
    __syncthreads();
    for (int i = tid; i < rep * HD; i += kAttnThreads) {
        float t = pw[i];
        for (int w = 1; w < kAttnWarps; ++w) t += pw[w * rep * HD + i];
        pout[i] = t;
    }
    cluster.sync();

    // 6. sum the CTAs' partials in rank order; CTA c writes its slice of the output
    const int total = rep * HD;
    const int chunk = (total + kAttnCtas - 1) / kAttnCtas;
    for (int i = rank * chunk + tid; i < min(total, (rank + 1) * chunk); i += kAttnThreads) {
        float t = 0.f;
        for (int c = 0; c < kAttnCtas; ++c) t += cluster.map_shared_rank(pout, c)[i];
        put_bf16(a.out, (int64_t)kv * rep * HD + i, t);
    }
    cluster.sync();       // keep this CTA's shared memory alive until every reader is done
}

__global__ void step_silu_mul_kernel(rvq_vec g, rvq_vec u, void* out) {
    pdl_launch_dependents();
    pdl_wait();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= g.n) return;
    const float gv = vec_value(g, i);
    const float act = bf16r(gv / (1.0f + expf(-gv)));
    put_bf16(out, i, act * vec_value(u, i));
}

bool vec_ok(const rvq_vec& v, int64_t n) {
    if (v.ptr == nullptr || v.n != n || v.ntiles < 1) return false;
    if (v.kind == RVQ_F32) return true;
    return (v.kind == RVQ_BF16 || v.kind == RVQ_F16) && v.ntiles == 1;
}

int launch_status() {
    const cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) {
        last_cuda_error_slot() = (int)err;
        return RVQ_ERR_CUDA;
    }
    return RVQ_OK;
}

template <int HD>
int launch_attn(const rvq_attn_args& a, cudaStream_t s) {
    const int rep = a.n_heads / a.n_kv;
    const int kpc_max = (a.max_len + kAttnCtas - 1) / kAttnCtas;
    const size_t smem = (size_t)attn_smem_floats(HD, rep, kpc_max) * sizeof(float);
    if (smem > 200 * 1024) return RVQ_ERR_UNSUPPORTED;
    if (cudaFuncSetAttribute(step_attn_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
        return launch_status();
    const cudaError_t e = launch_pdl(step_attn_kernel<HD>, dim3(kAttnCtas, a.n_kv), dim3(kAttnThreads), smem, s, a);
    if (e != cudaSuccess) last_cuda_error_slot() = (int)e;
    return e == cudaSuccess ? launch_status() : RVQ_ERR_CUDA;
}

}  // namespace
}  // namespace rvq

using namespace rvq;

extern "C" int rvq_step_norm(const rvq_norm_args* a, void* stream) {
    if (a == nullptr || a->h == nullptr || a->weight == nullptr || a->x == nullptr) return RVQ_ERR_INVALID;
    if (a->hidden < 1 || a->hidden > (int64_t)kNormCtas * kNormMaxSlice) return RVQ_ERR_UNSUPPORTED;
    if (a->token != nullptr && (a->embed == nullptr || a->vocab < 1)) return RVQ_ERR_INVALID;
    if (a->token == nullptr && a->add.ptr != nullptr && !vec_ok(a->add, a->hidden)) return RVQ_ERR_INVALID;
    if (a->arrivals != nullptr && (a->consumed == nullptr || a->add.kind != RVQ_F32)) return RVQ_ERR_INVALID;
    const cudaError_t e = launch_pdl(step_norm_kernel, dim3(kNormCtas), dim3(kNormThreads), 0,
                                     (cudaStream_t)stream, *a);
    if (e != cudaSuccess) last_cuda_error_slot() = (int)e;
    return e == cudaSuccess ? launch_status() : RVQ_ERR_CUDA;
}

extern "C" int rvq_step_attention(const rvq_attn_args* a, void* stream) {
    if (a == nullptr || a->q_norm == nullptr || a->k_norm == nullptr || a->cos == nullptr ||
        a->sin == nullptr || a->pos == nullptr || a->k_cache == nullptr || a->v_cache == nullptr ||
        a->out == nullptr)
        return RVQ_ERR_INVALID;
    if (a->n_kv < 1 || a->n_heads < a->n_kv || a->n_heads % a->n_kv != 0 || a->max_len < 1)
        return RVQ_ERR_INVALID;
    if (a->n_heads / a->n_kv > kMaxRep) return RVQ_ERR_UNSUPPORTED;
    const int64_t hd = a->head_dim;
    if (!vec_ok(a->q, (int64_t)a->n_heads * hd) || !vec_ok(a->k, (int64_t)a->n_kv * hd) ||
        !vec_ok(a->v, (int64_t)a->n_kv * hd))
        return RVQ_ERR_INVALID;
    cudaStream_t s = (cudaStream_t)stream;
    switch (a->head_dim) {
        case 64: return launch_attn<64>(*a, s);
        case 128: return launch_attn<128>(*a, s);
        case 256: return launch_attn<256>(*a, s);
        default: return RVQ_ERR_UNSUPPORTED;
    }
}

extern "C" int rvq_step_silu_mul(const rvq_vec* gate, const rvq_vec* up, void* out, void* stream) {
    if (gate == nullptr || up == nullptr || out == nullptr) return RVQ_ERR_INVALID;
    if (!vec_ok(*gate, gate->n) || !vec_ok(*up, gate->n) || gate->n < 1) return RVQ_ERR_INVALID;
    const int threads = 256;
    const unsigned blocks = (unsigned)((gate->n + threads - 1) / threads);
    const cudaError_t e = launch_pdl(step_silu_mul_kernel, dim3(blocks), dim3(threads), 0, (cudaStream_t)stream,
                                     *gate, *up, out);
    if (e != cudaSuccess) last_cuda_error_slot() = (int)e;
    return e == cudaSuccess ? launch_status() : RVQ_ERR_CUDA;
}

// ---------------------------------------------------------------------------
// Tensor-parallel push (see include/rvq_b200.h)
// ---------------------------------------------------------------------------
namespace rvq {
namespace {

constexpr int kPushThreads = 128;
constexpr int kPushPerThread = 1;     // one element per thread: its tile loads all in flight

struct TpPush {
    rvq_vec src;
    float* dst[RVQ_MAX_TP];
    uint32_t* arrivals[RVQ_MAX_TP];
    int64_t n;
    int32_t rank, tp;
};

// A read-only load issued where it is written (the chunk's loads leave before any add).
__device__ __forceinline__ float ldg_now(const float* p) {
    float v;
    asm volatile("ld.global.nc.f32 %0, [%1];\n" : "=f"(v) : "l"(p));
    return v;
}

// fp32 value of the projection output (tiles summed in order, not rounded),
// 32 tile loads in flight at a time
__device__ __forceinline__ float vec_value_f32(const rvq_vec& v, int64_t i) {
    if (v.kind != RVQ_F32) return load_as_f32(v.ptr, i, v.kind);
    const float* p = reinterpret_cast<const float*>(v.ptr) + i;
    const int64_t n = v.n;
    const int nt = v.ntiles;
    float s = __ldg(p);
    int t = 1;
    for (; t + 32 <= nt; t += 32) {
        float c[32];
#pragma unroll
        for (int k = 0; k < 32; ++k) c[k] = ldg_now(p + (int64_t)(t + k) * n);
#pragma unroll
        for (int k = 0; k < 32; k += 8)             // every load issued before the first add
            asm volatile("" : "+f"(c[k]), "+f"(c[k + 1]), "+f"(c[k + 2]), "+f"(c[k + 3]), "+f"(c[k + 4]),
                         "+f"(c[k + 5]), "+f"(c[k + 6]), "+f"(c[k + 7]));
#pragma unroll
        for (int k = 0; k < 32; ++k) s += c[k];
    }
    if (t < nt) {                                   // the rest: clamped loads, adds in order
        float c[31];
#pragma unroll
        for (int k = 0; k < 31; ++k) c[k] = ldg_now(p + (int64_t)min(t + k, nt - 1) * n);
#pragma unroll
        for (int k = 0; k < 24; k += 8)
            asm volatile("" : "+f"(c[k]), "+f"(c[k + 1]), "+f"(c[k + 2]), "+f"(c[k + 3]), "+f"(c[k + 4]),
                         "+f"(c[k + 5]), "+f"(c[k + 6]), "+f"(c[k + 7]));
        asm volatile("" : "+f"(c[24]), "+f"(c[25]), "+f"(c[26]), "+f"(c[27]), "+f"(c[28]), "+f"(c[29]), "+f"(c[30]));
#pragma unroll
        for (int k = 0; k < 31; ++k)
            if (t + k < nt) s += c[k];
    }
    return s;
}

__global__ void __launch_bounds__(kPushThreads) tp_push_kernel(TpPush a) {
    pdl_launch_dependents();
    pdl_wait();
    const int64_t base = (int64_t)blockIdx.x * kPushThreads * kPushPerThread;
    float v[kPushPerThread];
#pragma unroll
    for (int k = 0; k < kPushPerThread; ++k) {
        const int64_t i = base + k * kPushThreads + threadIdx.x;
        v[k] = i < a.n ? vec_value_f32(a.src, i) : 0.f;
    }
    for (int r = 0; r < a.tp; ++r) {
        float* d = a.dst[r] + (int64_t)a.rank * a.n;
#pragma unroll
        for (int k = 0; k < kPushPerThread; ++k) {
            const int64_t i = base + k * kPushThreads + threadIdx.x;
            if (i < a.n) d[i] = v[k];
        }
    }
    __threadfence_system();                 // this thread's peer stores before the arrivals
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int r = 0; r < a.tp; ++r) {
            asm volatile("red.release.sys.global.add.u32 [%0], 1;\n" ::"l"(a.arrivals[r]) : "memory");
        }
    }
}

}  // namespace
}  // namespace rvq

extern "C" uint32_t rvq_tp_push_ctas(int64_t n) {
    return n < 1 ? 0u : (uint32_t)((n + kPushThreads * kPushPerThread - 1) / (kPushThreads * kPushPerThread));
}

extern "C" int rvq_tp_push(const rvq_tp_push_args* a, void* stream) {
    if (a == nullptr || a->tp < 1 || a->tp > RVQ_MAX_TP || a->rank < 0 || a->rank >= a->tp || a->n < 1)
        return RVQ_ERR_INVALID;
    if (!vec_ok(a->src, a->n)) return RVQ_ERR_INVALID;
    TpPush p;
    memset(&p, 0, sizeof(p));
    p.src = a->src;
    p.n = a->n;
    p.rank = a->rank;
    p.tp = a->tp;
    for (int r = 0; r < a->tp; ++r) {
        if (a->dst[r] == nullptr || a->arrivals[r] == nullptr) return RVQ_ERR_INVALID;
        p.dst[r] = a->dst[r];
        p.arrivals[r] = a->arrivals[r];
    }
    const cudaError_t e = launch_pdl(tp_push_kernel, dim3(rvq_tp_push_ctas(a->n)), dim3(kPushThreads), 0,
                                     (cudaStream_t)stream, p);
    if (e != cudaSuccess) last_cuda_error_slot() = (int)e;
    return e == cudaSuccess ? launch_status() : RVQ_ERR_CUDA;
}

extern "C" int rvq_p2p_alloc(size_t bytes, void** out) {
    if (out == nullptr || bytes == 0) return RVQ_ERR_INVALID;
    cudaError_t e = cudaMalloc(out, bytes);
    if (e == cudaSuccess) e = cudaMemset(*out, 0, bytes);
    if (e != cudaSuccess) {
        last_cuda_error_slot() = (int)e;
        return RVQ_ERR_CUDA;
    }
    return RVQ_OK;
}

extern "C" int rvq_p2p_free(void* ptr) {
    const cudaError_t e = cudaFree(ptr);
    if (e != cudaSuccess) last_cuda_error_slot() = (int)e;
    return e == cudaSuccess ? RVQ_OK : RVQ_ERR_CUDA;
}

extern "C" int rvq_ipc_export(void* ptr, void* handle64) {
    if (ptr == nullptr || handle64 == nullptr) return RVQ_ERR_INVALID;
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, ptr);
    if (e != cudaSuccess) {
        last_cuda_error_slot() = (int)e;
        return RVQ_ERR_CUDA;
    }
    static_assert(sizeof(h) == 64, "IPC handle size");
    memcpy(handle64, &h, sizeof(h));
    return RVQ_OK;
}

extern "C" int rvq_ipc_import(const void* handle64, void** out) {
    if (handle64 == nullptr || out == nullptr) return RVQ_ERR_INVALID;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle64, sizeof(h));
    const cudaError_t e = cudaIpcOpenMemHandle(out, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
        last_cuda_error_slot() = (int)e;
        return RVQ_ERR_CUDA;
    }
    return RVQ_OK;
}

extern "C" int rvq_ipc_close(void* ptr) {
    const cudaError_t e = cudaIpcCloseMemHandle(ptr);
    if (e != cudaSuccess) last_cuda_error_slot() = (int)e;
    return e == cudaSuccess ? RVQ_OK : RVQ_ERR_CUDA;
}

extern "C" int rvq_take_tp_timeout(void) {
    int v = 0;
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&v, rvq::g_tp_timeout, sizeof(int));
    const int zero = 0;
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(rvq::g_tp_timeout, &zero, sizeof(int));
    if (e != cudaSuccess) {
        last_cuda_error_slot() = (int)e;
        return -RVQ_ERR_CUDA;
    }
    return v;
}
