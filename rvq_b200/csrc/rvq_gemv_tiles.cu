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
// One CTA owns one (job, tile, row range) unit.  Its rows' code words
// (interleaved layout, one 32-bit word per vector) stream into a two-slot
// shared-memory ring, 256 rows per TMA tile load (cp.async.bulk.tensor, zero
// fill past the matrix edge), while the CTA builds the tile's 128 KB table
// (4 stages x 256 codes x 32 groups, fp32, [stage][code][group]: lane g always
// reads bank g, so the random-code lookups never conflict).  Rows are reduced 8
// at a time with a warp reduce-scatter.  Nothing is shared between CTAs:
// partial sums go to [ntiles][rows] and the consumer adds them in tile order,
// so the result is deterministic and no cross-CTA synchronisation is needed.
// Matrices whose rows are not 16-byte aligned (cols / 8 not a multiple of 4)
// are staged with 4-byte cp.async instead of TMA.

#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>
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
constexpr int kPairs = kStages * kCodes;                    // (stage, code) table rows
constexpr int kLutFloats = kPairs * kGroups;                // 32768 floats, 128 KB
constexpr int kCbFloats = kPairs * 8;                       // codebook, fp32, 32 KB
constexpr int kBatchRows = 256;                             // rows per staged batch (TMA box height)
constexpr int kRing = 2;                                    // batches in flight
constexpr uint32_t kBatchBytes = kBatchRows * kGroups * 4;  // 32 KB
constexpr int kMaxJobs = 4;
constexpr int kMaxUnits = 1024;
constexpr long long kWaitLimit = 1ll << 22;                 // mbarrier polls before giving up
constexpr size_t kSmemBytes =
    (size_t)(kLutFloats + kCbFloats + kRing * kBatchRows * kGroups + kTileCols) * 4 + 64;

__device__ int g_wait_timeout;                              // sticky: a TMA wait gave up

struct TJob {
    const uint32_t* codes;      // [rows][G] interleaved code words
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
    int32_t use_tma;            // rows 16-byte aligned: TMA tile loads through maps[job]
};

struct TParams {
    CUtensorMap maps[kMaxJobs];   // [rows][G] uint32, box 32 x 256 (64-byte aligned, first)
    TJob jobs[kMaxJobs];
    int32_t n_units;
    int32_t pad;
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

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(smem_u32(dst)), "l"(src) : "memory");
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
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    for (long long i = 0; i < kWaitLimit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    atomicExch(&g_wait_timeout, 1);
    for (long long i = 0; i < kWaitLimit; ++i)
        if (mbar_try_wait(bar, parity)) break;
    return false;
}

// One 32 x 256 box of code words (tile columns x rows) into shared memory.
__device__ __forceinline__ void tma_load_rows(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    mbar_expect_tx(bar, kBatchBytes);
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n"
        ::"r"(dst), "l"(map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

// Fallback staging: rows [r0, r1) of a tile, 4 bytes at a time; one commit group.
__device__ __forceinline__ void stage_batch_words(const TJob& J, int tile, int gt, int r0, int r1, uint32_t* dst) {
    const int nrows = r1 - r0;
    const uint32_t* src = J.codes + (int64_t)r0 * J.G + (int64_t)tile * kGroups;
    for (int i = threadIdx.x; i < nrows * gt; i += kThreads) {
        const int r = i / gt, g = i - r * gt;
        cp_async4(dst + r * kGroups + g, src + (int64_t)r * J.G + g);
    }
    cp_async_commit();
}

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

// ---------------------------------------------------------------------------
// The tile's table LUT[q][g] = cb[q] . x[8g : 8g + 8], q = stage * 256 + code.
// ---------------------------------------------------------------------------

// FFMA: warp w builds table rows w + 32 j; lane = group.  Four rows'
// codebook entries are loaded (broadcast) before any of their table entries
// is stored; each store is one conflict-free 128-byte row.
__device__ __forceinline__ void build_lut_ffma(float* __restrict__ lut, const float* __restrict__ cbs,
                                               const float* __restrict__ xs) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float xr[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) xr[i] = xs[lane * 8 + i];
    const float4* cb4 = reinterpret_cast<const float4*>(cbs);
#pragma unroll 1
    for (int q0 = warp; q0 < kPairs; q0 += kWarps * 4) {
        float4 a[4], b[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            a[j] = cb4[(q0 + j * kWarps) * 2];
            b[j] = cb4[(q0 + j * kWarps) * 2 + 1];
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
        for (int j = 0; j < 4; ++j) lut[(q0 + j * kWarps) * kGroups + lane] = acc[j];
    }
}

__global__ void __launch_bounds__(kThreads, 1) rvq_gemv_tiles_kernel(const __grid_constant__ TParams p) {
    extern __shared__ __align__(128) float smem[];
    float* __restrict__ lut = smem;
    float* __restrict__ cbs = lut + kLutFloats;
    uint32_t* ring = reinterpret_cast<uint32_t*>(cbs + kCbFloats);
    float* xs = reinterpret_cast<float*>(ring + kRing * kBatchRows * kGroups);
    uint64_t* bars = reinterpret_cast<uint64_t*>(xs + kTileCols);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t bar0 = smem_u32(bars);

    __shared__ int slot_done[kRing];                     // warps finished with a ring slot
    if (tid < kRing) slot_done[tid] = 0;
    pdl_launch_dependents();
    if (tid == 0) {
        for (int s = 0; s < kRing; ++s) mbar_init(bar0 + 8 * s);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    __syncthreads();
    uint32_t phase_bits = 0;                             // bit s: parity of ring slot s's next phase

    for (int u = blockIdx.x; u < p.n_units; u += gridDim.x) {
        const uint32_t jt = p.unit_jt[u];
        const int ji = (int)(jt >> 24);
        const TJob& J = p.jobs[ji];
        const CUtensorMap* map = &p.maps[ji];
        const int tile = (int)(jt & 0xffffffu);
        const int r0 = p.unit_r0[u], r1 = p.unit_r1[u];
        const int G = J.G;
        const int gt = min(kGroups, G - tile * kGroups);
        const int nb = (r1 - r0 + kBatchRows - 1) / kBatchRows;
        const bool tma = J.use_tma != 0;
        if (u != (int)blockIdx.x) __syncthreads();      // the previous unit is done with shared memory

        // 1. code words of the first batches start streaming in
        if (tma) {
            if (tid == 0) {
                asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
                for (int b = 0; b < kRing && b < nb; ++b)
                    tma_load_rows(smem_u32(ring + b * kBatchRows * kGroups), map, tile * kGroups,
                                  r0 + b * kBatchRows, bar0 + 8 * b);
            }
        } else {
            for (int b = 0; b < kRing && b < nb; ++b)
                stage_batch_words(J, tile, gt, r0 + b * kBatchRows, min(r1, r0 + (b + 1) * kBatchRows),
                                  ring + b * kBatchRows * kGroups);
        }

        // 2. codebook (fp32) and the tile's operand slice
        if (J.cb_kind == RVQ_F32) {
            const float4* cb4 = reinterpret_cast<const float4*>(J.cb);
            for (int i = tid; i < kCbFloats / 4; i += kThreads) cp_async16(cbs + 4 * i, cb4 + i);
            cp_async_commit();
        } else {
            for (int i = tid; i < kCbFloats; i += kThreads) cbs[i] = load_as_f32(J.cb, i, J.cb_kind);
        }
        if (u == (int)blockIdx.x) pdl_wait();            // x comes from the previous kernel
        if (tid < kTileCols) {
            const int64_t col = (int64_t)tile * kTileCols + tid;
            float xv = 0.f;
            if (col < J.cols) {
                xv = operand(J.x, col);
                if (J.gate.ptr != nullptr) {
                    const float g = operand(J.gate, col);
                    xv = bf16r(bf16r(g / (1.0f + expf(-g))) * xv);
                }
            }
            xs[tid] = xv;
        }
        cp_async_wait<0>();          // the codebook (and, without TMA, the first code batches)
        __syncthreads();

        // 3. the tile's table (shared-memory bound: the codebook rows are broadcast
        //    loads, the table 128 KB of conflict-free stores)
        build_lut_ffma(lut, cbs, xs);
        __syncthreads();

        // 4. rows, batch by batch; batch b + 2 streams in while b + 1 is processed.
        //    With TMA every warp waits on the slot's barrier itself, and the last
        //    warp to finish a slot issues its refill: no CTA-wide barrier per batch.
        const float* lg = lut + lane;
        const uint32_t g_global = (uint32_t)tile * kGroups + lane;
        float* part = J.part + (int64_t)tile * J.rows;
        for (int b = 0; b < nb; ++b) {
            const int slot = b % kRing;
            if (tma) {
                mbar_wait(bar0 + 8 * slot, (phase_bits >> slot) & 1u);
                phase_bits ^= 1u << slot;
            } else {
                if (b + 1 < nb) cp_async_wait<1>();
                else cp_async_wait<0>();
                __syncthreads();
            }
            const int rb0 = r0 + b * kBatchRows;
            const int nrows = min(r1, rb0 + kBatchRows) - rb0;
            const uint32_t* cs = ring + slot * kBatchRows * kGroups + lane;
            for (int rb = warp * 8; rb < nrows; rb += kWarps * 8) {
                // this lane's output row (lanes 4i..4i+3 share row i): its scale is
                // fetched before the lookups so the load overlaps them
                const int orow = rb + ((lane >> 2) & 7);
                float oscale = 1.f;
                if (J.row_scales && (lane & 3) == 0 && orow < nrows)
                    oscale = load_as_f32(J.scales, fastdiv((uint32_t)(rb0 + orow), J.rpsdiv), J.scale_kind);
                float v[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const uint32_t w = cs[(rb + i) * kGroups];
                    float s = lg[(w & 0xffu) << 5];
                    s += lg[kCodes * kGroups + (((w >> 8) & 0xffu) << 5)];
                    s += lg[2 * kCodes * kGroups + (((w >> 16) & 0xffu) << 5)];
                    s += lg[3 * kCodes * kGroups + ((w >> 24) << 5)];
                    // rows past the unit (stale or next-unit words) and groups past
                    // the matrix edge (zero-filled or stale) contribute nothing
                    const bool valid = rb + i < nrows && lane < gt;
                    if (!J.row_scales)
                        s *= valid ? load_as_f32(J.scales,
                                                 fastdiv((uint32_t)(rb0 + rb + i) * (uint32_t)G + g_global, J.gvdiv),
                                                 J.scale_kind)
                                   : 0.f;
                    v[i] = valid ? s : 0.f;
                }
                const float tot = reduce8(v);
                if ((lane & 3) == 0 && orow < nrows) part[rb0 + orow] = tot * oscale;
            }
            if (b + kRing < nb) {
                const int nb0 = r0 + (b + kRing) * kBatchRows;
                uint32_t* buf = ring + slot * kBatchRows * kGroups;
                if (tma) {
                    __syncwarp();
                    if (lane == 0) {
                        __threadfence_block();
                        const int done = atomicAdd(&slot_done[slot], 1);
                        if (done == kWarps - 1) {               // every warp has left this slot
                            slot_done[slot] = 0;
                            __threadfence_block();
                            asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
                            tma_load_rows(smem_u32(buf), map, tile * kGroups, nb0, bar0 + 8 * slot);
                        }
                    }
                } else {
                    __syncthreads();                        // every warp is done with buf
                    stage_batch_words(J, tile, gt, nb0, min(r1, nb0 + kBatchRows), buf);
                }
            }
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
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

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
        if (e == cudaSuccess && prop.major == 10 && prop.sharedMemPerBlockOptin >= kSmemBytes) {
            d.sms = prop.multiProcessorCount;
            e = cudaFuncSetAttribute(rvq_gemv_tiles_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kSmemBytes);
            if (e == cudaSuccess && g_encode == nullptr) {
                void* fn = nullptr;
                cudaDriverEntryPointQueryResult q;
                e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
                if (e == cudaSuccess && q == cudaDriverEntryPointSuccess)
                    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
            }
            d.ok = e == cudaSuccess && g_encode != nullptr;
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
    if ((uintptr_t)w.indices & 3) return RVQ_ERR_INVALID;
    if (w.nvec >= (1ll << 32) || g.rows >= (1ll << 31) || (g.cols + kTileCols - 1) / kTileCols >= (1 << 24))
        return RVQ_ERR_TOO_LARGE;
    if (w.codebook_kind != RVQ_F32 && w.codebook_kind != RVQ_F16 && w.codebook_kind != RVQ_BF16)
        return RVQ_ERR_UNSUPPORTED;
    if (w.codebook_kind == RVQ_F32 && ((uintptr_t)w.codebook & 15)) return RVQ_ERR_INVALID;
    if (!operand_ok(g.x, g.cols) || (g.gate.ptr != nullptr && !operand_ok(g.gate, g.cols))) return RVQ_ERR_INVALID;
    if (g.partials == nullptr) return RVQ_ERR_INVALID;
    return RVQ_OK;
}

// Units: every (job, tile) gets CTAs in proportion to its work (rows x groups),
// at least one, the wave's remainder going to the largest fractional shares;
// each CTA takes an even share of its tile's rows.
int plan(const rvq_gemv_tile_job* jobs, int n, int sms, TParams& p) {
    struct T { int job, tile; double share; int ctas; int64_t rows; };
    static thread_local T ts[kMaxUnits];
    int nt = 0;
    double total = 0;
    for (int j = 0; j < n; ++j) {
        const int G = (int)(jobs[j].cols / 8);
        const int ntiles = (G + kGroups - 1) / kGroups;
        for (int t = 0; t < ntiles; ++t) {
            if (nt >= kMaxUnits) return RVQ_ERR_TOO_LARGE;
            const int gt = G - t * kGroups < kGroups ? G - t * kGroups : kGroups;
            ts[nt] = {j, t, (double)jobs[j].rows * gt, 1, jobs[j].rows};
            total += ts[nt].share;
            ++nt;
        }
    }
    int used = 0;
    const int budget = sms > nt ? sms : nt;
    for (int i = 0; i < nt; ++i) {
        const double want = ts[i].share / total * budget;
        int c = (int)want;
        if (c < 1) c = 1;
        if (c > ts[i].rows) c = (int)ts[i].rows;
        ts[i].ctas = c;
        ts[i].share = want - c;                  // remainder (negative when raised to 1)
        used += c;
    }
    while (used < budget) {                      // largest remainders first
        int best = -1;
        for (int i = 0; i < nt; ++i)
            if (ts[i].ctas < ts[i].rows && (best < 0 || ts[i].share > ts[best].share)) best = i;
        if (best < 0) break;
        ts[best].ctas += 1;
        ts[best].share -= 1.0;
        ++used;
    }
    int u = 0;
    for (int i = 0; i < nt; ++i) {
        for (int c = 0; c < ts[i].ctas; ++c) {
            if (u >= kMaxUnits) return RVQ_ERR_TOO_LARGE;
            p.unit_jt[u] = ((uint32_t)ts[i].job << 24) | (uint32_t)ts[i].tile;
            p.unit_r0[u] = (int32_t)(ts[i].rows * c / ts[i].ctas);
            p.unit_r1[u] = (int32_t)(ts[i].rows * (c + 1) / ts[i].ctas);
            ++u;
        }
    }
    p.n_units = u;
    return RVQ_OK;
}

// [rows][G] uint32 words, box 32 x 256; reads past either edge fill zeros.
int encode_map(CUtensorMap* m, const void* codes, int64_t rows, int64_t G) {
    const cuuint64_t dims[2] = {(cuuint64_t)G, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)G * 4};
    const cuuint32_t box[2] = {(cuuint32_t)kGroups, (cuuint32_t)kBatchRows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(codes), dims, strides, box,
                                estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? RVQ_OK : RVQ_ERR_INVALID;
}

}  // namespace tiles
}  // namespace rvq

using namespace rvq;
using namespace rvq::tiles;

extern "C" {

int64_t rvq_gemv_tiles_count(int64_t cols) { return cols < 1 ? 0 : (cols + kTileCols - 1) / kTileCols; }

int rvq_gemv_tiles(const rvq_gemv_tile_job* jobs, int n_jobs, void* stream) {
    if (jobs == nullptr || n_jobs < 1 || n_jobs > kMaxJobs) return RVQ_ERR_INVALID;
    for (int i = 0; i < n_jobs; ++i) {
        const int rc = check_job(jobs[i]);
        if (rc != RVQ_OK) return rc;
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
        J.use_tma = (J.G % 4 == 0) && (((uintptr_t)g.weight.indices & 15) == 0);
        if (J.use_tma) {
            rc = encode_map(&p.maps[i], g.weight.indices, g.rows, J.G);
            if (rc != RVQ_OK) return rc;
        }
    }
    rc = plan(jobs, n_jobs, d->sms, p);
    if (rc != RVQ_OK) return rc;
    const int grid = p.n_units < d->sms ? p.n_units : d->sms;
    cudaError_t e = launch_pdl(rvq_gemv_tiles_kernel, dim3(grid), dim3(kThreads), kSmemBytes, (cudaStream_t)stream, p);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) {
        last_cuda_error_slot() = (int)e;
        return RVQ_ERR_CUDA;
    }
    return RVQ_OK;
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
