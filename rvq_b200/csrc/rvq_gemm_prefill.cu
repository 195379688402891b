// Prefill GEMM with the RVQ weight decoded into shared memory (sm_100a):
//
//   Y[m][n] = bf16( sum_k X[m][k] * W[n][k] ),   W = RVQ entry [N, K]
//
// The reference prefills through decode-into-slot + F.linear
// (infer_compressed_layerwise_triton.py:263, 290-292): the bf16 weight makes
// a round trip through HBM.  Here each CTA owns a 128 x 256 tile of Y; for
// every 64-column chunk of K it
//   * loads X[m0 : m0 + 128][k0 : k0 + 64] by TMA (128-byte swizzle),
//   * decodes W[n0 : n0 + 256][k0 : k0 + 64] straight into shared memory in
//     the same K-major 128-byte-swizzled layout -- one RVQ vector is exactly
//     one 16-byte swizzle chunk -- with the reference's arithmetic (fp32 sum
//     of the stages from +0 in stage order, times the fp32 scale, rounded to
//     bf16: bit-identical to the slot),
//   * and one thread issues four tcgen05.mma (kind::f16, M=128, N=256, K=16)
//     accumulating into TMEM, committed to an mbarrier.
// Two stages: the decode and TMA of chunk i+1 overlap the MMAs of chunk i.
// The epilogue reads the accumulator with tcgen05.ld and stores bf16 rows.
// Only the codes (0.5 B / weight) and X are read from HBM.

#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <string.h>

#include "rvq_common.cuh"

namespace rvq {
namespace gemm {

constexpr int kDecodeWarps = 16;                               // decode the weight chunks
constexpr int kThreads = (kDecodeWarps + 1) * 32;               // + one TMA / MMA issuing warp
constexpr int kDecodeThreads = kDecodeWarps * 32;
constexpr int kTileM = 128;
constexpr int kTileN = 256;
constexpr int kChunkK = 64;                                    // one 128-byte swizzle row of bf16
constexpr int kStages = 3;                                     // W stages: decoders run up to 2 chunks ahead
constexpr int kXStages = 4;                                    // X stages: TMA runs 3 chunks ahead
constexpr int kXStageBytes = kTileM * kChunkK * 2;             // 16 KB
constexpr int kWStageBytes = kTileN * kChunkK * 2;             // 32 KB
constexpr int kCbFloats = 4 * 256 * 8;                          // fp32 codebook entries
constexpr int kCbCopies = 4;                                    // fp16 copies: lane & 3 reads copy lane & 3
constexpr int kCbHalfBytes = 4 * 256 * kCbCopies * 16;          // 64 KB (>= the 32 KB fp32 fallback)
constexpr int kVecPerThread = kTileN * 8 / kDecodeThreads;      // vectors each decoder thread does per chunk
constexpr int kTmemCols = 256;
constexpr long long kWaitLimit = 1ll << 24;
constexpr size_t kSmemBytes = 1024 /* alignment slack */ + kXStages * kXStageBytes + kStages * kWStageBytes +
                              kCbHalfBytes + 256 /* barriers, TMEM address */;

__device__ int g_gemm_timeout;

struct GParams {
    CUtensorMap xmap;           // X [M][K] bf16, box 64 x 128, 128-byte swizzle
    const uint32_t* codes;      // [N][K/8] interleaved code words (byte s = stage s)
    const float* cb;            // [4][256][8] fp32
    const void* scales;
    void* y;                    // [M][N] bf16
    int32_t M, N, K;
    int32_t scale_kind;
    FastDiv gvdiv;              // vectors per scale
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
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

// Bounded wait; on timeout sets the sticky flag and returns false.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    for (long long i = 0; i < kWaitLimit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    atomicExch(&g_gemm_timeout, 1);
    return false;
}

// K-major, 128-byte-swizzled operand: rows of 128 bytes, 8-row atoms of 1024
// bytes (stride byte offset), leading byte offset unused (1), descriptor
// version 1, layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)1u << 16;                     // leading byte offset (16 B units)
    d |= (uint64_t)(1024u >> 4) << 32;           // stride byte offset: 1024 B between 8-row groups
    d |= (uint64_t)1u << 46;                     // version
    d |= (uint64_t)2u << 61;                     // SWIZZLE_128B
    return d;
}

// kind::f16 instruction descriptor: D fp32, A and B bf16, both K-major, M x N.
__host__ __device__ constexpr uint32_t instr_desc(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
}

__global__ void __launch_bounds__(kThreads, 1) rvq_gemm_prefill_kernel(const __grid_constant__ GParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* xs = base;                                               // [4][16 KB]
    uint8_t* ws = xs + kXStages * kXStageBytes;                       // [3][32 KB]
    uint4* cbh = reinterpret_cast<uint4*>(ws + kStages * kWStageBytes);     // fp16, 4 copies (or fp32)
    uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(cbh) + kCbHalfBytes);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kXStages + kStages);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * kTileN, m0 = blockIdx.y * kTileM;
    // x_full[4] (TMA), done[4] (MMAs of chunk c, committed to done[c % 4]),
    // w_full[3] (the decoder warps of a stage)
    const uint32_t bar_x = smem_u32(bars), bar_done = smem_u32(bars + kXStages);
    const uint32_t bar_w = smem_u32(bars + 2 * kXStages);
    const int KC = p.K / kChunkK;
    const int G = p.K / 8;

    if (tid == 0) {
        for (int s = 0; s < kXStages; ++s) {
            mbar_init(bar_x + 8 * s, 1);
            mbar_init(bar_done + 8 * s, 1);
        }
        for (int s = 0; s < kStages; ++s) mbar_init(bar_w + 8 * s, kDecodeWarps);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    }
    // codebook: fp16 with 8 interleaved copies when every value survives the
    // round trip exactly (always for artifact codebooks), else fp32 (one copy)
    bool exact = true;
    for (int e = tid; e < 4 * 256; e += kThreads) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(p.cb) + 2 * e);
        const float4 b = __ldg(reinterpret_cast<const float4*>(p.cb) + 2 * e + 1);
        const __half2 h0 = __floats2half2_rn(a.x, a.y), h1 = __floats2half2_rn(a.z, a.w);
        const __half2 h2 = __floats2half2_rn(b.x, b.y), h3 = __floats2half2_rn(b.z, b.w);
        exact &= __low2float(h0) == a.x && __high2float(h0) == a.y && __low2float(h1) == a.z &&
                 __high2float(h1) == a.w && __low2float(h2) == b.x && __high2float(h2) == b.y &&
                 __low2float(h3) == b.z && __high2float(h3) == b.w;
        const uint4 q = make_uint4(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1),
                                   *reinterpret_cast<const uint32_t*>(&h2), *reinterpret_cast<const uint32_t*>(&h3));
#pragma unroll
        for (int c = 0; c < kCbCopies; ++c) cbh[e * kCbCopies + ((c + lane) & (kCbCopies - 1))] = q;
    }
    const bool f16cb = __syncthreads_and(exact) != 0;
    if (!f16cb) {
        float4* cbf = reinterpret_cast<float4*>(cbh);
        for (int i = tid; i < kCbFloats / 4; i += kThreads) cbf[i] = __ldg(reinterpret_cast<const float4*>(p.cb) + i);
    }
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    const uint32_t idesc = instr_desc(kTileM, kTileN);
    bool ok = true;

    if (warp == kDecodeWarps) {
        // ---- issuer warp: X by TMA (3 chunks ahead), MMAs as soon as a chunk's W is decoded
        if (lane == 0) {
            auto issue_x = [&](int c) {
                const int st = c % kXStages;
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar_x + 8 * st),
                             "r"((uint32_t)kXStageBytes)
                             : "memory");
                asm volatile(
                    "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
                    "%3}], [%4];\n" ::"r"(smem_u32(xs + st * kXStageBytes)),
                    "l"(&p.xmap), "r"(c * kChunkK), "r"(m0), "r"(bar_x + 8 * st)
                    : "memory");
            };
            for (int c = 0; c < kXStages - 1 && c < KC; ++c) issue_x(c);
            for (int kc = 0; kc < KC; ++kc) {
                const int xst = kc % kXStages, wst = kc % kStages;
                if (!mbar_wait(bar_w + 8 * wst, (kc / kStages) & 1)) ok = false;
                if (!mbar_wait(bar_x + 8 * xst, (kc / kXStages) & 1)) ok = false;
                asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
                const uint32_t xa = smem_u32(xs + xst * kXStageBytes), wa = smem_u32(ws + wst * kWStageBytes);
#pragma unroll
                for (int ks = 0; ks < kChunkK / 16; ++ks) {
                    const uint64_t da = sw128_desc(xa + 32 * ks), db = sw128_desc(wa + 32 * ks);
                    const uint32_t accum = (kc > 0 || ks > 0) ? 1u : 0u;
                    asm volatile(
                        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
                        "l"(da), "l"(db), "r"(idesc), "r"(accum)
                        : "memory");
                }
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                                 bar_done + 8 * xst)
                             : "memory");
                // X for chunk kc + 3 reuses chunk kc - 1's stage once its MMAs are done
                if (kc + kXStages - 1 < KC) {
                    if (kc >= 1 && !mbar_wait(bar_done + 8 * ((kc - 1) % kXStages), ((kc - 1) / kXStages) & 1))
                        ok = false;
                    issue_x(kc + kXStages - 1);
                }
            }
        }
        __syncwarp();
    } else {
        // ---- decoder warps: thread (v = t & 7, r = (t >> 3) + 64 j); code words and
        //      scales two chunks ahead in registers
        const int v = tid & 7;
        const float* cbf = reinterpret_cast<const float*>(cbh);
        uint32_t w1[kVecPerThread], w2[kVecPerThread];
        float s1[kVecPerThread], s2[kVecPerThread];
        auto fetch = [&](int kc, uint32_t (&wo)[kVecPerThread], float (&so)[kVecPerThread]) {
#pragma unroll
            for (int j = 0; j < kVecPerThread; ++j) {
                const int n = n0 + (tid >> 3) + (kDecodeThreads / 8) * j;
                wo[j] = 0u;
                so[j] = 0.f;
                if (n < p.N && kc < KC) {
                    const uint32_t vec = (uint32_t)n * (uint32_t)G + (uint32_t)(kc * 8 + v);
                    wo[j] = __ldg(p.codes + vec);
                    so[j] = load_as_f32(p.scales, fastdiv(vec, p.gvdiv), p.scale_kind);
                }
            }
        };
        fetch(0, w1, s1);
        fetch(1, w2, s2);
        for (int kc = 0; kc < KC; ++kc) {
            const int s = kc % kStages;
            uint32_t w[kVecPerThread];
            float sc[kVecPerThread];
#pragma unroll
            for (int j = 0; j < kVecPerThread; ++j) {
                w[j] = w1[j];
                sc[j] = s1[j];
                w1[j] = w2[j];
                s1[j] = s2[j];
            }
            fetch(kc + 2, w2, s2);
            if (kc >= kStages) {                    // the MMAs of chunk kc - 3 (stage s) are done
                const int c = kc - kStages;
                if (lane == 0 && !mbar_wait(bar_done + 8 * (c % kXStages), (c / kXStages) & 1)) ok = false;
                __syncwarp();
            }
            uint8_t* wst = ws + s * kWStageBytes;
#pragma unroll
            for (int j = 0; j < kVecPerThread; ++j) {
                const int r = (tid >> 3) + (kDecodeThreads / 8) * j;
                float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
                if (f16cb) {
#pragma unroll
                    for (int st = 0; st < 4; ++st) {
                        const uint32_t c = (w[j] >> (8 * st)) & 0xFFu;
                        const uint4 q = cbh[((st * 256u + c) * kCbCopies) + (lane & (kCbCopies - 1))];
                        add_f16x2_f32(acc[0], acc[1], q.x);
                        add_f16x2_f32(acc[2], acc[3], q.y);
                        add_f16x2_f32(acc[4], acc[5], q.z);
                        add_f16x2_f32(acc[6], acc[7], q.w);
                    }
                } else {
#pragma unroll
                    for (int st = 0; st < 4; ++st) {
                        const uint32_t c = (w[j] >> (8 * st)) & 0xFFu;
                        const float4 a = *reinterpret_cast<const float4*>(cbf + (st * 256 + c) * 8);
                        const float4 b = *reinterpret_cast<const float4*>(cbf + (st * 256 + c) * 8 + 4);
                        acc[0] = __fadd_rn(acc[0], a.x); acc[1] = __fadd_rn(acc[1], a.y);
                        acc[2] = __fadd_rn(acc[2], a.z); acc[3] = __fadd_rn(acc[3], a.w);
                        acc[4] = __fadd_rn(acc[4], b.x); acc[5] = __fadd_rn(acc[5], b.y);
                        acc[6] = __fadd_rn(acc[6], b.z); acc[7] = __fadd_rn(acc[7], b.w);
                    }
                }
                uint4 q;
                q.x = pack_bf16x2(__fmul_rn(acc[0], sc[j]), __fmul_rn(acc[1], sc[j]));
                q.y = pack_bf16x2(__fmul_rn(acc[2], sc[j]), __fmul_rn(acc[3], sc[j]));
                q.z = pack_bf16x2(__fmul_rn(acc[4], sc[j]), __fmul_rn(acc[5], sc[j]));
                q.w = pack_bf16x2(__fmul_rn(acc[6], sc[j]), __fmul_rn(acc[7], sc[j]));
                *reinterpret_cast<uint4*>(wst + r * 128 + ((v ^ (r & 7)) << 4)) = q;
            }
            // generic-proxy stores must be visible to the tensor core's async proxy
            asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar_w + 8 * s) : "memory");
        }
    }
    // every MMA is done once chunk KC - 1's commit has arrived
    if (KC > 0 && lane == 0 && !mbar_wait(bar_done + 8 * ((KC - 1) % kXStages), ((KC - 1) / kXStages) & 1)) ok = false;
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");

    // epilogue: warps 0-3 own TMEM lanes 32 w .. 32 w + 31 = rows of the tile
    const bool all_ok = __syncthreads_and(ok) != 0;
    if (warp < 4 && all_ok) {
        const int row = m0 + 32 * warp + lane;
        __nv_bfloat16* yrow = reinterpret_cast<__nv_bfloat16*>(p.y) + (int64_t)row * p.N;
        for (int c = 0; c < kTileN / 32; ++c) {
            uint32_t r[32];
            const uint32_t taddr = tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)(32 * c);
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
                "%13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, "
                "[%32];\n"
                : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                  "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                  "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
                  "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
                  "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                : "r"(taddr)
                : "memory");
            asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
            const int nc = n0 + 32 * c;
            if (row < p.M) {
                if (nc + 32 <= p.N) {
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        uint4 o;
                        o.x = pack_bf16x2(__uint_as_float(r[8 * i + 0]), __uint_as_float(r[8 * i + 1]));
                        o.y = pack_bf16x2(__uint_as_float(r[8 * i + 2]), __uint_as_float(r[8 * i + 3]));
                        o.z = pack_bf16x2(__uint_as_float(r[8 * i + 4]), __uint_as_float(r[8 * i + 5]));
                        o.w = pack_bf16x2(__uint_as_float(r[8 * i + 6]), __uint_as_float(r[8 * i + 7]));
                        *reinterpret_cast<uint4*>(yrow + nc + 8 * i) = o;
                    }
                } else {
                    for (int i = 0; i < 32; ++i)
                        if (nc + i < p.N) yrow[nc + i] = __float2bfloat16_rn(__uint_as_float(r[i]));
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

// ---------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------
std::mutex g_mu;
bool g_ready[64] = {}, g_ok[64] = {};
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int prepare() {
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
        if (e == cudaSuccess && prop.major == 10 && prop.sharedMemPerBlockOptin >= kSmemBytes) {
            e = cudaFuncSetAttribute(rvq_gemm_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kSmemBytes);
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
    return g_ok[dev] ? RVQ_OK : RVQ_ERR_UNAVAILABLE;
}

}  // namespace gemm
}  // namespace rvq

using namespace rvq;
using namespace rvq::gemm;

extern "C" {

int rvq_gemm_prefill(const rvq_gemm_job* job, void* stream) {
    if (job == nullptr || job->x == nullptr || job->y == nullptr) return RVQ_ERR_INVALID;
    const rvq_entry& w = job->weight;
    int rc = rvq_check_entry(&w);
    if (rc != RVQ_OK) return rc;
    if (w.stages != 4 || w.ncodes != 256 || w.index_kind != RVQ_U8 || w.codebook_kind != RVQ_F32 || w.d != 8)
        return RVQ_ERR_UNSUPPORTED;
    const int64_t M = job->m, N = job->n, K = job->k;
    if (M < 1 || N < 1 || K < kChunkK || K % kChunkK != 0) return RVQ_ERR_UNSUPPORTED;
    if (N * (K / 8) != w.nvec || w.trimmed != w.nvec * 8 || w.tail_numel != 0) return RVQ_ERR_UNSUPPORTED;
    if (M >= (1ll << 31) || w.nvec >= (1ll << 32)) return RVQ_ERR_TOO_LARGE;
    if (((uintptr_t)w.indices & 3) || ((uintptr_t)w.codebook & 15) || ((uintptr_t)job->x & 15) ||
        ((uintptr_t)job->y & 15) || N % 8 != 0)
        return RVQ_ERR_INVALID;
    if (job->x_kind != RVQ_BF16 || job->y_kind != RVQ_BF16) return RVQ_ERR_UNSUPPORTED;
    rc = prepare();
    if (rc != RVQ_OK) return rc;
    static thread_local GParams p;
    memset(&p, 0, sizeof(p));
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kChunkK, (cuuint32_t)kTileM};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult cr = g_encode(&p.xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(job->x), dims, strides,
                                 box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return RVQ_ERR_INVALID;
    p.codes = reinterpret_cast<const uint32_t*>(w.indices);
    p.cb = reinterpret_cast<const float*>(w.codebook);
    p.scales = w.scales;
    p.y = job->y;
    p.M = (int32_t)M;
    p.N = (int32_t)N;
    p.K = (int32_t)K;
    p.scale_kind = w.scale_kind;
    p.gvdiv = make_fastdiv((uint32_t)w.group_vecs);
    const dim3 grid((unsigned)((N + kTileN - 1) / kTileN), (unsigned)((M + kTileM - 1) / kTileM));
    rvq_gemm_prefill_kernel<<<grid, kThreads, kSmemBytes, (cudaStream_t)stream>>>(p);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        last_cuda_error_slot() = (int)e;
        return RVQ_ERR_CUDA;
    }
    return RVQ_OK;
}

int rvq_take_gemm_timeout(void) {
    int v = 0;
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&v, g_gemm_timeout, sizeof(int));
    const int zero = 0;
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_gemm_timeout, &zero, sizeof(int));
    if (e != cudaSuccess) {
        last_cuda_error_slot() = (int)e;
        return -RVQ_ERR_CUDA;
    }
    return v;
}

}  // extern "C"
