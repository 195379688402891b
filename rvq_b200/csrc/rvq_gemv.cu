// Fused RVQ dequant-GEMV for batch-1 decode (sm_100a): y = W x without
// materialising W.
//
// W is an RVQ entry (K=4 stages x 256 codes, d=8, uint8 codes; any scale
// grouping).  For column group j (8 columns) and stage k, a lookup table
// LUT_k[c][j] = dot(cb_k[c], x[8j .. 8j+8]) turns every 8-weight vector into
// 4 table lookups and 3 adds instead of 32 element reconstructions:
//
//   y[r] = sum_j  scale(r, j) * (((LUT_0[c0] + LUT_1[c1]) + LUT_2[c2]) + LUT_3[c3])
//
// This is the exact sum of W[r, :] x in real arithmetic; in floating point it
// differs from "reconstruct W, round it to bf16, then matmul" by the bf16
// rounding of each weight (relative 2^-9 per weight), which is why this path
// is compared against the reference reconstruct + matmul with a tolerance.
//
// Two launches per call:
// 1. rvq_lut_kernel builds every 256-column tile's table once ([4][256][32]
//    fp32 = 128 KB per tile) into the workspace: thread (code c, group g)
//    forms dot(cb[k][c], x of group g), so a warp writes 128 contiguous bytes.
// 2. rvq_gemv_kernel: CTA (tile, row range) copies its tile's table into
//    shared memory, then each warp walks 8 rows at a time.  Lane g owns column
//    group g of the tile: the codes of (row, group) come as one 32-bit word when
//    the codes are interleaved ([nvec][4], see rvq_interleave_codes), 4 bytes
//    from the 4 planes otherwise; table reads are conflict-free (lane g reads
//    bank g).  The 8 rows are reduced over the 32 lanes with a transpose
//    reduction (9 shuffles); per-tile row partials go to the workspace and the
//    last CTA of a row range (atomic ticket) sums the tiles in tile order, so
//    results are deterministic run to run.

#include <string.h>

#include <mutex>

#include "rvq_common.cuh"

namespace rvq {
namespace gemv {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr int kLutThreads = 256;
constexpr int kGroupsPerTile = 32;               // 256 columns per tile
constexpr int kStages = 4;
constexpr int kCodes = 256;
constexpr int kRowBatch = 8;                     // rows a warp decodes and reduces together
constexpr int kMaxJobs = 4;                       // q/k/v or gate/up share one launch
constexpr size_t kLutBytes = (size_t)kStages * kCodes * kGroupsPerTile * sizeof(float);   // 128 KB

struct Job {
    const uint8_t* idx;        // planar [4][stage_stride] or interleaved [nvec][4] codes
    const void* cb;            // [4][256][8] fp16 or fp32
    const void* scales;        // scale per group_vecs vectors
    const void* x;             // [cols]
    void* y;                   // [rows]
    float* partial;            // [ntiles][rows] workspace
    unsigned int* tickets;     // [nranges] workspace, zero between launches
    float* lut;                // [ntiles][4][256][32] workspace
    uint32_t rows;
    uint32_t groups;           // cols / 8
    uint32_t stage_stride;
    FastDiv gv;                // group_vecs
    uint32_t ntiles;           // ceil(groups / 32)
    uint32_t nranges;          // row ranges per tile
    uint32_t cta_begin;        // first CTA of this job (product launch)
    uint32_t lut_cta_begin;    // first CTA of this job (table launch)
    uint8_t cb_kind, scale_kind, x_kind, y_kind;
    uint8_t row_scales;        // one scale per row: applied once, after the tile sum
    uint8_t interleaved;       // codes are [nvec][4]
};

struct Params {
    Job jobs[kMaxJobs];
    int njobs;
};

__device__ __forceinline__ float ldf(const void* p, uint32_t i, int kind) {
    if (kind == RVQ_F16) return __half2float(__ldg(reinterpret_cast<const __half*>(p) + i));
    if (kind == RVQ_BF16) return __bfloat162float(__ldg(reinterpret_cast<const __nv_bfloat16*>(p) + i));
    return __ldg(reinterpret_cast<const float*>(p) + i);
}

// ---------------------------------------------------------------------------
// 1. tables
// ---------------------------------------------------------------------------

// CTA (job, tile, stage): LUT[stage][c][g] for 256 codes x 32 groups.
__global__ void __launch_bounds__(kLutThreads) rvq_lut_kernel(const __grid_constant__ Params p) {
    __shared__ float xs[kGroupsPerTile * 8];
    __shared__ float4 cw[kCodes * 2];
    int ji = 0;
    while (ji + 1 < p.njobs && blockIdx.x >= p.jobs[ji + 1].lut_cta_begin) ++ji;
    const Job& job = p.jobs[ji];
    const uint32_t local = blockIdx.x - job.lut_cta_begin;
    const uint32_t tile = local / kStages, k = local % kStages;
    const uint32_t g0 = tile * kGroupsPerTile;
    // activations of the tile's 32 groups (zero past the matrix) and stage k's codebook
    {
        const uint32_t col = g0 * 8 + threadIdx.x;
        xs[threadIdx.x] = col < job.groups * 8 ? ldf(job.x, col, job.x_kind) : 0.0f;
    }
    for (int e = threadIdx.x; e < kCodes * 2; e += kLutThreads) {
        float4 v;
        if (job.cb_kind == RVQ_F32) {
            v = __ldg(reinterpret_cast<const float4*>(job.cb) + (size_t)k * kCodes * 2 + e);
        } else {
            const uint2 h = __ldg(reinterpret_cast<const uint2*>(job.cb) + (size_t)k * kCodes * 2 + e);
            v.x = __half2float(__ushort_as_half((uint16_t)(h.x & 0xFFFFu)));
            v.y = __half2float(__ushort_as_half((uint16_t)(h.x >> 16)));
            v.z = __half2float(__ushort_as_half((uint16_t)(h.y & 0xFFFFu)));
            v.w = __half2float(__ushort_as_half((uint16_t)(h.y >> 16)));
        }
        cw[e] = v;
    }
    __syncthreads();
    const int g = threadIdx.x & 31, w = threadIdx.x >> 5;
    float xg[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) xg[t] = xs[g * 8 + t];
    float* out = job.lut + ((size_t)tile * kStages + k) * kCodes * kGroupsPerTile;
#pragma unroll 4
    for (int c = w; c < kCodes; c += kLutThreads / 32) {
        const float4 a = cw[2 * c], b = cw[2 * c + 1];
        float d = a.x * xg[0];
        d = fmaf(a.y, xg[1], d);
        d = fmaf(a.z, xg[2], d);
        d = fmaf(a.w, xg[3], d);
        d = fmaf(b.x, xg[4], d);
        d = fmaf(b.y, xg[5], d);
        d = fmaf(b.z, xg[6], d);
        d = fmaf(b.w, xg[7], d);
        out[c * kGroupsPerTile + g] = d;
    }
}

// ---------------------------------------------------------------------------
// 2. the product
// ---------------------------------------------------------------------------

// Codes of (row, this lane's group), one stage per byte.
__device__ __forceinline__ uint32_t load_codes(const Job& job, uint32_t row, uint32_t r1, uint32_t j, bool active) {
    if (!active || row >= r1) return 0u;
    const size_t n = (size_t)row * job.groups + j;
    if (job.interleaved) return __ldg(reinterpret_cast<const uint32_t*>(job.idx) + n);
    const uint8_t* s = job.idx + n;
    return (uint32_t)__ldg(s) | ((uint32_t)__ldg(s + job.stage_stride) << 8) |
           ((uint32_t)__ldg(s + 2 * (size_t)job.stage_stride) << 16) |
           ((uint32_t)__ldg(s + 3 * (size_t)job.stage_stride) << 24);
}

// The product for job J; J is a compile-time slot so the job's fields are
// read straight from the parameter bank instead of occupying registers.
template <int J>
__device__ __forceinline__ void gemv_job(const Params& p, float* lut, int* s_last_ptr) {
    int& s_last = *s_last_ptr;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const Job& job = p.jobs[J];
    const uint32_t local = blockIdx.x - job.cta_begin;
    const uint32_t tile = local / job.nranges, range = local % job.nranges;
    const uint32_t j = tile * kGroupsPerTile + lane;    // this lane's column group
    const bool active = j < job.groups;
    const uint32_t r0 = (uint32_t)(((uint64_t)job.rows * range) / job.nranges);
    const uint32_t r1 = (uint32_t)(((uint64_t)job.rows * (range + 1)) / job.nranges);

    // the tile's table into shared memory
    {
        const float4* src = reinterpret_cast<const float4*>(job.lut + (size_t)tile * kStages * kCodes * kGroupsPerTile);
        float4* dst = reinterpret_cast<float4*>(lut);
        constexpr int kPer = (int)(kLutBytes / 16) / kThreads;          // 8 float4 per thread
        float4 v[kPer];
#pragma unroll
        for (int i = 0; i < kPer; ++i) v[i] = __ldcg(src + threadIdx.x + i * kThreads);
#pragma unroll
        for (int i = 0; i < kPer; ++i) dst[threadIdx.x + i * kThreads] = v[i];
    }
    __syncthreads();

    const uint32_t G = job.groups;
    float* part = job.partial + (size_t)tile * job.rows;
    const float* lut_lane = lut + lane;
    bool wrote = false;
    // Lane sums of 8 rows -> row (rb + lane/4 % 8) complete in lanes 4m..4m+3.
    auto reduce8 = [&](float (&v)[kRowBatch]) -> float {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const bool up = lane & 16;
            const float send = up ? v[i] : v[i + 4], keep = up ? v[i + 4] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const bool up = lane & 8;
            const float send = up ? v[i] : v[i + 2], keep = up ? v[i + 2] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
        }
        const bool up = lane & 4;
        const float send = up ? v[0] : v[1], keep = up ? v[1] : v[0];
        float r = keep + __shfl_xor_sync(0xffffffffu, send, 4);
        r += __shfl_xor_sync(0xffffffffu, r, 2);
        r += __shfl_xor_sync(0xffffffffu, r, 1);
        return r;
    };
    // ((LUT_0[c0] + LUT_1[c1]) + LUT_2[c2]) + LUT_3[c3] for one code word
    auto lookup = [&](uint32_t cw) -> float {
        float a = lut_lane[(cw & 0xFFu) * kGroupsPerTile];
        a += lut_lane[((cw >> 8) & 0xFFu) * kGroupsPerTile + 1 * kCodes * kGroupsPerTile];
        a += lut_lane[((cw >> 16) & 0xFFu) * kGroupsPerTile + 2 * kCodes * kGroupsPerTile];
        a += lut_lane[(cw >> 24) * kGroupsPerTile + 3 * kCodes * kGroupsPerTile];
        return a;
    };

    const uint32_t step = kWarps * kRowBatch;
    uint32_t rb = r0 + warp * kRowBatch;
    // warp-uniform: every lane of a full tile has a live column
    const bool fast = job.interleaved && job.row_scales && (tile + 1) * kGroupsPerTile <= job.groups;
    if (fast) {
        // interleaved codes, one scale per row, a full tile: full batches
        // need no masks; the lane's code word of row r is codes[r * G]
        const uint32_t* codes = reinterpret_cast<const uint32_t*>(job.idx) + j;
        const uint32_t full_end = r1 >= kRowBatch ? r1 - kRowBatch + 1 : 0;     // rb < full_end: 8 rows in range
        uint32_t wa[kRowBatch];
        if (rb < full_end) {
#pragma unroll
            for (int i = 0; i < kRowBatch; ++i) wa[i] = __ldg(codes + (size_t)(rb + i) * G);
        }
        while (rb < full_end) {
            const uint32_t nb = rb + step;
            uint32_t wb[kRowBatch];
            if (nb < full_end) {
#pragma unroll
                for (int i = 0; i < kRowBatch; ++i) wb[i] = __ldg(codes + (size_t)(nb + i) * G);
            }
            float v[kRowBatch];
#pragma unroll
            for (int i = 0; i < kRowBatch; ++i) v[i] = lookup(wa[i]);
            const float r = reduce8(v);
            if ((lane & 3) == 0) part[rb + ((lane >> 2) & 7)] = r;
            wrote = true;
            rb = nb;
            if (rb >= full_end) break;
            const uint32_t nb2 = rb + step;
            if (nb2 < full_end) {
#pragma unroll
                for (int i = 0; i < kRowBatch; ++i) wa[i] = __ldg(codes + (size_t)(nb2 + i) * G);
            }
#pragma unroll
            for (int i = 0; i < kRowBatch; ++i) v[i] = lookup(wb[i]);
            const float r2 = reduce8(v);
            if ((lane & 3) == 0) part[rb + ((lane >> 2) & 7)] = r2;
            rb = nb2;
        }
    }
    // general rows (and the last partial batch of the fast path): masked
    for (; rb < r1; rb += step) {
        float v[kRowBatch];
#pragma unroll
        for (int i = 0; i < kRowBatch; ++i) {
            const uint32_t row = rb + i;
            const uint32_t cw = load_codes(job, row, r1, j, active);
            float a = lookup(cw);
            if (!job.row_scales)
                a *= (active && row < r1) ? ldf(job.scales, fastdiv(row * G + j, job.gv), job.scale_kind) : 0.0f;
            v[i] = (active && row < r1) ? a : 0.0f;
        }
        const float r = reduce8(v);
        const uint32_t row = rb + ((lane >> 2) & 7);
        if ((lane & 3) == 0 && row < r1) {
            part[row] = r;
            wrote = true;
        }
    }

    // ---- last CTA of this row range sums the tiles in tile order ----
    if (wrote) __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned int ticket = atomicAdd(job.tickets + range, 1u);
        s_last = ticket == job.ntiles - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (uint32_t r = r0 + threadIdx.x; r < r1; r += kThreads) {
        float acc = 0.0f;
        for (uint32_t t = 0; t < job.ntiles; ++t) acc += __ldcg(job.partial + (size_t)t * job.rows + r);
        if (job.row_scales) acc *= ldf(job.scales, r, job.scale_kind);
        store_from_f32(job.y, r, job.y_kind, acc);
    }
    if (threadIdx.x == 0) job.tickets[range] = 0u;      // ready for the next launch
}

__global__ void __launch_bounds__(kThreads, 1) rvq_gemv_kernel(const __grid_constant__ Params p) {
    extern __shared__ __align__(16) float lut[];                         // [4][256][32]
    __shared__ int s_last;
    int ji = 0;
    while (ji + 1 < p.njobs && blockIdx.x >= p.jobs[ji + 1].cta_begin) ++ji;
    switch (ji) {
        case 0: gemv_job<0>(p, lut, &s_last); break;
        case 1: gemv_job<1>(p, lut, &s_last); break;
        case 2: gemv_job<2>(p, lut, &s_last); break;
        default: gemv_job<3>(p, lut, &s_last); break;
    }
}

// codes[n] = planes[0][n] | planes[1][n] << 8 | planes[2][n] << 16 | planes[3][n] << 24
__global__ void rvq_interleave_kernel(const uint8_t* planes, uint64_t stage_stride, uint64_t nvec, uint32_t* out) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t n = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; n < nvec; n += stride) {
        out[n] = (uint32_t)planes[n] | ((uint32_t)planes[n + stage_stride] << 8) |
                 ((uint32_t)planes[n + 2 * stage_stride] << 16) | ((uint32_t)planes[n + 3 * stage_stride] << 24);
    }
}

// ---------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------

struct DevInfo {
    bool ready = false, ok = false;
    int sms = 0;
};
static DevInfo g_dev[64];
static std::mutex g_mu;

static int dev_info(DevInfo** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64) { last_cuda_error_slot() = (int)e; return RVQ_ERR_UNAVAILABLE; }
    std::lock_guard<std::mutex> lock(g_mu);
    DevInfo& d = g_dev[dev];
    if (!d.ready) {
        d.ready = true;
        cudaDeviceProp prop;
        e = cudaGetDeviceProperties(&prop, dev);
        if (e == cudaSuccess && prop.major == 10) {
            d.sms = prop.multiProcessorCount;
            e = cudaFuncSetAttribute(rvq_gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kLutBytes);
            d.ok = e == cudaSuccess;
        }
        if (e != cudaSuccess) last_cuda_error_slot() = (int)e;
    }
    if (!d.ok) return RVQ_ERR_UNAVAILABLE;
    *out = &d;
    return RVQ_OK;
}

static size_t align256(size_t n) { return (n + 255) & ~(size_t)255; }

static int check_job(const rvq_gemv_job* g) {
    const rvq_entry& w = g->weight;
    int rc = rvq_check_entry(&w);
    if (rc != RVQ_OK) return rc;
    if (w.stages != kStages || w.ncodes != kCodes || w.index_kind != RVQ_U8) return RVQ_ERR_UNSUPPORTED;
    if (g->rows < 1 || g->cols < 8 || g->cols % 8) return RVQ_ERR_UNSUPPORTED;
    if (g->rows * g->cols / 8 != w.nvec || w.trimmed != w.nvec * 8 || w.tail_numel != 0) return RVQ_ERR_UNSUPPORTED;
    if (g->codes_interleaved && ((uintptr_t)w.indices & 3)) return RVQ_ERR_INVALID;
    if (g->rows >= (1ll << 31) || g->cols / 8 >= (1ll << 24)) return RVQ_ERR_TOO_LARGE;
    if (!g->x || !g->y) return RVQ_ERR_INVALID;
    if (g->x_kind != RVQ_BF16 && g->x_kind != RVQ_F16 && g->x_kind != RVQ_F32) return RVQ_ERR_UNSUPPORTED;
    if (g->y_kind != RVQ_BF16 && g->y_kind != RVQ_F16 && g->y_kind != RVQ_F32) return RVQ_ERR_UNSUPPORTED;
    return RVQ_OK;
}

// CTAs per job: tiles x row ranges.  One CTA fits per SM (128 KB of shared
// memory), so the launch is kept to one wave: every job gets row ranges in
// proportion to its vectors, rounded down, at least one, and what is left of
// the wave goes to the jobs with the most rows per CTA.
static void plan(const rvq_gemv_job* jobs, int n, int sms, uint32_t* ntiles, uint32_t* nranges) {
    double total = 0;
    for (int i = 0; i < n; ++i) {
        total += (double)jobs[i].rows * (jobs[i].cols / 8);
        ntiles[i] = (uint32_t)((jobs[i].cols / 8 + kGroupsPerTile - 1) / kGroupsPerTile);
    }
    uint32_t used = 0;
    for (int i = 0; i < n; ++i) {
        const double share = sms * ((double)jobs[i].rows * (jobs[i].cols / 8) / total);
        uint32_t r = (uint32_t)(share / ntiles[i]);
        if (r < 1) r = 1;
        const uint32_t max_r = (uint32_t)((jobs[i].rows + kRowBatch - 1) / kRowBatch);
        if (r > max_r) r = max_r;
        nranges[i] = r;
        used += r * ntiles[i];
    }
    while (used < (uint32_t)sms) {
        int best = -1;
        double worst = 0;
        for (int i = 0; i < n; ++i) {
            const double per = (double)jobs[i].rows / nranges[i];
            if (used + ntiles[i] <= (uint32_t)sms && per > worst && per > 2 * kRowBatch) { worst = per; best = i; }
        }
        if (best < 0) break;
        ++nranges[best];
        used += ntiles[best];
    }
}

struct Layout {
    size_t tickets[kMaxJobs], partial[kMaxJobs], lut[kMaxJobs], total;
};

static Layout workspace_layout(const rvq_gemv_job* jobs, int n, const uint32_t* ntiles, const uint32_t* nranges) {
    Layout L;
    size_t off = 0;
    for (int i = 0; i < n; ++i) { L.tickets[i] = off; off = align256(off + nranges[i] * sizeof(unsigned int)); }
    for (int i = 0; i < n; ++i) { L.partial[i] = off; off = align256(off + (size_t)ntiles[i] * jobs[i].rows * 4); }
    for (int i = 0; i < n; ++i) { L.lut[i] = off; off = align256(off + (size_t)ntiles[i] * kLutBytes); }
    L.total = off;
    return L;
}

// Scratch for rvq_gemv_noalloc: a fixed array in the module's device memory,
// so that entry point never asks the CUDA allocator (or any other) for
// memory.  Every device that loads this library holds it until exit.
constexpr size_t kStaticScratchBytes = (size_t)8 << 20;          // 8 MiB
static __device__ __align__(256) unsigned char g_gemv_scratch[kStaticScratchBytes];

static void* g_scratch_addr[64];
static bool g_scratch_ready[64];

// Device address of g_gemv_scratch on the current device.  Host code may not
// use the array's name as a device pointer (it names a host-side stand-in),
// so the address is asked from the runtime once per device, with that device
// current, and kept.
static int static_scratch(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64) { last_cuda_error_slot() = (int)e; return RVQ_ERR_UNAVAILABLE; }
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_ready[dev]) {
        void* ptr = nullptr;
        e = cudaGetSymbolAddress(&ptr, g_gemv_scratch);
        if (e != cudaSuccess || !ptr) { last_cuda_error_slot() = (int)e; return RVQ_ERR_CUDA; }
        g_scratch_addr[dev] = ptr;
        g_scratch_ready[dev] = true;
    }
    *out = g_scratch_addr[dev];
    return RVQ_OK;
}

}  // namespace gemv
}  // namespace rvq

using namespace rvq;
using namespace rvq::gemv;

extern "C" {

size_t rvq_gemv_workspace_size(const rvq_gemv_job* jobs, int n_jobs) {
    if (n_jobs < 1 || n_jobs > kMaxJobs || !jobs) return 0;
    DevInfo* d = nullptr;
    int sms = dev_info(&d) == RVQ_OK ? d->sms : 148;
    uint32_t nt[kMaxJobs], nr[kMaxJobs];
    plan(jobs, n_jobs, sms, nt, nr);
    return workspace_layout(jobs, n_jobs, nt, nr).total;
}

int rvq_gemv(const rvq_gemv_job* jobs, int n_jobs, void* workspace, size_t workspace_bytes, void* stream) {
    if (n_jobs < 1 || n_jobs > kMaxJobs || !jobs) return RVQ_ERR_INVALID;
    for (int i = 0; i < n_jobs; ++i) {
        int rc = check_job(&jobs[i]);
        if (rc != RVQ_OK) return rc;
    }
    DevInfo* d = nullptr;
    int rc = dev_info(&d);
    if (rc != RVQ_OK) return rc;
    uint32_t nt[kMaxJobs], nr[kMaxJobs];
    plan(jobs, n_jobs, d->sms, nt, nr);
    const Layout L = workspace_layout(jobs, n_jobs, nt, nr);
    if (!workspace || workspace_bytes < L.total || ((uintptr_t)workspace & 255)) return RVQ_ERR_INVALID;
    Params p;
    memset(&p, 0, sizeof(p));
    p.njobs = n_jobs;
    uint32_t ctas = 0, lut_ctas = 0;
    char* ws = reinterpret_cast<char*>(workspace);
    for (int i = 0; i < n_jobs; ++i) {
        const rvq_gemv_job& g = jobs[i];
        Job& j = p.jobs[i];
        j.idx = reinterpret_cast<const uint8_t*>(g.weight.indices);
        j.cb = g.weight.codebook;
        j.scales = g.weight.scales;
        j.x = g.x;
        j.y = g.y;
        j.partial = reinterpret_cast<float*>(ws + L.partial[i]);
        j.tickets = reinterpret_cast<unsigned int*>(ws + L.tickets[i]);
        j.lut = reinterpret_cast<float*>(ws + L.lut[i]);
        j.rows = (uint32_t)g.rows;
        j.groups = (uint32_t)(g.cols / 8);
        j.stage_stride = (uint32_t)g.weight.stage_stride;
        j.gv = make_fastdiv((uint32_t)g.weight.group_vecs);
        j.ntiles = nt[i];
        j.nranges = nr[i];
        j.cta_begin = ctas;
        j.lut_cta_begin = lut_ctas;
        j.cb_kind = (uint8_t)g.weight.codebook_kind;
        j.scale_kind = (uint8_t)g.weight.scale_kind;
        j.x_kind = (uint8_t)g.x_kind;
        j.y_kind = (uint8_t)g.y_kind;
        j.row_scales = (uint64_t)g.weight.group_vecs == (uint64_t)(g.cols / 8);
        j.interleaved = g.codes_interleaved ? 1 : 0;
        ctas += nt[i] * nr[i];
        lut_ctas += nt[i] * kStages;
    }
    rvq_lut_kernel<<<lut_ctas, kLutThreads, 0, (cudaStream_t)stream>>>(p);
    rvq_gemv_kernel<<<ctas, kThreads, kLutBytes, (cudaStream_t)stream>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { last_cuda_error_slot() = (int)e; return RVQ_ERR_CUDA; }
    return RVQ_OK;
}

size_t rvq_gemv_noalloc_max_workspace(void) { return kStaticScratchBytes; }

int rvq_gemv_noalloc(const rvq_gemv_job* jobs, int n_jobs, void* stream) {
    if (n_jobs < 1 || n_jobs > kMaxJobs || !jobs) return RVQ_ERR_INVALID;
    for (int i = 0; i < n_jobs; ++i) {
        int rc = check_job(&jobs[i]);
        if (rc != RVQ_OK) return rc;
    }
    DevInfo* d = nullptr;
    int rc = dev_info(&d);
    if (rc != RVQ_OK) return rc;
    uint32_t nt[kMaxJobs], nr[kMaxJobs];
    plan(jobs, n_jobs, d->sms, nt, nr);
    const Layout L = workspace_layout(jobs, n_jobs, nt, nr);
    if (L.total > kStaticScratchBytes) return RVQ_ERR_TOO_LARGE;
    void* ws = nullptr;
    rc = static_scratch(&ws);
    if (rc != RVQ_OK) return rc;
    // the row-range tickets come first in the layout and must start at zero;
    // the previous call's tables and partials are overwritten before use
    cudaError_t e = cudaMemsetAsync(ws, 0, L.partial[0], (cudaStream_t)stream);
    if (e != cudaSuccess) { last_cuda_error_slot() = (int)e; return RVQ_ERR_CUDA; }
    return rvq_gemv(jobs, n_jobs, ws, kStaticScratchBytes, stream);
}

int rvq_interleave_codes(const void* planes, int64_t stage_stride, int64_t nvec, void* out, void* stream) {
    if (!planes || !out || nvec < 0 || stage_stride < nvec || ((uintptr_t)out & 3)) return RVQ_ERR_INVALID;
    if (nvec == 0) return RVQ_OK;
    DevInfo* d = nullptr;
    int rc = dev_info(&d);
    if (rc != RVQ_OK) return rc;
    const uint64_t blocks = ((uint64_t)nvec + 255) / 256;
    const unsigned grid = (unsigned)(blocks < (uint64_t)d->sms * 16 ? blocks : (uint64_t)d->sms * 16);
    rvq_interleave_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<const uint8_t*>(planes), (uint64_t)stage_stride, (uint64_t)nvec, reinterpret_cast<uint32_t*>(out));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { last_cuda_error_slot() = (int)e; return RVQ_ERR_CUDA; }
    return RVQ_OK;
}

}  // extern "C"
