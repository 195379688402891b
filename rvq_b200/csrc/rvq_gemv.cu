// Fused RVQ dequant-GEMV for batch-1 decode (sm_100a): y = W x without
// materialising W.
//
// W is an RVQ entry (K=4 stages x 256 codes, d=8, uint8 codes; any scale
// grouping).  Per column group j (8 columns) and stage k the kernel builds a
// lookup table LUT_k[c][j] = dot(cb_k[c], x[8j .. 8j+8]) in shared memory, so
// an 8-weight vector costs 4 table lookups and 3 adds instead of 32 codebook
// element reconstructions:
//
//   y[r] = sum_j  scale(r, j) * (((LUT_0[c0] + LUT_1[c1]) + LUT_2[c2]) + LUT_3[c3])
//
// This is the exact sum of W[r, :] x in real arithmetic; in floating point it
// differs from "reconstruct W, round it to bf16, then matmul" by the bf16
// rounding of each weight (relative 2^-9 per weight), which is why this path
// is compared against the reference reconstruct + matmul with a tolerance.
//
// Work split: column tiles of 32 groups (256 columns) x row ranges.  A CTA
// builds the 128 KB table of its tile (lane j of every warp owns group j, so
// table reads are conflict-free), then each warp takes rows, reads the 4 code
// bytes of its lane's group (32 consecutive bytes per plane per warp) and
// reduces the row over the 32 lanes with shuffles.  Per-tile row partials go
// to a workspace; the last CTA of a row range (atomic ticket) sums the tiles
// in tile order, so results are deterministic run to run.

#include <string.h>

#include <mutex>

#include "rvq_common.cuh"

namespace rvq {
namespace gemv {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr int kGroupsPerTile = 32;               // 256 columns per tile
constexpr int kStages = 4;
constexpr int kCodes = 256;
constexpr int kRowBatch = 8;                     // rows a warp decodes and reduces together
constexpr int kMaxJobs = 16;
constexpr size_t kLutBytes = (size_t)kStages * kCodes * kGroupsPerTile * sizeof(float);   // 128 KB
constexpr size_t kCbBytes = (size_t)kStages * kCodes * 8 * sizeof(float);                  // 32 KB
constexpr size_t kSmemBytes = kLutBytes + kCbBytes;                                        // 160 KB

struct Job {
    const uint8_t* idx;        // [4][stage_stride] codes
    const void* cb;            // [4][256][8] fp16 or fp32
    const void* scales;        // scale per group_vecs vectors
    const void* x;             // [cols]
    void* y;                   // [rows]
    float* partial;            // [ntiles][rows] workspace
    unsigned int* tickets;     // [nranges] workspace, zero between launches
    uint32_t rows;
    uint32_t groups;           // cols / 8
    uint32_t stage_stride;
    FastDiv gv;                // group_vecs
    uint32_t ntiles;           // ceil(groups / 32)
    uint32_t nranges;          // row ranges per tile
    uint32_t cta_begin;        // first CTA of this job
    uint8_t cb_kind, scale_kind, x_kind, y_kind;
    uint8_t row_scales;        // one scale per row: applied once, after the tile sum
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

// d += a * b on two fp32 lanes at once (sm_100 packed fp32 FMA).
__device__ __forceinline__ void fma2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
    asm("{.reg .b64 ra, rb, rd; mov.b64 ra, {%2,%3}; mov.b64 rb, {%4,%5}; mov.b64 rd, {%0,%1};"
        " fma.rn.f32x2 rd, ra, rb, rd; mov.b64 {%0,%1}, rd;}"
        : "+f"(d0), "+f"(d1) : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

// Code words of 4 consecutive rows, one plane: lanes 8q..8q+7 read row rb+q,
// lane L reads groups 4(L%8)..4(L%8)+3 of the tile (a 32-byte row segment per
// 8 lanes).  `valid` masks rows past the range and groups past the matrix.
__device__ __forceinline__ uint32_t load_quad(const Job& job, int k, uint32_t rb, uint32_t r1, uint32_t g0,
                                              int lane) {
    const uint32_t row = rb + (lane >> 3);
    const uint32_t grp = g0 + 4 * (lane & 7);
    if (row >= r1 || grp >= job.groups) return 0u;
    const uint8_t* src = job.idx + (size_t)k * job.stage_stride + (size_t)row * job.groups + grp;
    return __ldg(reinterpret_cast<const uint32_t*>(src));
}

__global__ void __launch_bounds__(kThreads, 1) rvq_gemv_kernel(const __grid_constant__ Params p) {
    extern __shared__ __align__(16) unsigned char smem[];
    float* lut = reinterpret_cast<float*>(smem);                         // [4][256][32]
    float* cbs = reinterpret_cast<float*>(smem + kLutBytes);             // [4][256][8]
    __shared__ int s_last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int ji = 0;
    while (ji + 1 < p.njobs && blockIdx.x >= p.jobs[ji + 1].cta_begin) ++ji;
    const Job& job = p.jobs[ji];
    const uint32_t local = blockIdx.x - job.cta_begin;
    const uint32_t tile = local / job.nranges, range = local % job.nranges;
    const uint32_t g0 = tile * kGroupsPerTile;
    const uint32_t j = g0 + lane;                       // this lane's column group
    const bool active = j < job.groups;
    const uint32_t r0 = (uint32_t)(((uint64_t)job.rows * range) / job.nranges);
    const uint32_t r1 = (uint32_t)(((uint64_t)job.rows * (range + 1)) / job.nranges);

    // ---- codebook (fp32) and this lane's 8 activations first ----
    for (int e = threadIdx.x; e < kStages * kCodes * 2; e += kThreads) {
        float4 v;
        if (job.cb_kind == RVQ_F32) {
            v = __ldg(reinterpret_cast<const float4*>(job.cb) + e);
        } else {
            const uint2 h = __ldg(reinterpret_cast<const uint2*>(job.cb) + e);
            v.x = __half2float(__ushort_as_half((uint16_t)(h.x & 0xFFFFu)));
            v.y = __half2float(__ushort_as_half((uint16_t)(h.x >> 16)));
            v.z = __half2float(__ushort_as_half((uint16_t)(h.y & 0xFFFFu)));
            v.w = __half2float(__ushort_as_half((uint16_t)(h.y >> 16)));
        }
        reinterpret_cast<float4*>(cbs)[e] = v;
    }
    float xs[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) xs[t] = active ? ldf(job.x, j * 8 + t, job.x_kind) : 0.0f;

    // first batch of code words in flight while the table is built
    uint32_t rb = r0 + warp * kRowBatch;
    uint32_t w[kStages][2];
#pragma unroll
    for (int k = 0; k < kStages; ++k) {
        w[k][0] = load_quad(job, k, rb, r1, g0, lane);
        w[k][1] = load_quad(job, k, rb + 4, r1, g0, lane);
    }
    __syncthreads();

    // ---- table of this tile: LUT[k][c][lane] = dot(cb[k][c], x[8j..8j+8]) ----
    for (int e = warp; e < kStages * kCodes; e += 2 * kWarps) {
        const float4* c0 = reinterpret_cast<const float4*>(cbs) + 2 * e;
        const float4* c1 = c0 + 2 * kWarps;
        const float4 a0 = c0[0], b0 = c0[1], a1 = c1[0], b1 = c1[1];
        float d0 = 0.0f, d0b = 0.0f, d1 = 0.0f, d1b = 0.0f;
        fma2(d0, d0b, a0.x, a0.y, xs[0], xs[1]);
        fma2(d1, d1b, a1.x, a1.y, xs[0], xs[1]);
        fma2(d0, d0b, a0.z, a0.w, xs[2], xs[3]);
        fma2(d1, d1b, a1.z, a1.w, xs[2], xs[3]);
        fma2(d0, d0b, b0.x, b0.y, xs[4], xs[5]);
        fma2(d1, d1b, b1.x, b1.y, xs[4], xs[5]);
        fma2(d0, d0b, b0.z, b0.w, xs[6], xs[7]);
        fma2(d1, d1b, b1.z, b1.w, xs[6], xs[7]);
        lut[e * kGroupsPerTile + lane] = d0 + d0b;
        lut[(e + kWarps) * kGroupsPerTile + lane] = d1 + d1b;
    }
    __syncthreads();                                    // table ready

    // ---- rows: 8 per warp per step, next step's code words prefetched ----
    const uint32_t G = job.groups;
    float* part = job.partial + (size_t)tile * job.rows;
    const uint32_t bsel = 0x4440u | (lane & 3);
    bool wrote = false;
    for (; rb < r1; rb += kWarps * kRowBatch) {
        uint32_t wn[kStages][2];
        const uint32_t nb = rb + kWarps * kRowBatch;
#pragma unroll
        for (int k = 0; k < kStages; ++k) {
            wn[k][0] = load_quad(job, k, nb, r1, g0, lane);
            wn[k][1] = load_quad(job, k, nb + 4, r1, g0, lane);
        }
        float v[kRowBatch];
#pragma unroll
        for (int i = 0; i < kRowBatch; ++i) {
            const int src = (i & 3) * 8 + (lane >> 2);  // lane holding this row's word for my group
            float a = lut[(0 * kCodes + __byte_perm(__shfl_sync(0xffffffffu, w[0][i >> 2], src), 0, bsel)) * kGroupsPerTile + lane];
            a += lut[(1 * kCodes + __byte_perm(__shfl_sync(0xffffffffu, w[1][i >> 2], src), 0, bsel)) * kGroupsPerTile + lane];
            a += lut[(2 * kCodes + __byte_perm(__shfl_sync(0xffffffffu, w[2][i >> 2], src), 0, bsel)) * kGroupsPerTile + lane];
            a += lut[(3 * kCodes + __byte_perm(__shfl_sync(0xffffffffu, w[3][i >> 2], src), 0, bsel)) * kGroupsPerTile + lane];
            const uint32_t row = rb + i;
            if (!job.row_scales)
                a *= (active && row < r1) ? ldf(job.scales, fastdiv(row * G + j, job.gv), job.scale_kind) : 0.0f;
            v[i] = (active && row < r1) ? a : 0.0f;
        }
        // transpose-reduce 8 rows over 32 lanes: lanes 4m..4m+3 end with row m
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
        {
            const bool up = lane & 4;
            const float send = up ? v[0] : v[1], keep = up ? v[1] : v[0];
            v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
        }
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], 2);
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
        const uint32_t row = rb + ((lane >> 2) & 7);
        if ((lane & 3) == 0 && row < r1) {
            part[row] = v[0];
            wrote = true;
        }
#pragma unroll
        for (int k = 0; k < kStages; ++k) {
            w[k][0] = wn[k][0];
            w[k][1] = wn[k][1];
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
            e = cudaFuncSetAttribute(rvq_gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
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
    // code words are read 4 bytes at a time: 4-byte aligned planes and rows
    if ((g->cols / 8) % 4 || w.stage_stride % 4 || ((uintptr_t)w.indices & 3)) return RVQ_ERR_UNSUPPORTED;
    if (g->rows >= (1ll << 31) || g->cols / 8 >= (1ll << 24)) return RVQ_ERR_TOO_LARGE;
    if (!g->x || !g->y) return RVQ_ERR_INVALID;
    if (g->x_kind != RVQ_BF16 && g->x_kind != RVQ_F16 && g->x_kind != RVQ_F32) return RVQ_ERR_UNSUPPORTED;
    if (g->y_kind != RVQ_BF16 && g->y_kind != RVQ_F16 && g->y_kind != RVQ_F32) return RVQ_ERR_UNSUPPORTED;
    return RVQ_OK;
}

// CTAs per job: tiles x row ranges.  One CTA fits per SM (192 KB of shared
// memory), so the launch is kept to one wave: every job gets row ranges in
// proportion to its vectors, rounded down, at least one, and the total never
// exceeds the SM count unless the tiles alone do.
static void plan(const rvq_gemv_job* jobs, int n, int sms, uint32_t* ntiles, uint32_t* nranges) {
    double total = 0;
    uint32_t tiles_total = 0;
    for (int i = 0; i < n; ++i) {
        total += (double)jobs[i].rows * (jobs[i].cols / 8);
        ntiles[i] = (uint32_t)((jobs[i].cols / 8 + kGroupsPerTile - 1) / kGroupsPerTile);
        tiles_total += ntiles[i];
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
    // spend what is left of the wave on the jobs with the most rows per CTA
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
    (void)tiles_total;
}

static size_t workspace_layout(const rvq_gemv_job* jobs, int n, const uint32_t* ntiles, const uint32_t* nranges,
                               size_t* ticket_off, size_t* partial_off) {
    size_t off = 0;
    for (int i = 0; i < n; ++i) { ticket_off[i] = off; off = align256(off + nranges[i] * sizeof(unsigned int)); }
    for (int i = 0; i < n; ++i) { partial_off[i] = off; off = align256(off + (size_t)ntiles[i] * jobs[i].rows * 4); }
    return off;
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
    size_t to[kMaxJobs], po[kMaxJobs];
    plan(jobs, n_jobs, sms, nt, nr);
    return workspace_layout(jobs, n_jobs, nt, nr, to, po);
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
    size_t to[kMaxJobs], po[kMaxJobs];
    plan(jobs, n_jobs, d->sms, nt, nr);
    const size_t need = workspace_layout(jobs, n_jobs, nt, nr, to, po);
    if (!workspace || workspace_bytes < need || ((uintptr_t)workspace & 255)) return RVQ_ERR_INVALID;
    Params p;
    memset(&p, 0, sizeof(p));
    p.njobs = n_jobs;
    uint32_t ctas = 0;
    for (int i = 0; i < n_jobs; ++i) {
        const rvq_gemv_job& g = jobs[i];
        Job& j = p.jobs[i];
        j.idx = reinterpret_cast<const uint8_t*>(g.weight.indices);
        j.cb = g.weight.codebook;
        j.scales = g.weight.scales;
        j.x = g.x;
        j.y = g.y;
        j.partial = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + po[i]);
        j.tickets = reinterpret_cast<unsigned int*>(reinterpret_cast<char*>(workspace) + to[i]);
        j.rows = (uint32_t)g.rows;
        j.groups = (uint32_t)(g.cols / 8);
        j.stage_stride = (uint32_t)g.weight.stage_stride;
        j.gv = make_fastdiv((uint32_t)g.weight.group_vecs);
        j.ntiles = nt[i];
        j.nranges = nr[i];
        j.cta_begin = ctas;
        j.cb_kind = (uint8_t)g.weight.codebook_kind;
        j.scale_kind = (uint8_t)g.weight.scale_kind;
        j.x_kind = (uint8_t)g.x_kind;
        j.y_kind = (uint8_t)g.y_kind;
        j.row_scales = (uint64_t)g.weight.group_vecs == (uint64_t)(g.cols / 8);
        ctas += nt[i] * nr[i];
    }
    rvq_gemv_kernel<<<ctas, kThreads, kSmemBytes, (cudaStream_t)stream>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { last_cuda_error_slot() = (int)e; return RVQ_ERR_CUDA; }
    return RVQ_OK;
}

}  // extern "C"
