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
#include "rvq_tiles.cuh"
#include "rvq_vecdecode.cuh"

namespace rvq {
namespace tiles {

__global__ void __launch_bounds__(kThreads, 1) rvq_gemv_tiles_kernel(const __grid_constant__ TParams p) {
    extern __shared__ __align__(128) float smem[];
    __shared__ int slot_done[kRing];
    __shared__ float xmax[kTileCols / 32];
    __shared__ volatile int aborted;
    const TileSmem S = tile_smem(smem, slot_done, xmax, &aborted);
    pdl_launch_dependents();
    tile_smem_init(S);
    UnitState st;
    const int u_first = p.cta_first[blockIdx.x], u_last = p.cta_first[blockIdx.x + 1];
    for (int u = u_first; u < u_last; ++u) {
        const uint32_t jt = p.unit_jt[u];
        const TJob& J = p.jobs[jt >> 24];
        const int tile = (int)(jt & 0xffffffu);
        if (u != u_first) __syncthreads();              // the previous unit is done with shared memory
        run_unit(J, tile, p.unit_r0[u], p.unit_r1[u], S, st, true, [&] {
            if (u == u_first) pdl_wait();                // x comes from the previous kernel
            stage_operand(J, tile, S);
        });
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
    for (int i = 0; i < n_jobs; ++i) p.jobs[i] = make_tjob(jobs[i]);
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
