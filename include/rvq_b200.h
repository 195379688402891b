/*
 * rvq_b200 -- C ABI of the B200 (sm_100a) RVQ weight-reconstruction kernels.
 *
 * Plain pointers and sizes only: no torch or CUDA types in the signatures.
 * Every pointer named "device" below is CUDA device memory on the device that
 * is current for the calling thread; `stream` is a cudaStream_t of that
 * device (NULL = legacy default stream).  Calls are asynchronous on `stream`:
 * nothing here synchronises the device.
 *
 * Entry format: one "entry" is one RVQ-compressed tensor as written by the
 * reference compressor (compress_full_model.py:375-388): `indices` [K, nvec]
 * (uint8 when the codebook has <= 256 codes, else int16), a codebook
 * [K, ncodes, d] (fp16 in the artifact, fp32 after the engine's upload,
 * infer_compressed_layerwise_triton.py:424-427), one scale per `group_size`
 * flattened elements (fp16) and a bf16 `tail`.  Only d == 8 is supported, as
 * in the reference kernel (triton_decode_kernels.py:126-127).
 *
 * Results are bit-identical to the reference's reconstruction:
 *   out[8n+t] = cast( float(scale[n / group_vecs]) * (((0 + cb0) + cb1) + ...) )
 * with fp32 accumulation in stage order and round-to-nearest-even casts.
 */
#ifndef RVQ_B200_H
#define RVQ_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  The Python layer maps them onto the reference's exceptions
 * (triton_decode_kernels.py:119-165): RVQ_ERR_UNAVAILABLE -> RuntimeError,
 * RVQ_ERR_UNSUPPORTED -> NotImplementedError, RVQ_ERR_INVALID -> ValueError. */
enum rvq_status {
    RVQ_OK = 0,
    RVQ_ERR_INVALID = 1,      /* bad argument (null pointer, bad size, misuse) */
    RVQ_ERR_UNSUPPORTED = 2,  /* valid input this build does not handle (d != 8, dtype) */
    RVQ_ERR_UNAVAILABLE = 3,  /* no usable CUDA device / not an sm_100 device */
    RVQ_ERR_CUDA = 4,         /* a CUDA runtime call failed; see rvq_last_cuda_error() */
    RVQ_ERR_TOO_LARGE = 5     /* a size exceeds a documented limit */
};

/* Element kinds.  The output kinds keep the reference's OUT_KIND numbering
 * (triton_decode_kernels.py:158-165). */
enum rvq_kind {
    RVQ_F16 = 0,
    RVQ_BF16 = 1,
    RVQ_F32 = 2,
    RVQ_U8 = 3,
    RVQ_I16 = 4,
    /* uint8 codes of exactly 4 stages in the "quad" layout this library
     * writes with rvq_quad_codes: 16 bytes per 4 consecutive vectors, byte
     * 4 k + j = the stage-k code of vector 4 q + j.  Not an artifact layout. */
    RVQ_U8X4 = 5
};

/* One RVQ entry to decode.  Replaces the arguments that
 * decode_rvq_triton_into (triton_decode_kernels.py:114-185) passes to
 * _rvq_decode_into_kernel plus the tail copy of lines 187-188. */
typedef struct rvq_entry {
    const void* indices;      /* device, [stages][stage_stride], index_kind elements */
    const void* codebook;     /* device, [stages][ncodes][8] contiguous, codebook_kind */
    const void* scales;       /* device, ceil(nvec / group_vecs) values, scale_kind */
    const void* tail;         /* device, tail_numel values of tail_kind (may be NULL if 0) */
    void* out;                /* device, >= trimmed + tail_numel elements of out_kind */
    int64_t nvec;             /* vectors of d = 8 elements (indices.shape[1]) */
    int64_t stage_stride;     /* elements between index planes (indices.stride(0)) */
    int64_t group_vecs;       /* group_size / d: vectors sharing one scale */
    int64_t trimmed;          /* trimmed_numel: core elements written (masked) */
    int64_t tail_numel;       /* tail elements copied to out[trimmed ...] */
    int32_t stages;           /* K >= 1 */
    int32_t ncodes;           /* codebook entries per stage */
    int32_t d;                /* must be 8 */
    int32_t index_kind;       /* RVQ_U8 or RVQ_I16 */
    int32_t codebook_kind;    /* RVQ_F16 or RVQ_F32 */
    int32_t scale_kind;       /* RVQ_F16, RVQ_BF16 or RVQ_F32 */
    int32_t tail_kind;        /* RVQ_F16, RVQ_BF16 or RVQ_F32 */
    int32_t out_kind;         /* RVQ_F16, RVQ_BF16 or RVQ_F32 */
} rvq_entry;

/* A raw device-to-device copy of a `bf16_raw` entry (a 1-D norm weight),
 * the int16 view copy of infer_compressed_layerwise_triton.py:165-167. */
typedef struct rvq_copy {
    const void* src;          /* device */
    void* dst;                /* device */
    int64_t nbytes;
} rvq_copy;

/* One int8_groupwise entry (compress_full_model.py:391-425, the artifact's
 * other method): out[i] = cast(float(q[i]) * float(scale[i / group_size])) for
 * i < trimmed, then the tail.  Replaces _decode_int8_into
 * (infer_compressed_layerwise_single_slot.py:110-120), which the single-slot
 * engine calls from _decode_entry_into (lines 155-157). */
typedef struct rvq_int8_entry {
    const void* q;            /* device int8, trimmed values (the artifact's q [groups][group_size]) */
    const void* scales;       /* device, trimmed / group_size values of scale_kind */
    const void* tail;         /* device, tail_numel values of tail_kind (may be NULL if 0) */
    void* out;                /* device, >= trimmed + tail_numel elements of out_kind */
    int64_t trimmed;          /* trimmed_numel, a multiple of group_size */
    int64_t group_size;
    int64_t tail_numel;
    int32_t scale_kind;       /* RVQ_F16, RVQ_BF16 or RVQ_F32 */
    int32_t tail_kind;        /* RVQ_F16, RVQ_BF16 or RVQ_F32 */
    int32_t out_kind;         /* RVQ_F16, RVQ_BF16 or RVQ_F32 */
    int32_t reserved;
} rvq_int8_entry;

/* Maximum entries + copies one rvq_decode_layer call takes. */
#define RVQ_MAX_LAYER_JOBS 32

/* 1 when a device with compute capability 10.x is current and the kernels
 * of this library load on it, else 0.  Replaces triton_available()
 * (triton_decode_kernels.py:31-32). */
int rvq_available(void);

/* RVQ_OK when rvq_decode would accept `e`, else the status it would return.
 * Host-only check: reads no device memory.  Replaces rvq_triton_supported
 * (triton_decode_kernels.py:35-44) plus the argument checks of
 * decode_rvq_triton_into (lines 122-165). */
int rvq_check_entry(const rvq_entry* e);

/* Decode one entry into e->out, then copy its tail.  Replaces
 * decode_rvq_triton_into (triton_decode_kernels.py:114-190): one kernel
 * launch on `stream`, no allocation, no synchronisation. */
int rvq_decode(const rvq_entry* e, void* stream);

/* Decode a whole layer slot in ONE launch: `n_entries` RVQ entries and
 * `n_copies` raw copies (n_entries + n_copies <= RVQ_MAX_LAYER_JOBS).
 * Replaces the per-key decode_into loop of prefetch_layer
 * (infer_compressed_layerwise_triton.py:246-266) and the per-key
 * _decode_entry_into calls of SlotResidency._decode_layer_async
 * (infer_compressed_layerwise_single_slot.py:652-668). */
int rvq_decode_layer(const rvq_entry* entries, int n_entries, const rvq_copy* copies,
                     int n_copies, void* stream);

/* RVQ_OK when rvq_decode_int8 would accept `e`, else its status (host-only). */
int rvq_check_int8_entry(const rvq_int8_entry* e);

/* Decode one int8_groupwise entry (one launch, no allocation, no sync). */
int rvq_decode_int8(const rvq_int8_entry* e, void* stream);

/* rvq_decode_layer for a layer that also holds int8_groupwise entries:
 * n_entries + n_int8 + n_copies <= RVQ_MAX_LAYER_JOBS, one launch. */
int rvq_decode_layer_mixed(const rvq_entry* entries, int n_entries, const rvq_int8_entry* int8s,
                           int n_int8, const rvq_copy* copies, int n_copies, void* stream);

/* rvq_decode_layer_mixed on at most `max_ctas` CTAs (0: one per SM; each
 * CTA takes a whole SM).  A decode on a side stream that leaves SMs free lets
 * the kernels of the layer being computed on the main stream run beside it
 * (the ping-pong of infer_compressed_layerwise_triton.py:246-277) instead of
 * queueing behind it. */
int rvq_decode_layer_ctas(const rvq_entry* entries, int n_entries, const rvq_int8_entry* int8s,
                          int n_int8, const rvq_copy* copies, int n_copies, int max_ctas, void* stream);

/* One fused dequant-GEMV y = W x for a batch of one (no counterpart in the
 * reference, which reconstructs W into the slot and then calls F.linear:
 * infer_compressed_layerwise_triton.py:290-292 / lines 296-297).  W is an
 * RVQ entry with K=4 stages, 256 codes, uint8 codes, no tail; `rows` x `cols`
 * is its shape (cols a multiple of 8).  The product is computed through
 * per-stage lookup tables of codeword . x dot products, i.e. W is never
 * materialised and never rounded to bf16: results match "reconstruct, round
 * to bf16, matmul" to within the bf16 rounding of W (about 1e-3 relative). */
typedef struct rvq_gemv_job {
    rvq_entry weight;         /* the weight entry; weight.out is ignored */
    const void* x;            /* device, [cols] activations of x_kind */
    void* y;                  /* device, [rows] output of y_kind */
    int64_t rows;
    int64_t cols;
    int32_t x_kind;           /* RVQ_BF16, RVQ_F16 or RVQ_F32 */
    int32_t y_kind;           /* RVQ_BF16, RVQ_F16 or RVQ_F32 */
    int32_t codes_interleaved;/* 0: weight.indices are the artifact's planes [4][stage_stride];
                                 1: [nvec][4] bytes as written by rvq_interleave_codes */
    int32_t reserved;
} rvq_gemv_job;

/* Bytes of device workspace rvq_gemv needs for these jobs (lookup tables,
 * per-tile row partials and row-range tickets).  The workspace must be zero-filled once
 * when it is allocated; every launch leaves its tickets at zero again.
 * Launches that share a workspace must not overlap on the GPU. */
size_t rvq_gemv_workspace_size(const rvq_gemv_job* jobs, int n_jobs);

/* Up to 4 GEMVs (e.g. q, k and v of one layer, sharing x) in one launch.
 * Deterministic: partial sums over 256-column tiles are added in tile order.
 * `workspace` is 256-byte aligned device memory of at least
 * rvq_gemv_workspace_size() bytes. */
int rvq_gemv(const rvq_gemv_job* jobs, int n_jobs, void* workspace, size_t workspace_bytes, void* stream);

/* rvq_gemv without a caller-supplied workspace, for callers that cannot
 * allocate device memory: e.g. a serving process that reserves its whole
 * memory budget at start-up and forbids allocation afterwards, or a plug-in
 * running inside a host runtime that owns every device allocation.  No
 * counterpart in the reference.  The workspace is a fixed array of
 * rvq_gemv_noalloc_max_workspace() bytes (8 MiB) in this library's device
 * memory, held by every device that loads the library until exit; jobs whose
 * workspace would exceed it return RVQ_ERR_TOO_LARGE.  Nothing is allocated:
 * no cudaMalloc/cudaFree and no allocating library routine.  The first call
 * on a device looks up the array's device address (cudaGetSymbolAddress)
 * with that device current; make that first call before any stream capture.
 * All calls share the one array, which keeps the last call's contents (each
 * call clears the part that must start at zero), so calls that overlap on the
 * GPU -- concurrent streams, or several host threads -- race with each other
 * and must be serialised by the caller. */
int rvq_gemv_noalloc(const rvq_gemv_job* jobs, int n_jobs, void* stream);

/* Size of the fixed workspace rvq_gemv_noalloc uses. */
size_t rvq_gemv_noalloc_max_workspace(void);

/* Repack uint8 code planes [4][stage_stride] of `nvec` vectors into the quad
 * layout (index_kind RVQ_U8X4): out holds rvq_quad_codes_bytes(nvec) bytes
 * (whole 128-vector tiles), 16-byte aligned, zero past the last vector.  A decode thread then gets the 4 stage
 * codes of its 4 vectors with one 16-byte load instead of 4 plane loads (the
 * resident layout of layer plans; the artifact keeps its planes). */
int rvq_quad_codes(const void* planes, int64_t stage_stride, int64_t nvec, void* out, void* stream);
int64_t rvq_quad_codes_bytes(int64_t nvec);

/* Repack uint8 code planes [4][stage_stride] into one 32-bit word per vector
 * ([nvec][4] bytes, stage k in byte k), the layout rvq_gemv reads with one
 * load per vector (codes_interleaved = 1).  `out` holds nvec * 4 bytes,
 * 4-byte aligned.  A layout of this library, not of the reference artifact. */
int rvq_interleave_codes(const void* planes, int64_t stage_stride, int64_t nvec, void* out, void* stream);

/* ---- Batch-1 decode-step operations --------------------------------------
 * The reference runs each Qwen3 decoder layer through the HF module
 * (functional_call of Qwen3DecoderLayer, infer_compressed_layerwise_triton.py:
 * 279-294), i.e. dozens of small PyTorch kernels per layer.  These entry points
 * are that layer's non-GEMM work as a few launches, for a CUDA-graph-captured
 * batch-1 decode step; they have no counterpart entry point in the reference.
 * Every value is rounded to bf16 where the HF module rounds it (RMSNorm:
 * modeling_qwen3.Qwen3RMSNorm; attention: eager_attention_forward; MLP:
 * Qwen3MLP), so only fp32 summation order differs. */

/* A vector operand.  kind RVQ_BF16 / RVQ_F16: a plain [n] vector (ntiles 1).
 * kind RVQ_F32: fp32 partial sums [ntiles][n]; the operand is their sum in
 * tile order, rounded to bf16 (a projection's output). */
typedef struct rvq_vec {
    const void* ptr;          /* device */
    int64_t n;
    int32_t ntiles;
    int32_t kind;
} rvq_vec;

/* Residual add + RMSNorm of one token:
 *   h <- token ? embed[*token] : h + add      (bf16, in place)
 *   x <- weight * bf16(h * rsqrt(mean(h^2) + eps))   (bf16)
 * One launch of an 8-CTA cluster.  hidden <= 16384. */
typedef struct rvq_norm_args {
    void* h;                  /* device bf16 [hidden], the residual stream */
    rvq_vec add;              /* added to h first; add.ptr NULL: nothing added */
    const int64_t* token;     /* device; non-NULL: h = embed row *token (first layer) */
    const void* embed;        /* device bf16 [vocab][hidden], read when token is set */
    const void* weight;       /* device bf16 [hidden] */
    void* x;                  /* device bf16 [hidden] output */
    int64_t hidden;
    float eps;
    int32_t vocab;            /* rows of embed; a token outside [0, vocab) reads row 0 */
    /* Tensor-parallel landing buffer (rvq_tp_push): when `arrivals` is set, the
     * kernel first waits (bounded) until *arrivals has advanced by
     * arrivals_per_use past *consumed, reads `add` (the [tp][hidden] fp32
     * landing buffer, ntiles = tp) through L2, and then advances *consumed. */
    const uint32_t* arrivals; /* device; NULL: no wait */
    uint32_t* consumed;       /* device, this rank's count of arrivals already used */
    uint32_t arrivals_per_use;
    int32_t reserved;
} rvq_norm_args;

int rvq_step_norm(const rvq_norm_args* a, void* stream);

/* Attention of one new token at position *pos (device int64) for one layer:
 * per-head RMSNorm of q and k (q_norm / k_norm), rotary embedding with the
 * given cos / sin tables, append k and v to the cache at *pos, then for
 * every query head (GQA: head h reads kv head h / (n_heads / n_kv))
 *   s_j = bf16(bf16(bf16(q . k_j) * scaling) + valid_bias),  j = 0..*pos
 *   out = bf16(sum_j bf16(softmax(s)_j) * v_j).
 * valid_bias is 1.0 to reproduce the reference engine's all-ones additive mask,
 * 0.0 for the plain causal forward.  A cluster of 8 CTAs per kv head.
 * A position outside [0, max_len) touches no cache row and yields zeros.
 * head_dim 64, 128 or 256; n_heads / n_kv <= 16; *pos < max_len. */
typedef struct rvq_attn_args {
    rvq_vec q, k, v;          /* q [n_heads*head_dim], k and v [n_kv*head_dim] */
    const void* q_norm;       /* device bf16 [head_dim] */
    const void* k_norm;       /* device bf16 [head_dim] */
    const void* cos;          /* device bf16 [max_len][head_dim] */
    const void* sin;          /* device bf16 [max_len][head_dim] */
    const int64_t* pos;       /* device, one value */
    void* k_cache;            /* device bf16 [n_kv][max_len][head_dim], this layer */
    void* v_cache;            /* device bf16 [n_kv][max_len][head_dim] */
    void* out;                /* device bf16 [n_heads*head_dim] */
    int32_t n_heads;
    int32_t n_kv;
    int32_t head_dim;
    int32_t max_len;
    float eps;
    float scaling;
    float valid_bias;
    int32_t reserved;
} rvq_attn_args;

int rvq_step_attention(const rvq_attn_args* a, void* stream);

/* ---- Tensor parallelism over NVLink peer memory -----------------------------
 * The all-reduce after a row-parallel projection as one push kernel: each
 * rank sums its own projection output (fp32 partials [tiles][n] in tile order,
 * or a bf16 vector) and stores the fp32 result into slot [rank] of every
 * rank's landing buffer [tp][n] by plain peer stores over NVLink, then adds
 * rvq_tp_push_ctas(n) to every rank's arrival counter (system-scope release).
 * The consumer (rvq_step_norm with `arrivals` set) waits for all ranks and
 * sums the tp slots in rank order, so every rank computes the same bits.
 * Buffers and counters come from rvq_p2p_alloc on each rank and reach the
 * other ranks through rvq_ipc_export / rvq_ipc_import.  No counterpart in the
 * reference (it runs on one GPU). */
#define RVQ_MAX_TP 8

typedef struct rvq_tp_push_args {
    rvq_vec src;                      /* this rank's projection output, [n] */
    float* dst[RVQ_MAX_TP];           /* rank r's landing buffer [tp][n] (own rank: local pointer) */
    uint32_t* arrivals[RVQ_MAX_TP];   /* rank r's arrival counter */
    int64_t n;
    int32_t rank;
    int32_t tp;
} rvq_tp_push_args;

/* Arrivals one rank's push adds to every counter (its CTA count for n). */
uint32_t rvq_tp_push_ctas(int64_t n);
int rvq_tp_push(const rvq_tp_push_args* a, void* stream);

/* Zero-filled device memory for landing buffers and counters (cudaMalloc). */
int rvq_p2p_alloc(size_t bytes, void** out);
int rvq_p2p_free(void* ptr);
/* 64-byte IPC handle of an rvq_p2p_alloc allocation, and its mapping in
 * another process on the same node (peer access enabled). */
int rvq_ipc_export(void* ptr, void* handle64);
int rvq_ipc_import(const void* handle64, void** out);
int rvq_ipc_close(void* ptr);
/* Reads and clears the sticky flag set when a landing-buffer wait gave up. */
int rvq_take_tp_timeout(void);

/* out = bf16(bf16(silu(gate)) * up), [n] bf16 (Qwen3MLP's act_fn(gate) * up). */
int rvq_step_silu_mul(const rvq_vec* gate, const rvq_vec* up, void* out, void* stream);

/* Fused dequant-GEMV of a batch of one that leaves the cross-tile reduction to
 * its consumer: for every 256-column tile t of W,
 *   partials[t][r] = sum over the columns c of tile t of W[r][c] * x[c]
 * with W never materialised (per-tile tables of codeword . x products, 4
 * lookups per 8 weights).  The partials are an rvq_vec operand (kind RVQ_F32,
 * ntiles = rvq_gemv_tiles_count(cols)) of rvq_step_norm / rvq_step_attention
 * / rvq_step_silu_mul or of another rvq_gemv_tiles job, which add them in tile
 * order: deterministic, and no reduction launch or cross-CTA fence.
 * No counterpart in the reference (it reconstructs W into the slot and calls
 * F.linear: infer_compressed_layerwise_triton.py:290-292).
 * W: K=4, 256 codes, uint8 codes in the tile-major layout of rvq_tile_codes
 * (weight.indices, 16-byte aligned), no tail, d = 8, cols a multiple of 8;
 * codebook fp32 (16-byte aligned), fp16 or bf16. */
typedef struct rvq_gemv_tile_job {
    rvq_entry weight;         /* weight.out is ignored */
    rvq_vec x;                /* [cols] operand */
    rvq_vec gate;             /* gate.ptr non-NULL: the operand is bf16(bf16(silu(gate)) * x),
                                 Qwen3MLP's down-projection input */
    float* partials;          /* device, [rvq_gemv_tiles_count(cols)][rows] */
    int64_t rows;
    int64_t cols;
} rvq_gemv_tile_job;

/* Number of 256-column tiles (rows of the partials) for `cols` columns. */
int64_t rvq_gemv_tiles_count(int64_t cols);

/* Up to 4 jobs in one launch (e.g. q, k and v).  No workspace, no allocation. */
int rvq_gemv_tiles(const rvq_gemv_tile_job* jobs, int n_jobs, void* stream);

/* rvq_gemv_tiles with exact bf16 weights: every weight is rebuilt
 * bit-identically to rvq_decode's bf16 output (fp32 sum of the stage codewords
 * in stage order, times the fp32 scale, rounded to nearest even) and
 * multiplied by the bf16 operand in fp32, so the products are exactly those
 * that F.linear forms on the decoded slot (infer_compressed_layerwise_triton.py:
 * 290-292, cuBLAS on bf16 weights) and only the fp32 summation order differs.
 * Same jobs, partials layout and consumers as rvq_gemv_tiles; operands must be
 * bf16 vectors or fp32 partials (fp16 operands: RVQ_ERR_UNSUPPORTED).  Reference
 * counterpart: the slot decode + F.linear pair it replaces. */
int rvq_gemv_tiles_exact(const rvq_gemv_tile_job* jobs, int n_jobs, void* stream);

/* Repack uint8 code planes [4][stage_stride] of a rows x cols weight into the
 * tile-major layout rvq_gemv_tiles reads: [tiles][rows][32] 32-bit words, word
 * (t, r, w) = the 4 stage codes (stage k in byte k) of vector (r, 32 t + w),
 * zero past the last vector of a row.  Every 256-column tile's rows are then
 * one contiguous range of 128-byte lines.  `out` holds rvq_tile_codes_bytes()
 * bytes, 16-byte aligned.  A layout of this library, not of the reference
 * artifact. */
int64_t rvq_tile_codes_bytes(int64_t rows, int64_t cols);
int rvq_tile_codes(const void* planes, int64_t stage_stride, int64_t rows, int64_t cols, void* out, void* stream);

/* Fused dequant-GEMM on the tensor cores for small batches and prompts (no
 * counterpart in the reference, which reconstructs W into the slot and calls
 * F.linear: infer_compressed_layerwise_triton.py:263, 290-292):
 *   y[t][r] = bf16( sum_c x[t][c] * W[r][c] ),  t < tokens (1..65536)
 * W is rebuilt on chip straight into tensor memory as the A operand of
 * tcgen05.mma (M = 128 weight rows, N = a block of up to 192 tokens, fp32
 * accumulation in TMEM); only the codes, scales and x are read from HBM.
 * More than 192 tokens run as equal blocks of at most 192, each weight chunk
 * decoded once per block.
 * exact != 0: every weight is bit-identical to rvq_decode's bf16 slot value;
 * exact == 0: the four fp16 codewords are summed in fp16, then widened to
 * fp32, scaled and rounded to bf16 (a codebook fp16 cannot hold always takes
 * the exact path).  A job of 2^31 or more (row tile, token block, 64-column
 * chunk) units returns RVQ_ERR_TOO_LARGE.  W: K=4 stages, 256 codes, uint8
 * codes in the tile-major layout of rvq_tile_codes (weight.indices, 16-byte
 * aligned), no tail; codebook fp32, fp16 or bf16.  x bf16 [tokens][cols]
 * row-major, 16-byte aligned, cols a multiple of 8; y bf16 [tokens][rows].
 * Deterministic: split-K pieces are added in a fixed order. */
typedef struct rvq_gemv_batch_job {
    rvq_entry weight;         /* weight.out is ignored */
    const void* x;            /* device, [tokens][cols] */
    void* y;                  /* device, [tokens][rows] */
    int64_t rows;
    int64_t cols;
    int64_t tokens;
    int32_t x_kind;           /* RVQ_BF16 */
    int32_t y_kind;           /* RVQ_BF16 */
    int32_t exact;            /* 1: bit-exact bf16 weights; 0: fp16 stage sums */
    int32_t reserved;         /* 0 */
} rvq_gemv_batch_job;

/* Bytes of workspace rvq_gemv_batch needs for this job on the current device
 * (split-K partial sums and one ticket per 128-row tile); 0 if the job is not
 * supported.  The workspace is 256-byte aligned device memory, zero-filled
 * once when allocated (every launch leaves its tickets at zero again);
 * launches that share a workspace must not overlap on the GPU. */
size_t rvq_gemv_batch_workspace_size(const rvq_gemv_batch_job* job);
int rvq_gemv_batch(const rvq_gemv_batch_job* job, void* workspace, size_t workspace_bytes, void* stream);

/* Reads and clears the sticky flag set when an rvq_gemv_batch wait on an
 * mbarrier gave up (the result of that launch is then invalid).  Synchronises
 * the current device.  Returns 1 if set, 0 if not, or -RVQ_ERR_CUDA. */
int rvq_take_batch_timeout(void);

/* Persistent batch-1 decode step: ONE cooperative launch (one CTA per SM)
 * runs every layer of a Qwen3 decoder for one token, i.e. per layer the
 * residual add + RMSNorm, the q/k/v, o, gate/up and down table GEMVs
 * (rvq_gemv_tiles, silu(gate) * up fused into down) and the decode attention,
 * then the final norm.  It replaces the per-layer kernel sequence
 * rvq_step_norm, rvq_gemv_tiles, rvq_step_attention, ... (the reference's
 * per-layer module calls of _layerwise_logits, infer_compressed_layerwise_
 * triton.py:271-292, with the weight never materialised).  Phases hand over
 * through counters in `sync` (bounded waits: a wait that gives up sets the
 * flag rvq_persist_take_error reads).  Every phase repeats the arithmetic
 * of the kernel it replaces in the same order, so h, x_final and the KV cache
 * are bit-identical to that kernel sequence.  Limits: tensor-parallel size 1,
 * head_dim 128, n_heads / n_kv <= 8, (n_heads / n_kv) * max_len <= 15360,
 * hidden <= 16384, every projection K=4 / 256 codes / d=8 / uint8 codes in
 * the tile-major layout of rvq_tile_codes. */
typedef struct rvq_persist_layer {
    rvq_entry proj[7];        /* q, k, v, o, gate, up, down; weight.out ignored */
    const void* input_norm;   /* device bf16 [hidden] */
    const void* post_norm;    /* device bf16 [hidden] */
    const void* q_norm;       /* device bf16 [head_dim] */
    const void* k_norm;       /* device bf16 [head_dim] */
    void* k_cache;            /* device bf16 [n_kv][max_len][head_dim], this layer */
    void* v_cache;
} rvq_persist_layer;

typedef struct rvq_persist_model {
    int32_t n_layers;
    int32_t hidden;
    int32_t intermediate;
    int32_t n_heads;
    int32_t n_kv;
    int32_t head_dim;
    int32_t max_len;
    int32_t vocab;
    float eps;
    float scaling;
    float valid_bias;         /* as rvq_attn_args */
    int32_t reserved;         /* 0 */
    const void* embed;        /* device bf16 [vocab][hidden] */
    const void* final_norm;   /* device bf16 [hidden] */
    const void* cos;          /* device bf16 [max_len][head_dim] */
    const void* sin;
    const int64_t* token;     /* device, the step's token */
    const int64_t* pos;       /* device, its position */
    void* h;                  /* device bf16 [hidden], the residual stream */
    void* x_final;            /* device bf16 [hidden], output: final-normed h */
    void* attn_out;           /* device bf16 [n_heads * head_dim] */
    float* q_part;            /* device fp32 partials [rvq_gemv_tiles_count(cols)][rows] of q, ... */
    float* k_part;
    float* v_part;
    float* o_part;
    float* gate_part;
    float* up_part;
    float* down_part;
    uint32_t* sync;           /* device, RVQ_PERSIST_SYNC_WORDS words, 16-byte aligned, zero before the
                                 first step; every step leaves its counters at zero */
} rvq_persist_model;

#define RVQ_PERSIST_SYNC_WORDS 1024

/* Bytes of the step plan for this model on the current device (0: not
 * supported; rvq_persist_plan tells why). */
int64_t rvq_persist_plan_bytes(const rvq_persist_model* m, const rvq_persist_layer* layers);

/* Writes the plan (host memory, `bytes` from rvq_persist_plan_bytes): the
 * model, every layer's GEMV jobs and the unit split of each GEMV phase over
 * the CTAs.  The caller copies it to device memory (16-byte aligned). */
int rvq_persist_plan(const rvq_persist_model* m, const rvq_persist_layer* layers, void* plan, int64_t bytes);

/* Host-only: the plan for `n_ctas` CTAs (16..160) without a device, for
 * inspection.  plan NULL: returns the size; else writes it and returns the
 * size; a negative value is -status. */
int64_t rvq_persist_plan_for(const rvq_persist_model* m, const rvq_persist_layer* layers, int32_t n_ctas,
                             void* plan, int64_t bytes);

/* One decode step with the plan at `plan_dev` (device).  No allocation, no
 * sync; may be captured in a CUDA graph. */
int rvq_persist_step(const void* plan_dev, void* stream);

/* Reads and clears the sticky flag of rvq_persist_step (a phase wait or a
 * code-word copy gave up; that step's outputs are invalid).  Synchronises the
 * current device.  Returns 1 if set, 0 if not, or -RVQ_ERR_CUDA. */
int rvq_persist_take_error(void);

/* Prefill GEMM with the weight decoded into shared memory, never into HBM:
 *   y[m][n] = bf16( sum_k x[m][k] * W[n][k] )
 * with W the RVQ entry reconstructed exactly as rvq_decode would (bit-identical
 * bf16 values) and the products accumulated in fp32 by tcgen05 tensor-core
 * MMAs in TMEM.  Replaces decode-into-slot + F.linear for a prompt
 * (infer_compressed_layerwise_triton.py:263, 290-292); no counterpart entry
 * point in the reference.  W: K=4 stages, 256 codes, uint8 codes in the
 * interleaved layout of rvq_interleave_codes (weight.indices), fp32 codebook
 * (16-byte aligned), no tail; k a multiple of 64, n a multiple of 8; x and y
 * bf16 row-major, 16-byte aligned. */
typedef struct rvq_gemm_job {
    rvq_entry weight;         /* weight.out is ignored */
    const void* x;            /* device, [m][k] */
    void* y;                  /* device, [m][n] */
    int64_t m;
    int64_t n;
    int64_t k;
    int32_t x_kind;           /* RVQ_BF16 */
    int32_t y_kind;           /* RVQ_BF16 */
} rvq_gemm_job;

int rvq_gemm_prefill(const rvq_gemm_job* job, void* stream);

/* Reads and clears the sticky flag set when an rvq_gemm_prefill or
 * rvq_gemv_tiles wait on an mbarrier gave up (bounded waits; the result of
 * that launch is then invalid).  Synchronises the current device.
 * Returns 1 if set, 0 if not, or -RVQ_ERR_CUDA. */
int rvq_take_gemm_timeout(void);
int rvq_take_wait_timeout(void);

/* Reads and clears the sticky device flag that kernels set when an index is
 * outside [0, ncodes) (the decoded element then uses code 0).  Synchronises
 * the current device.  Returns 1 if the flag was set, 0 if not, or -RVQ_ERR_CUDA. */
int rvq_take_index_error(void);

/* ---- Encoder (the offline compressor's hot loops on the GPU) -----------------
 * Replace assign_codes / kmeans_train / encode_rvq_tensor's stage loop
 * (compress_full_model.py:196-234, 337-366), which the reference runs on the
 * CPU.  Distances are pairwise_sqdist's (|x|^2 + |c|^2) - 2 x.c in fp32; the
 * argmin keeps the first minimum, as torch.argmin does.  Only d = 8. */

/* codes[k][i] = nearest codeword of stage k to residual_k(i), residual_0 = x,
 * residual_{k+1} = residual_k - codebooks[k][codes[k][i]] (fp32).  x: device
 * fp32 [n][8], 16-byte aligned; codebooks: device fp32 [stages][ncodes][8]
 * (ncodes <= 4096); codes: device [stages][n] of code_kind (RVQ_U8 when
 * ncodes <= 256, or RVQ_I16); residual_out: device fp32 [n][8] or NULL. */
int rvq_encode_vectors(const float* x, int64_t n, const float* codebooks, int stages, int ncodes, int d, void* codes,
                       int code_kind, float* residual_out, void* stream);

/* One Lloyd step's statistics: assign[i] = nearest centroid (or assign NULL),
 * and when `sums` is set, sums[c][t] += round(x[i][t] * 2^32) and counts[c]
 * += 1 in 64-bit integer atomics (order-independent: the same input always
 * gives the same sums).  sums [k][8] and counts [k] must be zeroed before. */
int rvq_kmeans_step(const float* x, int64_t n, const float* centroids, int k, int d, int32_t* assign,
                    unsigned long long* sums, unsigned long long* counts, void* stream);

/* ---- Artifact pack loader ---------------------------------------------------
 * Replaces the artifact load of infer_compressed_layerwise_triton.py:421-432
 * (torch.load of the compressor's pickle, compress_full_model.py:624-631, then
 * one host-to-device copy per tensor) for an artifact rewritten once as a pack
 * (rvq_b200/pack.py: a JSON header, then every tensor's bytes at page-aligned
 * offsets).  Copies `nbytes` bytes of the file at `path`, starting at byte
 * `offset`, to device memory `device_dst`: a reader thread fills a ring of
 * pinned buffers with pread() while the copies run on `stream`.  Returns once
 * the bytes are on the device (it waits for its own copies only). */
int rvq_pack_load(const char* path, uint64_t offset, uint64_t nbytes, void* device_dst, void* stream);

/* Last CUDA error code seen by this library on the calling thread (0 = none). */
int rvq_last_cuda_error(void);

/* Static description of a status code. */
const char* rvq_status_string(int status);

/* Library version as 10000*major + 100*minor + patch. */
int rvq_version(void);

#ifdef __cplusplus
}
#endif

#endif /* RVQ_B200_H */
