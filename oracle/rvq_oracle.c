/*
 * CPU oracle for RVQ weight reconstruction (C restatement, OpenMP).
 *
 * TEST INFRASTRUCTURE ONLY.  Used by tests/ as a second, independent
 * restatement of the reference arithmetic and by bench.py's CPU-baseline leg
 * (reported as a "port" of the reference's CPU path).  Nothing in the
 * rvq_b200 product links or calls it.
 *
 * Arithmetic restated from the reference:
 *   _rvq_decode_into_kernel   triton_decode_kernels.py:74-111
 *     acc = 0.0f                                      (78)
 *     for k in 0..K-1: acc += cb[k][idx[k][n]][0..7]  (80-97, sequential)
 *     acc *= float(scale[n // GROUP_VECS])            (99-101)
 *     store cast(acc) where 8n+t < TRIMMED            (103-111)
 *   tail copy                 triton_decode_kernels.py:187-188
 *   _decode_rvq_into          infer_compressed_layerwise_single_slot.py:123-149
 *     (same result: torch's stage sum is sequential from +0.0 for K <= 17)
 *
 * Casts are round-to-nearest-even, written here from the IEEE-754 binary16 /
 * bfloat16 definitions.  Build with -ffp-contract=off so no add/mul pair is
 * fused.
 */
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum { OUT_F16 = 0, OUT_BF16 = 1, OUT_F32 = 2 };

static inline uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* fp32 -> binary16, round to nearest, ties to even, with subnormals. */
static inline uint16_t f32_to_f16_rne(float f) {
    uint32_t x = f32_bits(f);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t a = x & 0x7FFFFFFFu;
    if (a >= 0x7F800000u)                    /* inf / nan */
        return (uint16_t)(sign | (a > 0x7F800000u ? 0x7E00u : 0x7C00u));
    if (a >= 0x477FF000u)                    /* >= 65520 rounds to inf */
        return (uint16_t)(sign | 0x7C00u);
    if (a < 0x38800000u) {                   /* below 2^-14: fp16 subnormal */
        if (a <= 0x33000000u)                /* <= 2^-25 rounds to zero */
            return (uint16_t)sign;
        uint32_t e = a >> 23;                /* 102..112 */
        uint32_t m = (a & 0x7FFFFFu) | 0x800000u;
        uint32_t shift = 126u - e;           /* 14..24 */
        uint32_t q = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t e = (a >> 23) - 112u;           /* rebias 127 -> 15 */
    uint32_t m = a & 0x7FFFFFu;
    uint32_t q = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
    return (uint16_t)(sign | q);
}

/* fp32 -> bfloat16, round to nearest, ties to even. */
static inline uint16_t f32_to_bf16_rne(float f) {
    uint32_t x = f32_bits(f);
    if ((x & 0x7FFFFFFFu) > 0x7F800000u)
        return (uint16_t)(((x >> 16) & 0x8000u) | 0x7FC0u);
    uint32_t lsb = (x >> 16) & 1u;
    return (uint16_t)((x + 0x7FFFu + lsb) >> 16);
}

static inline void store_cast(void* out, int out_kind, int64_t pos, float v) {
    if (out_kind == OUT_F16)       ((uint16_t*)out)[pos] = f32_to_f16_rne(v);
    else if (out_kind == OUT_BF16) ((uint16_t*)out)[pos] = f32_to_bf16_rne(v);
    else                           ((float*)out)[pos] = v;
}

/*
 * indices      [stages][stage_stride] (uint8 when index_bytes == 1, int16 when 2)
 * codebook     [stages][ncodes][d] fp32
 * scales       fp32, one per group of group_vecs vectors
 * tail         fp32 tail values, copied to out[trimmed .. trimmed+tail_numel)
 * out          raw output buffer of out_kind
 * Returns 0, or -1 on bad arguments, -2 on an out-of-range index.
 */
int rvq_oracle_decode(const void* indices, int index_bytes, int64_t stage_stride,
                      int stages, int64_t nvec, const float* codebook, int ncodes, int d,
                      const float* scales, int64_t group_vecs, int64_t trimmed,
                      const float* tail, int64_t tail_numel, void* out, int out_kind,
                      int nthreads) {
    if (stages < 1 || d < 1 || d > 64 || ncodes < 1 || group_vecs < 1 || nvec < 0)
        return -1;
    if (index_bytes != 1 && index_bytes != 2) return -1;
    if (out_kind < OUT_F16 || out_kind > OUT_F32) return -1;
    int bad = 0;
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel for schedule(static) num_threads(nthreads) reduction(| : bad)
#endif
    for (int64_t n = 0; n < nvec; n++) {
        float acc[64];
        for (int t = 0; t < d; t++) acc[t] = 0.0f;
        for (int k = 0; k < stages; k++) {
            int64_t c;
            if (index_bytes == 1) c = ((const uint8_t*)indices)[(int64_t)k * stage_stride + n];
            else                  c = ((const int16_t*)indices)[(int64_t)k * stage_stride + n];
            if (c < 0 || c >= ncodes) { bad = 1; c = 0; }
            const float* cw = codebook + ((int64_t)k * ncodes + c) * d;
            for (int t = 0; t < d; t++) acc[t] += cw[t];
        }
        float s = scales[n / group_vecs];
        for (int t = 0; t < d; t++) {
            int64_t pos = n * d + t;
            if (pos < trimmed) store_cast(out, out_kind, pos, acc[t] * s);
        }
    }
    for (int64_t i = 0; i < tail_numel; i++) store_cast(out, out_kind, trimmed + i, tail[i]);
    return bad ? -2 : 0;
}

/* Number of threads OpenMP would use by default (the host's cores). */
int rvq_oracle_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Conversion helpers exported so tests can cross-check them against numpy. */
void rvq_oracle_f32_to_f16(const float* x, uint16_t* y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = f32_to_f16_rne(x[i]);
}
void rvq_oracle_f32_to_bf16(const float* x, uint16_t* y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = f32_to_bf16_rne(x[i]);
}
