/*
 * ggml_oracle.c -- CPU restatement of ggml's block-quantised arithmetic
 * (TEST INFRASTRUCTURE ONLY; see ggml_oracle.h for provenance and scope).
 *
 * Block formats (ggml's public ABI, also the reference weight-file payload,
 * sam3.cpp:3095-3198):
 *   Q8_0 = { fp16 d; int8 qs[32]; }              34 B, x = d * q
 *   Q4_0 = { fp16 d; uint8 qs[16]; }             18 B, x = d * (nib - 8),
 *          low nibbles hold elements 0..15, high nibbles 16..31
 *   Q4_1 = { fp16 d; fp16 m; uint8 qs[16]; }     20 B, x = d * nib + m
 *   Q8_1 = { fp16 d; fp16 s; int8 qs[32]; }      36 B, s = d * sum(q)
 */
#include "ggml_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#if defined(__AVX2__)
#include <immintrin.h>
#endif

#define QK 32

typedef struct { uint16_t d; int8_t qs[QK]; } blk_q8_0;
typedef struct { uint16_t d; uint8_t qs[QK / 2]; } blk_q4_0;
typedef struct { uint16_t d; uint16_t m; uint8_t qs[QK / 2]; } blk_q4_1;
typedef struct { uint16_t d; uint16_t s; int8_t qs[QK]; } blk_q8_1;

_Static_assert(sizeof(blk_q8_0) == 34, "q8_0 size");
_Static_assert(sizeof(blk_q4_0) == 18, "q4_0 size");
_Static_assert(sizeof(blk_q4_1) == 20, "q4_1 size");
_Static_assert(sizeof(blk_q8_1) == 36, "q8_1 size");

/* IEEE binary16 conversions, round-to-nearest-even (what F16C's
 * vcvtps2ph with imm 0 and ggml's software fallback both implement). */
uint16_t orc_fp32_to_fp16(float f) {
    _Float16 h = (_Float16)f;
    uint16_t u;
    memcpy(&u, &h, 2);
    return u;
}

float orc_fp16_to_fp32(uint16_t u) {
    _Float16 h;
    memcpy(&h, &u, 2);
    return (float)h;
}

int64_t orc_row_size(int type, int64_t k) {
    switch (type) {
    case ORC_F32:  return 4 * k;
    case ORC_F16:  return 2 * k;
    case ORC_Q8_0: return (k / QK) * (int64_t)sizeof(blk_q8_0);
    case ORC_Q4_0: return (k / QK) * (int64_t)sizeof(blk_q4_0);
    case ORC_Q4_1: return (k / QK) * (int64_t)sizeof(blk_q4_1);
    case ORC_Q8_1: return (k / QK) * (int64_t)sizeof(blk_q8_1);
    default: return -1;
    }
}

/* ---- weight quantisers (ggml-quants.c quantize_row_*_ref) ------------- */

void orc_quantize_q8_0_ref(const float *x, void *vy, int64_t k) {
    blk_q8_0 *y = (blk_q8_0 *)vy;
    for (int64_t i = 0; i < k / QK; i++) {
        const float *xb = x + i * QK;
        float amax = 0.0f;
        for (int j = 0; j < QK; j++) amax = fmaxf(amax, fabsf(xb[j]));
        const float d = amax / 127;
        const float id = d ? 1.0f / d : 0.0f;
        y[i].d = orc_fp32_to_fp16(d);
        for (int j = 0; j < QK; j++) y[i].qs[j] = (int8_t)roundf(xb[j] * id);
    }
}

void orc_quantize_q4_0_ref(const float *x, void *vy, int64_t k) {
    blk_q4_0 *y = (blk_q4_0 *)vy;
    for (int64_t i = 0; i < k / QK; i++) {
        const float *xb = x + i * QK;
        float amax = 0.0f, max = 0.0f;
        for (int j = 0; j < QK; j++) {
            const float v = xb[j];
            if (amax < fabsf(v)) { amax = fabsf(v); max = v; }
        }
        const float d = max / -8;
        const float id = d ? 1.0f / d : 0.0f;
        y[i].d = orc_fp32_to_fp16(d);
        for (int j = 0; j < QK / 2; j++) {
            const float x0 = xb[j] * id;
            const float x1 = xb[QK / 2 + j] * id;
            int xi0 = (int8_t)(x0 + 8.5f); if (xi0 > 15) xi0 = 15;
            int xi1 = (int8_t)(x1 + 8.5f); if (xi1 > 15) xi1 = 15;
            y[i].qs[j] = (uint8_t)(xi0 | (xi1 << 4));
        }
    }
}

void orc_quantize_q4_1_ref(const float *x, void *vy, int64_t k) {
    blk_q4_1 *y = (blk_q4_1 *)vy;
    for (int64_t i = 0; i < k / QK; i++) {
        const float *xb = x + i * QK;
        float min = FLT_MAX, max = -FLT_MAX;
        for (int j = 0; j < QK; j++) {
            const float v = xb[j];
            if (v < min) min = v;
            if (v > max) max = v;
        }
        const float d = (max - min) / 15;
        const float id = d ? 1.0f / d : 0.0f;
        y[i].d = orc_fp32_to_fp16(d);
        y[i].m = orc_fp32_to_fp16(min);
        for (int j = 0; j < QK / 2; j++) {
            const float x0 = (xb[j] - min) * id;
            const float x1 = (xb[QK / 2 + j] - min) * id;
            int xi0 = (int8_t)(x0 + 0.5f); if (xi0 > 15) xi0 = 15;
            int xi1 = (int8_t)(x1 + 0.5f); if (xi1 > 15) xi1 = 15;
            y[i].qs[j] = (uint8_t)(xi0 | (xi1 << 4));
        }
    }
}

int64_t orc_quantize_chunk(int type, const float *x, void *y, int64_t n_rows, int64_t n_per_row) {
    const int64_t rs = orc_row_size(type, n_per_row);
    for (int64_t r = 0; r < n_rows; r++) {
        const float *xr = x + r * n_per_row;
        void *yr = (char *)y + r * rs;
        switch (type) {
        case ORC_Q8_0: orc_quantize_q8_0_ref(xr, yr, n_per_row); break;
        case ORC_Q4_0: orc_quantize_q4_0_ref(xr, yr, n_per_row); break;
        case ORC_Q4_1: orc_quantize_q4_1_ref(xr, yr, n_per_row); break;
        default: return -1;
        }
    }
    return n_rows * rs;
}

/* ---- activation quantisers (ggml-cpu x86 from_float) ------------------
 * d = amax / 127 (stored as fp16), id = 127 / amax (0 when amax == 0),
 * q = round-half-to-even(x * id).  rintf rounds to nearest even under the
 * default rounding mode, like _mm256_round_ps(v, _MM_ROUND_NEAREST). */

void orc_quantize_q8_0_act(const float *x, void *vy, int64_t k) {
    blk_q8_0 *y = (blk_q8_0 *)vy;
    for (int64_t i = 0; i < k / QK; i++) {
        const float *xb = x + i * QK;
        float amax = 0.0f;
        for (int j = 0; j < QK; j++) amax = fmaxf(amax, fabsf(xb[j]));
        const float d = amax / 127.f;
        const float id = (amax != 0.0f) ? 127.f / amax : 0.0f;
        y[i].d = orc_fp32_to_fp16(d);
        for (int j = 0; j < QK; j++) y[i].qs[j] = (int8_t)rintf(xb[j] * id);
    }
}

void orc_quantize_q8_1_act(const float *x, void *vy, int64_t k) {
    blk_q8_1 *y = (blk_q8_1 *)vy;
    for (int64_t i = 0; i < k / QK; i++) {
        const float *xb = x + i * QK;
        float amax = 0.0f;
        for (int j = 0; j < QK; j++) amax = fmaxf(amax, fabsf(xb[j]));
        const float d = amax / 127.f;
        const float id = (amax != 0.0f) ? 127.f / amax : 0.0f;
        y[i].d = orc_fp32_to_fp16(d);
        int sum = 0;
        for (int j = 0; j < QK; j++) {
            y[i].qs[j] = (int8_t)rintf(xb[j] * id);
            sum += y[i].qs[j];
        }
        y[i].s = orc_fp32_to_fp16(d * (float)sum);
    }
}

void orc_dequantize_row(int type, const void *vx, float *y, int64_t k) {
    const int64_t nb = k / QK;
    switch (type) {
    case ORC_F32: memcpy(y, vx, (size_t)k * 4); break;
    case ORC_F16: {
        const uint16_t *x = (const uint16_t *)vx;
        for (int64_t i = 0; i < k; i++) y[i] = orc_fp16_to_fp32(x[i]);
    } break;
    case ORC_Q8_0: {
        const blk_q8_0 *x = (const blk_q8_0 *)vx;
        for (int64_t i = 0; i < nb; i++) {
            const float d = orc_fp16_to_fp32(x[i].d);
            for (int j = 0; j < QK; j++) y[i * QK + j] = x[i].qs[j] * d;
        }
    } break;
    case ORC_Q4_0: {
        const blk_q4_0 *x = (const blk_q4_0 *)vx;
        for (int64_t i = 0; i < nb; i++) {
            const float d = orc_fp16_to_fp32(x[i].d);
            for (int j = 0; j < QK / 2; j++) {
                y[i * QK + j] = ((x[i].qs[j] & 0x0F) - 8) * d;
                y[i * QK + j + QK / 2] = ((x[i].qs[j] >> 4) - 8) * d;
            }
        }
    } break;
    case ORC_Q4_1: {
        const blk_q4_1 *x = (const blk_q4_1 *)vx;
        for (int64_t i = 0; i < nb; i++) {
            const float d = orc_fp16_to_fp32(x[i].d);
            const float m = orc_fp16_to_fp32(x[i].m);
            for (int j = 0; j < QK / 2; j++) {
                y[i * QK + j] = (x[i].qs[j] & 0x0F) * d + m;
                y[i * QK + j + QK / 2] = (x[i].qs[j] >> 4) * d + m;
            }
        }
    } break;
    case ORC_Q8_1: {
        const blk_q8_1 *x = (const blk_q8_1 *)vx;
        for (int64_t i = 0; i < nb; i++) {
            const float d = orc_fp16_to_fp32(x[i].d);
            for (int j = 0; j < QK; j++) y[i * QK + j] = x[i].qs[j] * d;
        }
    } break;
    default: break;
    }
}

int orc_vec_dot_type(int wtype) {
    switch (wtype) {
    case ORC_Q8_0: return ORC_Q8_0;
    case ORC_Q4_0: return ORC_Q8_0;
    case ORC_Q4_1: return ORC_Q8_1;
    case ORC_F16:  return ORC_F16;
    case ORC_F32:  return ORC_F32;
    default: return -1;
    }
}

#if defined(__AVX2__)
/* Exact int32 dot of 32 int8 pairs with |a| <= 127 (ggml's x86 form: |a| times
 * sign(b, a) by maddubs -- pairwise int16 sums of at most 2 * 127 * 128, no
 * saturation -- then madd against ones and a horizontal sum). */
static inline int32_t dot32_i8(__m256i a, __m256i b) {
    const __m256i ax = _mm256_sign_epi8(a, a);
    const __m256i sb = _mm256_sign_epi8(b, a);
    const __m256i d32 = _mm256_madd_epi16(_mm256_maddubs_epi16(ax, sb), _mm256_set1_epi16(1));
    __m128i s = _mm_add_epi32(_mm256_castsi256_si128(d32), _mm256_extracti128_si256(d32, 1));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0x4E));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0xB1));
    return _mm_cvtsi128_si32(s);
}
#endif

/* Integer dot of block b (exact; the AVX2 form and the scalar loop give the
 * same int32). */
static int32_t block_isum(int wtype, const void *w, const void *xq, int64_t b) {
    int32_t s = 0;
    if (wtype == ORC_Q8_0) {
        const blk_q8_0 *wb = (const blk_q8_0 *)w + b;
        const blk_q8_0 *xb = (const blk_q8_0 *)xq + b;
#if defined(__AVX2__)
        return dot32_i8(_mm256_loadu_si256((const __m256i *)xb->qs), _mm256_loadu_si256((const __m256i *)wb->qs));
#else
        for (int j = 0; j < QK; j++) s += (int32_t)wb->qs[j] * xb->qs[j];
#endif
    } else if (wtype == ORC_Q4_0) {
        const blk_q4_0 *wb = (const blk_q4_0 *)w + b;
        const blk_q8_0 *xb = (const blk_q8_0 *)xq + b;
#if defined(__AVX2__)
        /* nibbles -> int8: low nibbles are elements 0..15, high 16..31, minus 8 */
        const __m128i raw = _mm_loadu_si128((const __m128i *)wb->qs);
        const __m256i nib = _mm256_and_si256(
            _mm256_set_m128i(_mm_srli_epi16(raw, 4), raw), _mm256_set1_epi8(0x0F));
        const __m256i wv = _mm256_sub_epi8(nib, _mm256_set1_epi8(8));
        return dot32_i8(_mm256_loadu_si256((const __m256i *)xb->qs), wv);
#else
        for (int j = 0; j < QK / 2; j++) {
            s += ((wb->qs[j] & 0x0F) - 8) * xb->qs[j];
            s += ((wb->qs[j] >> 4) - 8) * xb->qs[j + QK / 2];
        }
#endif
    } else if (wtype == ORC_Q4_1) {
        const blk_q4_1 *wb = (const blk_q4_1 *)w + b;
        const blk_q8_1 *xb = (const blk_q8_1 *)xq + b;
        for (int j = 0; j < QK / 2; j++) {
            s += (wb->qs[j] & 0x0F) * xb->qs[j];
            s += (wb->qs[j] >> 4) * xb->qs[j + QK / 2];
        }
    }
    return s;
}

/* Generic vec_dot: sumf = fma((float)isum_b, d_w*d_x, sumf) block by block
 * in order, plus m_w*s_x for Q4_1.  The product d_w*d_x of two fp16 values
 * is exact in fp32. */
float orc_vec_dot(int wtype, int64_t k, const void *w, const void *xq) {
    const int64_t nb = k / QK;
    float sumf = 0.0f;
    if (wtype == ORC_F32 || wtype == ORC_F16) {
        /* F32/F16 weights: f32 products summed in fp32 (x already in the
         * vec_dot_type, i.e. f32 or f16). */
        for (int64_t i = 0; i < k; i++) {
            float a, b;
            if (wtype == ORC_F32) { a = ((const float *)w)[i]; b = ((const float *)xq)[i]; }
            else { a = orc_fp16_to_fp32(((const uint16_t *)w)[i]); b = orc_fp16_to_fp32(((const uint16_t *)xq)[i]); }
            sumf = fmaf(a, b, sumf);
        }
        return sumf;
    }
    for (int64_t b = 0; b < nb; b++) {
        const int32_t isum = block_isum(wtype, w, xq, b);
        float dw, dx;
        if (wtype == ORC_Q8_0) {
            dw = orc_fp16_to_fp32(((const blk_q8_0 *)w)[b].d);
            dx = orc_fp16_to_fp32(((const blk_q8_0 *)xq)[b].d);
        } else if (wtype == ORC_Q4_0) {
            dw = orc_fp16_to_fp32(((const blk_q4_0 *)w)[b].d);
            dx = orc_fp16_to_fp32(((const blk_q8_0 *)xq)[b].d);
        } else {
            dw = orc_fp16_to_fp32(((const blk_q4_1 *)w)[b].d);
            dx = orc_fp16_to_fp32(((const blk_q8_1 *)xq)[b].d);
        }
        sumf = fmaf((float)isum, dw * dx, sumf);
        if (wtype == ORC_Q4_1) {
            const float mw = orc_fp16_to_fp32(((const blk_q4_1 *)w)[b].m);
            const float sx = orc_fp16_to_fp32(((const blk_q8_1 *)xq)[b].s);
            sumf = fmaf(mw, sx, sumf);
        }
    }
    return sumf;
}

void orc_block_dots(int wtype, int64_t k, const void *w, const void *xq, int32_t *out) {
    for (int64_t b = 0; b < k / QK; b++) out[b] = block_isum(wtype, w, xq, b);
}

static void quantize_act_row(int vtype, const float *x, void *y, int64_t k) {
    if (vtype == ORC_Q8_0) orc_quantize_q8_0_act(x, y, k);
    else if (vtype == ORC_Q8_1) orc_quantize_q8_1_act(x, y, k);
    else if (vtype == ORC_F16) {
        uint16_t *h = (uint16_t *)y;
        for (int64_t i = 0; i < k; i++) h[i] = orc_fp32_to_fp16(x[i]);
    } else memcpy(y, x, (size_t)k * 4);
}

void orc_mul_mat(int wtype, const void *w, int64_t K, int64_t N,
                 const float *x, int64_t ldx, int64_t M,
                 float *y, int64_t ldy, int n_threads) {
    const int vtype = orc_vec_dot_type(wtype);
    const int64_t wrs = orc_row_size(wtype, K);
    const int64_t xrs = orc_row_size(vtype, K);
    char *xq = (char *)malloc((size_t)(xrs * (M > 0 ? M : 1)));
    if (n_threads < 1) n_threads = 1;
    #pragma omp parallel for num_threads(n_threads) schedule(static)
    for (int64_t m = 0; m < M; m++) quantize_act_row(vtype, x + m * ldx, xq + m * xrs, K);
    #pragma omp parallel for num_threads(n_threads) schedule(dynamic, 4)
    for (int64_t m = 0; m < M; m++) {
        for (int64_t n = 0; n < N; n++) {
            y[m * ldy + n] = orc_vec_dot(wtype, K, (const char *)w + n * wrs, xq + m * xrs);
        }
    }
    free(xq);
}

void orc_mul_mat_block_dots(int wtype, const void *w, int64_t K, int64_t N,
                            const float *x, int64_t M, int32_t *out, int n_threads) {
    const int vtype = orc_vec_dot_type(wtype);
    const int64_t wrs = orc_row_size(wtype, K);
    const int64_t xrs = orc_row_size(vtype, K);
    const int64_t nb = K / QK;
    char *xq = (char *)malloc((size_t)(xrs * (M > 0 ? M : 1)));
    if (n_threads < 1) n_threads = 1;
    for (int64_t m = 0; m < M; m++) quantize_act_row(vtype, x + m * K, xq + m * xrs, K);
    #pragma omp parallel for num_threads(n_threads) schedule(static)
    for (int64_t m = 0; m < M; m++)
        for (int64_t n = 0; n < N; n++)
            orc_block_dots(wtype, K, (const char *)w + n * wrs, xq + m * xrs, out + (m * N + n) * nb);
    free(xq);
}
