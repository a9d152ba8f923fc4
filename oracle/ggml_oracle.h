/*
 * ggml_oracle.h -- CPU restatement of the ggml arithmetic that sam3.cpp's
 * encoder hot path relies on.  TEST INFRASTRUCTURE ONLY: the product library
 * (libsam3_b200.so) never links or calls this code; only tests/, the smoke
 * check in __graft_entry__.py and bench.py's CPU-baseline leg load it, and
 * only as the checker / the timed CPU restatement.
 *
 * The arithmetic lives in ggml (git submodule PABannier/ggml, pinned commit
 * not recorded in the reference snapshot; the submodule directory
 * reference/ggml is empty).  What is restated here is ggml's published
 * algorithm for these entry points, anchored on the reference call sites:
 *   - weight quantisers (ggml-quants.c *_ref rules), used by
 *     examples/quantize.cpp:244 (ggml_quantize_chunk) -- pinned against the
 *     gguf 0.19.0 Python mirror (gguf/quants.py) by tests/golden fixtures;
 *   - the activation quantiser ggml-cpu runs as from_float for vec_dot_type
 *     (x86 AVX rule: id = 127/amax, round-half-to-even) -- parity unpinned
 *     by any reference-owned vector;
 *   - the generic vec_dot block formula: per 32-block an int32 dot of the
 *     integer codes, scaled by fp16(d_w) * fp16(d_x), summed in fp32;
 *   - ggml_mul_mat(w, x) at sam3.cpp:3742,3783,3796,3799.
 */
#ifndef SAM3_B200_GGML_ORACLE_H
#define SAM3_B200_GGML_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml_type enum values (the reference's weight-file dtype codes,
 * sam3.cpp:3246-3255). */
enum orc_type {
    ORC_F32  = 0,
    ORC_F16  = 1,
    ORC_Q4_0 = 2,
    ORC_Q4_1 = 3,
    ORC_Q8_0 = 8,
    ORC_Q8_1 = 9,
};

uint16_t orc_fp32_to_fp16(float f);
float    orc_fp16_to_fp32(uint16_t h);

/* bytes of one row of k elements of `type` (ggml_row_size) */
int64_t orc_row_size(int type, int64_t k);

/* weight quantisers: ggml-quants.c quantize_row_*_ref */
void orc_quantize_q8_0_ref(const float *x, void *y, int64_t k);
void orc_quantize_q4_0_ref(const float *x, void *y, int64_t k);
void orc_quantize_q4_1_ref(const float *x, void *y, int64_t k);
/* quantize n_rows rows of n_per_row (ggml_quantize_chunk without imatrix) */
int64_t orc_quantize_chunk(int type, const float *x, void *y, int64_t n_rows, int64_t n_per_row);

/* activation quantisers: ggml-cpu from_float for vec_dot_type (x86 rule) */
void orc_quantize_q8_0_act(const float *x, void *y, int64_t k);
void orc_quantize_q8_1_act(const float *x, void *y, int64_t k);

void orc_dequantize_row(int type, const void *x, float *y, int64_t k);

/* activation type a weight type is dotted against (ggml vec_dot_type) */
int orc_vec_dot_type(int wtype);

/* one output element: weight row (wtype) . quantised activation row */
float orc_vec_dot(int wtype, int64_t k, const void *w_row, const void *xq_row);

/* per-32-block integer dots of one weight row with one activation row */
void orc_block_dots(int wtype, int64_t k, const void *w_row, const void *xq_row, int32_t *out);

/* ggml_mul_mat(w, x): w is [K, N] of wtype (N rows of K), x is f32 [K, M]
 * (M rows of K, row stride ldx floats), y is f32 [N, M] (row stride ldy).
 * Quantises x with the activation rule, then y[m][n] = vec_dot. */
void orc_mul_mat(int wtype, const void *w, int64_t K, int64_t N,
                 const float *x, int64_t ldx, int64_t M,
                 float *y, int64_t ldy, int n_threads);

/* block dots for every (m, n, b): out[(m*N + n)*(K/32) + b] */
void orc_mul_mat_block_dots(int wtype, const void *w, int64_t K, int64_t N,
                            const float *x, int64_t M, int32_t *out, int n_threads);

#ifdef __cplusplus
}
#endif
#endif
