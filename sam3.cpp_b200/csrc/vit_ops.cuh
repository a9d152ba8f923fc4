// vit_ops.cuh -- memory-bound kernels of the SAM3 visual encoder (HBM
// roofline): preprocessing, layout changes folded into their producers,
// LayerNorm fused with Q8_0 activation quantisation, RoPE, pooling.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace b200 {

// sam3_preprocess_image (sam3.cpp:3490-3518): uint8 HWC img x img ->
// f32 CHW (p/255 - 0.5)/0.5.  Inputs of another size go through
// resize_bilinear_u8 first (sam3.cpp:3445-3485, double precision).
cudaError_t preprocess_sam3(const uint8_t *rgb, int img, float *out_chw, cudaStream_t s);

// sam2_preprocess_image (sam3.cpp:3522-3548): the same layout with the
// ImageNet normalisation, mean (0.485, 0.456, 0.406), std (0.229, 0.224, 0.225).
cudaError_t preprocess_sam2(const uint8_t *rgb, int img, float *out_chw, cudaStream_t s);
cudaError_t resize_bilinear_u8(const uint8_t *src, int sw, int sh, uint8_t *dst, int dw, int dh, cudaStream_t s);

// im2col of the 14x14 stride-14 patch embedding (ggml_conv_2d_sk_p0,
// sam3.cpp:3819): A[t][k] fp16, k = (c*p + ky)*p + kx, zero-padded to kp.
cudaError_t im2col_patch(const float *img_chw, int img, int patch, int kp, void *a_f16, cudaStream_t s);

// x[t][e] = conv[t][e] + pos[(w%g) + g*(h%g)][e], then LayerNorm (eps) with
// w/b (sam3.cpp:3823-3831).  G = grid side, rows = G*G.
cudaError_t add_pos_layernorm(const float *conv, const float *pos, int g, int G, int E, const float *w,
                              const float *b, float eps, float *x, cudaStream_t s);

// LayerNorm of rows of x (eps, w, b) quantised to Q8_0 into codes/quads
// (mmq.cuh layout).  win > 0: row t of the G x G grid is written at its
// ggml_win_part position (window-major, sam3.cpp:3734); rows may hold several
// G x G images stacked image-major, each partitioned on its own.
cudaError_t layernorm_q8(const float *x, int rows, int E, const float *w, const float *b, float eps, int G, int win,
                         void *codes, void *quads, int ld, cudaStream_t s);
// layernorm_q8's LayerNorm and Q8_0 quantisation (same codes and scales),
// written dequantised -- fp16(q * fp16(d)) [rows][E] in the same row order --
// as the A operand of mmq_dq16.  E in {256, 512, 768, 1024, 1280, 1536};
// cudaErrorInvalidValue otherwise.
cudaError_t layernorm_dq16(const float *x, int rows, int E, const float *w, const float *b, float eps, int G, int win,
                           void *out16, cudaStream_t s);

// Attention inputs from ggml f32 tensors Q, K, V [64, N, H, B] (contiguous:
// [BH][N][64]) -> bf16 Q, K (same layout) and V^T [BH][64][N].  N % 8 == 0.
cudaError_t attn_inputs_from_f32(const float *q, const float *k, const float *v, int BH, int N, void *qb, void *kb,
                                 void *vt, cudaStream_t s);

// Row map of ggml_win_unpart: windowed row -> token row (G x G grid), for
// nimg images stacked image-major (rows of image i at [i G^2, (i + 1) G^2)).
cudaError_t window_rowmap(int G, int win, int *rowmap, cudaStream_t s, int nimg = 1);

cudaError_t f32_to_f16(const float *x, int64_t n, void *y, cudaStream_t s);

// Rows [0, M) of an f32 matrix with row stride ldx -> dense fp16 [M][K]
// (round to nearest even, as ggml_fp32_to_fp16).
cudaError_t f32_rows_to_f16(const float *x, int64_t ldx, int M, int K, void *y, cudaStream_t s);

// 2x2 stride-2 max pool of an HWC f32 map (G x G x C) -> fp16 (G/2)^2 x C.
cudaError_t maxpool2x2_f16(const float *x, int G, int C, void *y, cudaStream_t s);

// im2col of a 3x3 pad-1 convolution over an HWC fp16 map (W x H x C):
// A[p][(ky*3 + kx)*C + ci].
cudaError_t im2col3x3_f16(const void *x, int W, int H, int C, void *a, cudaStream_t s);

}  // namespace b200
