/*
 * vit_oracle.h -- CPU restatement of the SAM3 visual encoder graph that
 * sam3_encode_image builds (TEST INFRASTRUCTURE ONLY, like ggml_oracle.h):
 * preprocessing, the ViT prefix, the ViT blocks and the SimpleFPN neck, on
 * top of the ggml arithmetic restated in ggml_oracle.c.
 *
 * Layouts are ggml's: an activation [E, W, H] is stored token-major,
 * x[(w + W*h)*E + e]; a neck feature map [C, W, H] the same way.
 */
#ifndef SAM3_B200_VIT_ORACLE_H
#define SAM3_B200_VIT_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int img;            /* input side (1008)                      sam3.cpp:80  */
    int patch;          /* patch size (14)                        sam3.cpp:81  */
    int E;              /* embed dim (1024)                       sam3.cpp:82  */
    int depth;          /* blocks (32)                            sam3.cpp:83  */
    int heads;          /* heads (16), head_dim = E / heads = 64  sam3.cpp:84  */
    int mlp;            /* MLP dim (4736)                         sam3.cpp:85  */
    int window;         /* window side (24)                       sam3.cpp:86  */
    int n_global;       /* global blocks (4)                      sam3.cpp:87  */
    int global_idx[4];  /* {7, 15, 23, 31}                        sam3.cpp:88  */
    int pos_grid;       /* pos_embed grid (24 = img/patch/3)      sam3.cpp:2534 */
    int neck_dim;       /* 256                                    sam3.cpp:95  */
    int wtype;          /* ggml type of the 4 linear weights per block */
} orc_vit_hparams;

typedef struct {
    const float *norm1_w, *norm1_b, *norm2_w, *norm2_b;  /* [E] */
    const void *qkv_w;  const float *qkv_b;   /* ggml [E, 3E] (3E rows of E), [3E] */
    const void *proj_w; const float *proj_b;  /* [E, E], [E] */
    const void *fc1_w;  const float *fc1_b;   /* [E, mlp], [mlp] */
    const void *fc2_w;  const float *fc2_b;   /* [mlp, E], [E] */
    const float *freqs;                       /* [2, 32, N] = N x 32 (cos, sin) pairs */
} orc_vit_block_w;

typedef struct {
    const float *dc1_w, *dc1_b;  /* ConvT 2x2 s2: ggml [2, 2, Cout, Cin] (scales 0, 1) */
    const float *dc2_w, *dc2_b;  /* second ConvT of scale 0 */
    const float *c1_w, *c1_b;    /* conv 1x1: ggml [1, 1, Cin, Cout] */
    const float *c3_w, *c3_b;    /* conv 3x3 pad 1: ggml [3, 3, Cin, Cout] */
} orc_neck_scale_w;

typedef struct {
    const float *patch_w;              /* ggml [p, p, 3, E] */
    const float *pos_embed;            /* ggml [E, g, g] */
    const float *ln_pre_w, *ln_pre_b;  /* [E] */
    orc_vit_block_w blocks[64];
    orc_neck_scale_w neck[4];
} orc_vit_w;

/* sam3_preprocess_image (sam3.cpp:3490-3518, resize :3445-3485):
 * uint8 HWC (w x h) -> f32 CHW img x img, (p/255 - 0.5)/0.5 */
void orc_preprocess_sam3(const uint8_t *rgb, int w, int h, int img, float *out_chw);

/* sam2_preprocess_image (sam3.cpp:3522-3548): ImageNet mean/std. */
void orc_preprocess_sam2(const uint8_t *rgb, int w, int h, int img, float *out_chw);

/* ggml_norm over rows of n (sam3_layer_norm, sam3.cpp:1041-1051) then * w + b */
void orc_layer_norm(const float *x, float *y, int64_t rows, int n, float eps, const float *w, const float *b,
                    int n_threads);

/* sam3_build_vit_prefix_graph (sam3.cpp:3810-3834): image CHW -> x [T][E] */
void orc_vit_prefix(const orc_vit_hparams *hp, const orc_vit_w *vw, const float *img_chw, float *x, int n_threads);

/* sam3_vit_block_forward (sam3.cpp:3714-3805), in place on x [T][E] */
void orc_vit_block(const orc_vit_hparams *hp, const orc_vit_block_w *bw, int block_idx, float *x, int n_threads);

/* stage helpers of the block, exposed for per-stage parity tests */
void orc_win_part(const float *x, float *y, int E, int W, int H, int ws);     /* ggml_win_part   */
void orc_win_unpart(const float *y, float *x, int E, int W, int H, int ws);   /* ggml_win_unpart */
/* qkv [B*N][3E] -> RoPE'd Q, K and V as [B][heads][N][64] (sam3.cpp:3747-3776) */
void orc_qkv_split_rope(const float *qkv, const float *freqs, int B, int N, int E, int heads, float *q, float *k,
                        float *v);
/* ggml_flash_attn_ext without mask: out [B][N][heads*64] (sam3.cpp:3778-3781) */
/* 1: orc_attention computes in float64 (a second valid evaluation); 0: float32 (default). */
void orc_set_attention_f64(int on);
void orc_attention(const float *q, const float *k, const float *v, int B, int N, int heads, float scale, float *out,
                   int n_threads);
void orc_gelu_erf(float *x, int64_t n);

/* sam3_build_neck_graph (sam3.cpp:3867-3925): x [T][E] (T = g*g) -> out[i]
 * as [C][W][H] token-major [(w + W*h)*C + c], C = neck_dim, W = H = g*4, g*2, g, g/2 */
void orc_neck(const orc_vit_hparams *hp, const orc_neck_scale_w *nw, const float *x, float *out[4], int n_threads);

#ifdef __cplusplus
}
#endif
#endif
