/*
 * vit_oracle.c -- CPU restatement of the SAM3 visual encoder (TEST
 * INFRASTRUCTURE ONLY; see vit_oracle.h).  Each function names the
 * sam3.cpp lines whose ggml graph it evaluates.
 */
#include "vit_oracle.h"
#include "ggml_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

static float r16(float v) { return orc_fp16_to_fp32(orc_fp32_to_fp16(v)); }

/* ---- preprocessing: sam3.cpp:3445-3485 (resize), 3490-3518 (normalise) --- */
static void resize_bilinear(const uint8_t *src, int sw, int sh, uint8_t *dst, int dw, int dh) {
    const double sx = (double)sw / dw, sy = (double)sh / dh;
    for (int y = 0; y < dh; ++y) {
        double fy = (y + 0.5) * sy - 0.5;
        if (fy < 0.0) fy = 0.0;
        const int y0 = (int)fy, y1 = (y0 < sh - 1) ? y0 + 1 : y0;
        const double wy = fy - y0, wy0 = 1.0 - wy;
        for (int x = 0; x < dw; ++x) {
            double fx = (x + 0.5) * sx - 0.5;
            if (fx < 0.0) fx = 0.0;
            const int x0 = (int)fx, x1 = (x0 < sw - 1) ? x0 + 1 : x0;
            const double wx = fx - x0, wx0 = 1.0 - wx;
            for (int c = 0; c < 3; ++c) {
                const double p00 = src[(y0 * sw + x0) * 3 + c], p01 = src[(y0 * sw + x1) * 3 + c];
                const double p10 = src[(y1 * sw + x0) * 3 + c], p11 = src[(y1 * sw + x1) * 3 + c];
                const double v = wy0 * (wx0 * p00 + wx * p01) + wy * (wx0 * p10 + wx * p11);
                int iv = (int)(v + 0.5);
                if (iv < 0) iv = 0;
                if (iv > 255) iv = 255;
                dst[(y * dw + x) * 3 + c] = (uint8_t)iv;
            }
        }
    }
}

void orc_preprocess_sam3(const uint8_t *rgb, int w, int h, int img, float *out) {
    uint8_t *tmp = NULL;
    const uint8_t *px = rgb;
    if (w != img || h != img) {
        tmp = (uint8_t *)malloc((size_t)img * img * 3);
        resize_bilinear(rgb, w, h, tmp, img, img);
        px = tmp;
    }
    for (int c = 0; c < 3; ++c)
        for (int y = 0; y < img; ++y)
            for (int x = 0; x < img; ++x) {
                const float v = px[(y * img + x) * 3 + c] / 255.0f;
                out[(size_t)c * img * img + (size_t)y * img + x] = (v - 0.5f) / 0.5f;
            }
    free(tmp);
}

/* sam2_preprocess_image, sam3.cpp:3522-3548: the same resize, ImageNet
 * normalisation (v - mean[c]) / std[c] with v = p / 255.0f. */
void orc_preprocess_sam2(const uint8_t *rgb, int w, int h, int img, float *out) {
    static const float mean[3] = {0.485f, 0.456f, 0.406f};
    static const float std_d[3] = {0.229f, 0.224f, 0.225f};
    uint8_t *tmp = NULL;
    const uint8_t *px = rgb;
    if (w != img || h != img) {
        tmp = (uint8_t *)malloc((size_t)img * img * 3);
        resize_bilinear(rgb, w, h, tmp, img, img);
        px = tmp;
    }
    for (int c = 0; c < 3; ++c)
        for (int y = 0; y < img; ++y)
            for (int x = 0; x < img; ++x) {
                const float v = px[(y * img + x) * 3 + c] / 255.0f;
                out[(size_t)c * img * img + (size_t)y * img + x] = (v - mean[c]) / std_d[c];
            }
    free(tmp);
}

/* ---- ggml_norm + affine: sam3.cpp:1041-1051 ---------------------------- */
void orc_layer_norm(const float *x, float *y, int64_t rows, int n, float eps, const float *w, const float *b,
                    int n_threads) {
    #pragma omp parallel for num_threads(n_threads) schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const float *xr = x + r * n;
        float *yr = y + r * n;
        double sum = 0.0;
        for (int i = 0; i < n; ++i) sum += xr[i];
        const float mean = (float)(sum / n);
        double sum2 = 0.0;
        for (int i = 0; i < n; ++i) {
            const float v = xr[i] - mean;
            yr[i] = v;
            sum2 += (double)(v * v);
        }
        const float variance = (float)(sum2 / n);
        const float scale = 1.0f / sqrtf(variance + eps);
        for (int i = 0; i < n; ++i) {
            float v = yr[i] * scale;
            if (w) v = v * w[i];
            if (b) v = v + b[i];
            yr[i] = v;
        }
    }
}

/* ---- prefix: sam3.cpp:3810-3834 ---------------------------------------- */
void orc_vit_prefix(const orc_vit_hparams *hp, const orc_vit_w *vw, const float *img, float *x, int n_threads) {
    const int p = hp->patch, E = hp->E, G = hp->img / p, S = hp->img, g = hp->pos_grid;
    const int K = 3 * p * p;
    /* ggml_conv_2d_sk_p0 = im2col (c, ky, kx) + f32 mul_mat */
    #pragma omp parallel num_threads(n_threads)
    {
        float *col = (float *)malloc(sizeof(float) * K);
        #pragma omp for schedule(static)
        for (int t = 0; t < G * G; ++t) {
            const int px = t % G, py = t / G;
            for (int c = 0; c < 3; ++c)
                for (int ky = 0; ky < p; ++ky)
                    for (int kx = 0; kx < p; ++kx)
                        col[(c * p + ky) * p + kx] = img[(size_t)c * S * S + (size_t)(py * p + ky) * S + px * p + kx];
            for (int e = 0; e < E; ++e) {
                const float *wr = vw->patch_w + (size_t)e * K;
                float s = 0.f;
                for (int k = 0; k < K; ++k) s = fmaf(col[k], wr[k], s);
                /* + ggml_repeat(pos_embed) tile, sam3.cpp:3823-3827 */
                const int gw = px % g, gh = py % g;
                x[(size_t)t * E + e] = s + vw->pos_embed[(size_t)(gw + g * gh) * E + e];
            }
        }
        free(col);
    }
    orc_layer_norm(x, x, (int64_t)G * G, E, 1e-5f, vw->ln_pre_w, vw->ln_pre_b, n_threads);
}

/* ---- ggml_win_part / ggml_win_unpart (no padding: W, H multiples of ws) -- */
void orc_win_part(const float *x, float *y, int E, int W, int H, int ws) {
    const int npx = W / ws, npy = H / ws;
    for (int py = 0; py < npy; ++py)
        for (int px = 0; px < npx; ++px)
            for (int i2 = 0; i2 < ws; ++i2)
                for (int i1 = 0; i1 < ws; ++i1) {
                    const int b = py * npx + px, n = i1 + ws * i2;
                    const int t = (px * ws + i1) + W * (py * ws + i2);
                    memcpy(y + ((size_t)b * ws * ws + n) * E, x + (size_t)t * E, sizeof(float) * E);
                }
}

void orc_win_unpart(const float *y, float *x, int E, int W, int H, int ws) {
    const int npx = W / ws, npy = H / ws;
    for (int py = 0; py < npy; ++py)
        for (int px = 0; px < npx; ++px)
            for (int i2 = 0; i2 < ws; ++i2)
                for (int i1 = 0; i1 < ws; ++i1) {
                    const int b = py * npx + px, n = i1 + ws * i2;
                    const int t = (px * ws + i1) + W * (py * ws + i2);
                    memcpy(x + (size_t)t * E, y + ((size_t)b * ws * ws + n) * E, sizeof(float) * E);
                }
}

/* ---- qkv split + head permute + RoPE: sam3.cpp:3747-3776, 3671-3710 ---- */
void orc_qkv_split_rope(const float *qkv, const float *freqs, int B, int N, int E, int heads, float *q, float *k,
                        float *v) {
    const int HD = E / heads;
    for (int b = 0; b < B; ++b)
        for (int n = 0; n < N; ++n) {
            const float *row = qkv + ((size_t)b * N + n) * 3 * E;
            for (int h = 0; h < heads; ++h) {
                const size_t o = (((size_t)b * heads + h) * N + n) * HD;
                for (int i = 0; i < HD / 2; ++i) {
                    const float c = freqs ? freqs[((size_t)n * (HD / 2) + i) * 2 + 0] : 1.f;
                    const float s = freqs ? freqs[((size_t)n * (HD / 2) + i) * 2 + 1] : 0.f;
                    const float qr = row[h * HD + 2 * i], qi = row[h * HD + 2 * i + 1];
                    const float kr = row[E + h * HD + 2 * i], ki = row[E + h * HD + 2 * i + 1];
                    if (freqs) {
                        /* out_re = x_re*cos - x_im*sin, out_im = x_re*sin + x_im*cos,
                         * each product rounded (separate ggml_mul nodes) */
                        q[o + 2 * i] = qr * c - qi * s;
                        q[o + 2 * i + 1] = qr * s + qi * c;
                        k[o + 2 * i] = kr * c - ki * s;
                        k[o + 2 * i + 1] = kr * s + ki * c;
                    } else {
                        q[o + 2 * i] = qr; q[o + 2 * i + 1] = qi;
                        k[o + 2 * i] = kr; k[o + 2 * i + 1] = ki;
                    }
                }
                for (int d = 0; d < HD; ++d) v[o + d] = row[2 * E + h * HD + d];
            }
        }
}

/* ---- attention: softmax(q k^T * scale) v, f32 (ggml_flash_attn_ext, F32 K/V) */
/* Arithmetic of orc_attention: 0 = float32 (the default, as ggml's CPU backend
 * computes an F32 FLASH_ATTN_EXT), 1 = float64 throughout.  The float64 form is
 * a second, equally valid evaluation of the same graph; the tests use the
 * distance between the two to measure how far a rounding-level change in
 * attention carries through the quantised blocks. */
static int g_attn_f64 = 0;

void orc_set_attention_f64(int on) { g_attn_f64 = on ? 1 : 0; }

static void attention_f64(const float *q, const float *k, const float *v, int B, int N, int heads, float scale,
                          float *out, int n_threads) {
    const int HD = 64;
    #pragma omp parallel num_threads(n_threads)
    {
        double *s = (double *)malloc(sizeof(double) * N);
        double acc[64];
        #pragma omp for collapse(2) schedule(static)
        for (int bh = 0; bh < B * heads; ++bh)
            for (int n = 0; n < N; ++n) {
                const float *qr = q + ((size_t)bh * N + n) * HD;
                const float *kb = k + (size_t)bh * N * HD;
                const float *vb = v + (size_t)bh * N * HD;
                double mx = -INFINITY;
                for (int m = 0; m < N; ++m) {
                    double d = 0.0;
                    for (int i = 0; i < HD; ++i) d += (double)qr[i] * kb[(size_t)m * HD + i];
                    s[m] = d * scale;
                    if (s[m] > mx) mx = s[m];
                }
                double sum = 0.0;
                for (int i = 0; i < HD; ++i) acc[i] = 0.0;
                for (int m = 0; m < N; ++m) {
                    const double e = exp(s[m] - mx);
                    sum += e;
                    for (int i = 0; i < HD; ++i) acc[i] += e * vb[(size_t)m * HD + i];
                }
                const int b = bh / heads, h = bh % heads;
                float *o = out + ((size_t)b * N + n) * heads * HD + h * HD;
                for (int i = 0; i < HD; ++i) o[i] = (float)(acc[i] / sum);
            }
        free(s);
    }
}

void orc_attention(const float *q, const float *k, const float *v, int B, int N, int heads, float scale, float *out,
                   int n_threads) {
    const int HD = 64;
    if (g_attn_f64) {
        attention_f64(q, k, v, B, N, heads, scale, out, n_threads);
        return;
    }
    #pragma omp parallel num_threads(n_threads)
    {
        float *s = (float *)malloc(sizeof(float) * N);
        float acc[64];
        #pragma omp for collapse(2) schedule(static)
        for (int bh = 0; bh < B * heads; ++bh)
            for (int n = 0; n < N; ++n) {
                const float *qr = q + ((size_t)bh * N + n) * HD;
                const float *kb = k + (size_t)bh * N * HD;
                const float *vb = v + (size_t)bh * N * HD;
                float mx = -INFINITY;
                for (int m = 0; m < N; ++m) {
                    float d = 0.f;
                    for (int i = 0; i < HD; ++i) d = fmaf(qr[i], kb[(size_t)m * HD + i], d);
                    s[m] = d * scale;
                    if (s[m] > mx) mx = s[m];
                }
                double sum = 0.0;
                for (int i = 0; i < HD; ++i) acc[i] = 0.f;
                for (int m = 0; m < N; ++m) {
                    const float e = expf(s[m] - mx);
                    sum += e;
                    for (int i = 0; i < HD; ++i) acc[i] = fmaf(e, vb[(size_t)m * HD + i], acc[i]);
                }
                const int b = bh / heads, h = bh % heads;
                float *o = out + ((size_t)b * N + n) * heads * HD + h * HD;
                for (int i = 0; i < HD; ++i) o[i] = acc[i] / (float)sum;
            }
        free(s);
    }
}

void orc_gelu_erf(float *x, int64_t n) {
    for (int64_t i = 0; i < n; ++i) x[i] = 0.5f * x[i] * (1.0f + erff(x[i] * 0.70710678118654752440f));
}

static void add_bias_rows(float *y, const float *b, int64_t rows, int n) {
    if (!b) return;
    for (int64_t r = 0; r < rows; ++r)
        for (int i = 0; i < n; ++i) y[r * n + i] = y[r * n + i] + b[i];
}

static int is_global(const orc_vit_hparams *hp, int idx) {
    for (int i = 0; i < hp->n_global; ++i)
        if (hp->global_idx[i] == idx) return 1;
    return 0;
}

/* ---- block: sam3.cpp:3714-3805 ------------------------------------------ */
void orc_vit_block(const orc_vit_hparams *hp, const orc_vit_block_w *bw, int idx, float *x, int nt) {
    const int E = hp->E, G = hp->img / hp->patch, T = G * G, heads = hp->heads;
    const int glob = is_global(hp, idx);
    const int ws = hp->window;
    const int B = glob ? 1 : (G / ws) * (G / ws);
    const int N = glob ? T : ws * ws;
    float *xn = (float *)malloc(sizeof(float) * (size_t)T * E);
    float *xw = (float *)malloc(sizeof(float) * (size_t)T * E);
    float *qkv = (float *)malloc(sizeof(float) * (size_t)T * 3 * E);
    float *q = (float *)malloc(sizeof(float) * (size_t)T * E);
    float *k = (float *)malloc(sizeof(float) * (size_t)T * E);
    float *v = (float *)malloc(sizeof(float) * (size_t)T * E);
    float *att = (float *)malloc(sizeof(float) * (size_t)T * E);
    float *hid = (float *)malloc(sizeof(float) * (size_t)T * hp->mlp);

    orc_layer_norm(x, xn, T, E, 1e-5f, bw->norm1_w, bw->norm1_b, nt);
    const float *src = xn;
    if (!glob) {
        orc_win_part(xn, xw, E, G, G, ws);
        src = xw;
    }
    orc_mul_mat(hp->wtype, bw->qkv_w, E, 3 * E, src, E, T, qkv, 3 * E, nt);
    add_bias_rows(qkv, bw->qkv_b, T, 3 * E);
    orc_qkv_split_rope(qkv, bw->freqs, B, N, E, heads, q, k, v);
    orc_attention(q, k, v, B, N, heads, 1.0f / sqrtf((float)(E / heads)), att, nt);
    orc_mul_mat(hp->wtype, bw->proj_w, E, E, att, E, T, xw, E, nt);
    add_bias_rows(xw, bw->proj_b, T, E);
    const float *pr = xw;
    if (!glob) {
        orc_win_unpart(xw, xn, E, G, G, ws);
        pr = xn;
    }
    for (size_t i = 0; i < (size_t)T * E; ++i) x[i] = x[i] + pr[i];

    orc_layer_norm(x, xn, T, E, 1e-5f, bw->norm2_w, bw->norm2_b, nt);
    orc_mul_mat(hp->wtype, bw->fc1_w, E, hp->mlp, xn, E, T, hid, hp->mlp, nt);
    add_bias_rows(hid, bw->fc1_b, T, hp->mlp);
    orc_gelu_erf(hid, (int64_t)T * hp->mlp);
    orc_mul_mat(hp->wtype, bw->fc2_w, hp->mlp, E, hid, hp->mlp, T, xw, E, nt);
    add_bias_rows(xw, bw->fc2_b, T, E);
    for (size_t i = 0; i < (size_t)T * E; ++i) x[i] = x[i] + xw[i];

    free(xn); free(xw); free(qkv); free(q); free(k); free(v); free(att); free(hid);
}

/* ---- neck: sam3.cpp:3867-3925 ------------------------------------------- */
/* ConvTranspose 2x2 stride 2 with ggml's F16 kernel cast and F16 input
 * (sam3_conv_transpose_weight, sam3.cpp:1087-1090); products of fp16
 * values, summed in fp32.  in/out are HWC. */
static void convt2x2(const float *in, int W, int H, int Cin, const float *w, const float *b, int Cout, float *out,
                     int nt) {
    const int OW = 2 * W;
    float *w16 = (float *)malloc(sizeof(float) * (size_t)4 * Cout * Cin);  /* [ky][kx][co][ci] */
    for (int ci = 0; ci < Cin; ++ci)
        for (int co = 0; co < Cout; ++co)
            for (int ky = 0; ky < 2; ++ky)
                for (int kx = 0; kx < 2; ++kx)
                    w16[(((size_t)ky * 2 + kx) * Cout + co) * Cin + ci] =
                        r16(w[kx + 2 * (ky + 2 * (co + (size_t)Cout * ci))]);
    #pragma omp parallel num_threads(nt)
    {
        float *row = (float *)malloc(sizeof(float) * Cin);
        #pragma omp for schedule(static)
        for (int p = 0; p < W * H; ++p) {
            const int ix = p % W, iy = p / W;
            for (int ci = 0; ci < Cin; ++ci) row[ci] = r16(in[(size_t)p * Cin + ci]);
            for (int ky = 0; ky < 2; ++ky)
                for (int kx = 0; kx < 2; ++kx)
                    for (int co = 0; co < Cout; ++co) {
                        const float *wr = w16 + (((size_t)ky * 2 + kx) * Cout + co) * Cin;
                        float s = 0.f;
                        for (int ci = 0; ci < Cin; ++ci) s = fmaf(row[ci], wr[ci], s);
                        out[((size_t)(2 * iy + ky) * OW + 2 * ix + kx) * Cout + co] = s + b[co];
                    }
        }
        free(row);
    }
    free(w16);
}

/* conv kxk stride 1, padding k/2, f32 (im2col + f32 mul_mat), HWC */
static void conv_same(const float *in, int W, int H, int Cin, int ks, const float *w, const float *b, int Cout,
                      float *out, int nt) {
    const int pad = ks / 2, K = ks * ks * Cin;
    #pragma omp parallel num_threads(nt)
    {
        float *col = (float *)malloc(sizeof(float) * K);  /* ggml im2col order (ci, ky, kx) */
        #pragma omp for schedule(static)
        for (int p = 0; p < W * H; ++p) {
            const int x = p % W, y = p / W;
            for (int ci = 0; ci < Cin; ++ci)
                for (int ky = 0; ky < ks; ++ky)
                    for (int kx = 0; kx < ks; ++kx) {
                        const int sx = x + kx - pad, sy = y + ky - pad;
                        col[(ci * ks + ky) * ks + kx] =
                            (sx < 0 || sy < 0 || sx >= W || sy >= H) ? 0.f : in[((size_t)sy * W + sx) * Cin + ci];
                    }
            for (int co = 0; co < Cout; ++co) {
                const float *wr = w + (size_t)co * K;
                float s = 0.f;
                for (int kk = 0; kk < K; ++kk) s = fmaf(col[kk], wr[kk], s);
                out[(size_t)p * Cout + co] = s + b[co];
            }
        }
        free(col);
    }
}

void orc_neck(const orc_vit_hparams *hp, const orc_neck_scale_w *nw, const float *x, float *out[4], int nt) {
    const int E = hp->E, G = hp->img / hp->patch, D = hp->neck_dim, MID = 512;
    /* scale 0: ConvT(E->512) GELU ConvT(512->D) conv1x1 conv3x3 at 4G */
    {
        float *a = (float *)malloc(sizeof(float) * (size_t)4 * G * G * MID);
        float *c = (float *)malloc(sizeof(float) * (size_t)16 * G * G * D);
        float *d = (float *)malloc(sizeof(float) * (size_t)16 * G * G * D);
        convt2x2(x, G, G, E, nw[0].dc1_w, nw[0].dc1_b, MID, a, nt);
        orc_gelu_erf(a, (int64_t)4 * G * G * MID);
        convt2x2(a, 2 * G, 2 * G, MID, nw[0].dc2_w, nw[0].dc2_b, D, c, nt);
        conv_same(c, 4 * G, 4 * G, D, 1, nw[0].c1_w, nw[0].c1_b, D, d, nt);
        conv_same(d, 4 * G, 4 * G, D, 3, nw[0].c3_w, nw[0].c3_b, D, out[0], nt);
        free(a); free(c); free(d);
    }
    /* scale 1: ConvT(E->512) conv1x1(512->D) conv3x3 at 2G */
    {
        float *a = (float *)malloc(sizeof(float) * (size_t)4 * G * G * MID);
        float *c = (float *)malloc(sizeof(float) * (size_t)4 * G * G * D);
        convt2x2(x, G, G, E, nw[1].dc1_w, nw[1].dc1_b, MID, a, nt);
        conv_same(a, 2 * G, 2 * G, MID, 1, nw[1].c1_w, nw[1].c1_b, D, c, nt);
        conv_same(c, 2 * G, 2 * G, D, 3, nw[1].c3_w, nw[1].c3_b, D, out[1], nt);
        free(a); free(c);
    }
    /* scale 2: conv1x1(E->D) conv3x3 at G */
    {
        float *c = (float *)malloc(sizeof(float) * (size_t)G * G * D);
        conv_same(x, G, G, E, 1, nw[2].c1_w, nw[2].c1_b, D, c, nt);
        conv_same(c, G, G, D, 3, nw[2].c3_w, nw[2].c3_b, D, out[2], nt);
        free(c);
    }
    /* scale 3: maxpool 2x2 s2, conv1x1(E->D) conv3x3 at G/2 */
    {
        const int g = G / 2;
        float *mp = (float *)malloc(sizeof(float) * (size_t)g * g * E);
        float *c = (float *)malloc(sizeof(float) * (size_t)g * g * D);
        for (int y = 0; y < g; ++y)
            for (int xx = 0; xx < g; ++xx)
                for (int e = 0; e < E; ++e) {
                    float m = x[((size_t)(2 * y) * G + 2 * xx) * E + e];
                    const float v1 = x[((size_t)(2 * y) * G + 2 * xx + 1) * E + e];
                    const float v2 = x[((size_t)(2 * y + 1) * G + 2 * xx) * E + e];
                    const float v3 = x[((size_t)(2 * y + 1) * G + 2 * xx + 1) * E + e];
                    if (v1 > m) m = v1;
                    if (v2 > m) m = v2;
                    if (v3 > m) m = v3;
                    mp[((size_t)y * g + xx) * E + e] = m;
                }
        conv_same(mp, g, g, E, 1, nw[3].c1_w, nw[3].c1_b, D, c, nt);
        conv_same(c, g, g, D, 3, nw[3].c3_w, nw[3].c3_b, D, out[3], nt);
        free(mp); free(c);
    }
}
