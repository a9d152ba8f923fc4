// sam_dec.cu -- the SAM prompt encoder + mask decoder on the B200 backend: the
// graph sam3_segment_pvs builds (sam3.cpp:10765-11115; prompt tokens
// :10365-10398, positional encodings :10273-10363, decoder graph
// sam3_build_sam_dec_graph :10548-10763, two-way block :10442-10509,
// attention :10168-10271) executed as a fixed sequence of kernels.
//
//   tokens  = [obj_score?, iou, mask x4, sparse prompt embeddings]   (queries, and their PE)
//   keys    = image features + no_mem_embed + no-mask dense embedding  (key PE: dense sine grid)
//   depth x two-way block: self-attn (block 0: no PE, no residual), LN;
//             token->image cross-attn, LN; MLP (ReLU), LN; image->token cross-attn, LN (keys)
//   final token->image attention, LN
//   upscale: ConvT 2x2 s2 (D -> 64) + conv_s1(feat_s1), LayerNorm2d, GELU;
//            ConvT 2x2 s2 (64 -> 32) + conv_s0(feat_s0), GELU
//   masks   = hypernetwork MLP(mask token m) . upscaled embedding     (4 maps of 4H x 4H)
//   iou     = sigmoid(MLP(iou token)), obj = MLP(obj token)
// Linear layers go through run_mul_mat (the exact quantised MUL_MAT for
// Q8_0/Q4_0/Q4_1 weights, fp16 GEMM for F16/F32); attention through
// attention_simt (head dims 32 and 16); the transposed convolutions through
// the CONV_TRANSPOSE_2D op (F16 kernel, as ggml_cast does at sam3.cpp:1087);
// the 1x1 high-resolution convolutions keep their F32 kernels in fp32.
#include "../../include/sam3_b200.h"
#include "attn_simt.cuh"
#include "model_util.h"
#include "row_norm.cuh"
#include "sgemm.cuh"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

namespace b200 {
namespace {

constexpr int DEC_SPLITS = 32;  // key ranges of the token -> image attentions (x 8 heads = 256 CTAs)

inline unsigned nblocks(int64_t n, int per) { return static_cast<unsigned>((n + per - 1) / per); }

// c = a + b (+ per-column vectors v1, v2 when given): rows x D
// (c may alias a or b)
__global__ void add_kernel(const float *a, const float *b, const float *__restrict__ v1, const float *__restrict__ v2,
                           int64_t rows, int D, float *c) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= rows * D) return;
    const int d = static_cast<int>(i % D);
    float v = b ? __fadd_rn(a[i], b[i]) : a[i];
    if (v1) v = __fadd_rn(v, v1[d]);
    if (v2) v = __fadd_rn(v, v2[d]);
    c[i] = v;
}

// act: 1 ReLU, 2 GELU (erf form), 3 sigmoid -- in place, optionally after a per-row-channel bias
// (channel-major [C][P]: bias[c] with c = i / P)
__global__ void act_kernel(float *__restrict__ x, int64_t n, int act, const float *__restrict__ cbias, int64_t P) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float v = x[i];
    if (cbias) v = __fadd_rn(v, cbias[i / P]);
    if (act == 1) v = fmaxf(v, 0.0f);
    else if (act == 2) v = __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, erff(__fmul_rn(v, 0.70710678118654752440f))));
    else if (act == 3) v = 1.0f / (1.0f + expf(-v));
    x[i] = v;
}

// token-major [P][C] -> channel-major [C][P]
__global__ void to_channels_kernel(const float *__restrict__ x, int64_t P, int C, float *__restrict__ y) {
    __shared__ float tile[32][33];
    const int64_t p0 = static_cast<int64_t>(blockIdx.x) * 32;
    const int c0 = blockIdx.y * 32, tx = threadIdx.x, ty = threadIdx.y;
    for (int j = ty; j < 32; j += 8) {
        const int64_t p = p0 + j;
        const int c = c0 + tx;
        tile[j][tx] = (p < P && c < C) ? x[p * C + c] : 0.f;
    }
    __syncthreads();
    for (int j = ty; j < 32; j += 8) {
        const int c = c0 + j;
        const int64_t p = p0 + tx;
        if (c < C && p < P) y[static_cast<int64_t>(c) * P + p] = tile[tx][j];
    }
}

// masks[m][p] = sum_c hyp[m][c] * up[c][p] (ggml_mul_mat(up_flat, hyper), sam3.cpp:10710)
__global__ void hyper_masks_kernel(const float *__restrict__ hyp, int nm, const float *__restrict__ up, int64_t P,
                                   float *__restrict__ masks) {
    __shared__ float hs[4 * 32];
    for (int i = threadIdx.x; i < nm * 32; i += blockDim.x) hs[i] = hyp[i];
    __syncthreads();
    const int64_t p = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (p >= P) return;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int c = 0; c < 32; ++c) {
        const float v = up[static_cast<int64_t>(c) * P + p];
        for (int m = 0; m < nm; ++m) acc[m] = fmaf(hs[m * 32 + c], v, acc[m]);
    }
    for (int m = 0; m < nm; ++m) masks[static_cast<int64_t>(m) * P + p] = acc[m];
}

// Bilinear resize (half-pixel centres, clamped, double coordinates) of a mask
// of logits and the 0 threshold (sam3_bilinear_interpolate, sam3.cpp:9617-9643,
// and the binarisation at :11071-11075): dst 255 / 0.
__global__ void mask_resize_kernel(const float *__restrict__ src, int sw, int sh, int dw, int dh,
                                   uint8_t *__restrict__ dst) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<int64_t>(dw) * dh) return;
    const int x = static_cast<int>(i % dw), y = static_cast<int>(i / dw);
    double fy = (y + 0.5) * (static_cast<double>(sh) / dh) - 0.5;
    fy = fmax(0.0, fmin(fy, static_cast<double>(sh - 1)));
    const int y0 = min(static_cast<int>(fy), sh - 2), y1 = y0 + 1;
    const float wy = static_cast<float>(fy - y0);
    double fx = (x + 0.5) * (static_cast<double>(sw) / dw) - 0.5;
    fx = fmax(0.0, fmin(fx, static_cast<double>(sw - 1)));
    const int x0 = min(static_cast<int>(fx), sw - 2), x1 = x0 + 1;
    const float wx = static_cast<float>(fx - x0);
    const float v = (1 - wy) * ((1 - wx) * src[y0 * sw + x0] + wx * src[y0 * sw + x1]) +
                    wy * ((1 - wx) * src[y1 * sw + x0] + wx * src[y1 * sw + x1]);
    dst[i] = v > 0.0f ? 255 : 0;
}

}  // namespace

// The same resize + binarisation for another owner of a decoder mask (the video tracker's kept masks).
cudaError_t launch_mask_resize(const float *src, int S, int out_w, int out_h, uint8_t *dst, cudaStream_t s) {
    const int64_t n = static_cast<int64_t>(out_w) * out_h;
    mask_resize_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(src, S, S, out_w, out_h, dst);
    return cudaGetLastError();
}

namespace {

struct DecAttn {
    sam3b200_weight *q = nullptr, *k = nullptr, *v = nullptr, *o = nullptr;
    DevBuf qb, kb, vb, ob;
    int id = 0;  // internal dim
};

struct DecBlock {
    DecAttn sa, t2i, i2t;
    DevBuf n1w, n1b, n2w, n2b, n3w, n3b, n4w, n4b, fc1b, fc2b;
    sam3b200_weight *fc1 = nullptr, *fc2 = nullptr;
};

struct Mlp3 {
    sam3b200_weight *w[3] = {nullptr, nullptr, nullptr};
    DevBuf b[3];
};

}  // namespace

struct SamDec {
    Backend *be = nullptr;
    sam3b200_sam_dec_hparams hp{};
    int H = 0, D = 0, nmask = 0, nspecial = 0, ntok_max = 0;
    std::vector<DecBlock> blk;
    DecAttn final_attn;
    DevBuf final_nw, final_nb, special_tokens;  // [nspecial][D]: obj?, iou, masks
    std::vector<float> tok_obj, tok_iou, tok_masks;
    DevBuf up1_w16, up1_b, up1_nw, up1_nb, up2_w16, up2_b, cs0_w, cs0_b, cs1_w, cs1_b, no_mem;
    Mlp3 hyper[4], iou_head, obj_head;
    // prompt encoder (host copies: the sparse embeddings are formed on the host per call)
    std::vector<float> pe_gauss, point_emb[4], not_a_point, no_mask;
    DevBuf dense_pe, no_mask_dev, track_tok;  // track_tok: the token rows of a propagated frame's decode
    std::vector<std::string> missing;
    // activations
    DevBuf tok, qpe, q2, keys, kpe, k2, tq, tk, tv, to, tmp_tok, tmp_keys, mlp, cm, up1, up1b, hs1, up2, hs0,
        hyp, masks, heads_tmp;
    DevBuf part_o, part_ml;  // split-over-keys partials of the token -> image attentions
    float iou[4] = {0, 0, 0, 0}, obj = 0;
    int ntok = 0;
};

namespace {

bool dlaunched(SamDec *d, cudaError_t e, const char *what, int n = 1) {
    d->be->count(n);
    return cuda_ok(e, what);
}

bool lin(SamDec *d, const sam3b200_weight *w, const float *x, int64_t ldx, int64_t M, const DevBuf &b, float *y,
         int64_t ldy) {
    return run_mul_mat(d->be, reinterpret_cast<const Weight *>(w), x, ldx, M, b.as<float>(), y, ldy, nullptr) ==
           SAM3B200_STATUS_SUCCESS;
}

// sam3_sam_attention: projections, 8-head attention, output projection -> out [nq][D]
bool attention(SamDec *d, const DecAttn &a, const float *q_in, int nq, const float *k_in, int nk, const float *v_in,
               float *out) {
    const int D = d->D, ID = a.id, HD = ID / d->hp.heads;
    if (!lin(d, a.q, q_in, D, nq, a.qb, d->tq.as<float>(), ID) || !lin(d, a.k, k_in, D, nk, a.kb, d->tk.as<float>(), ID) ||
        !lin(d, a.v, v_in, D, nk, a.vb, d->tv.as<float>(), ID))
        return false;
    const AttnStrides qs{static_cast<int64_t>(nq) * ID, HD, ID}, ks{static_cast<int64_t>(nk) * ID, HD, ID};
    // the prompt tokens against the 4096 image tokens: a handful of query rows per head, so the keys
    // are split over DEC_SPLITS CTAs per head and merged by the combine pass
    const int splits = nq <= d->ntok_max && nk >= 64 * DEC_SPLITS && HD <= 32 ? DEC_SPLITS : 1;
    const float scale = 1.0f / sqrtf(static_cast<float>(HD));
    if (!dlaunched(d,
                   splits > 1 ? attention_simt_split(HD, d->tq.as<float>(), qs, nq, d->tk.as<float>(), ks,
                                                     d->tv.as<float>(), ks, nk, 1, d->hp.heads, scale,
                                                     d->to.as<float>(), qs, splits, d->part_o.as<float>(),
                                                     d->part_ml.as<float2>(), d->be->stream)
                              : attention_simt(HD, d->tq.as<float>(), qs, nq, d->tk.as<float>(), ks, d->tv.as<float>(),
                                               ks, nk, 1, d->hp.heads, nullptr, 0, scale, d->to.as<float>(), qs,
                                               d->be->stream),
                   "sam_dec attention", splits > 1 ? 2 : 1))
        return false;
    return lin(d, a.o, d->to.as<float>(), ID, nq, a.ob, out, D);
}

bool add(SamDec *d, const float *a, const float *b, int64_t rows, float *c, const float *v1 = nullptr,
         const float *v2 = nullptr) {
    add_kernel<<<nblocks(rows * d->D, 256), 256, 0, d->be->stream>>>(a, b, v1, v2, rows, d->D, c);
    return dlaunched(d, cudaGetLastError(), "sam_dec add");
}

bool ln(SamDec *d, const float *x, int rows, const DevBuf &w, const DevBuf &b, float *y) {
    ln_rows_kernel<<<nblocks(rows, 8), 256, 0, d->be->stream>>>(x, rows, d->D, w.as<float>(), b.as<float>(), 1e-5f, y);
    return dlaunched(d, cudaGetLastError(), "sam_dec ln");
}

bool act(SamDec *d, float *x, int64_t n, int a, const float *cbias = nullptr, int64_t P = 1) {
    act_kernel<<<nblocks(n, 256), 256, 0, d->be->stream>>>(x, n, a, cbias, P);
    return dlaunched(d, cudaGetLastError(), "sam_dec act");
}

bool mlp3(SamDec *d, const Mlp3 &m, const float *x, int out_dim, float *y, bool sigmoid) {
    float *t0 = d->heads_tmp.as<float>(), *t1 = t0 + d->D;
    return lin(d, m.w[0], x, d->D, 1, m.b[0], t0, d->D) && act(d, t0, d->D, 1) &&
           lin(d, m.w[1], t0, d->D, 1, m.b[1], t1, d->D) && act(d, t1, d->D, 1) &&
           lin(d, m.w[2], t1, d->D, 1, m.b[2], y, out_dim) && (!sigmoid || act(d, y, out_dim, 3));
}

// sam3_twoway_block_forward (sam3.cpp:10442-10509) on tok [ntok][D], keys [HH][D]
bool twoway(SamDec *d, const DecBlock &b, bool skip_pe) {
    const int nt = d->ntok, HH = d->H * d->H;
    float *tok = d->tok.as<float>(), *keys = d->keys.as<float>(), *q2 = d->q2.as<float>(), *k2 = d->k2.as<float>();
    float *tt = d->tmp_tok.as<float>();
    // 1. self-attention
    if (skip_pe) {
        if (!attention(d, b.sa, tok, nt, tok, nt, tok, tt) || !ln(d, tt, nt, b.n1w, b.n1b, tok)) return false;
    } else {
        if (!add(d, tok, d->qpe.as<float>(), nt, q2) || !attention(d, b.sa, q2, nt, q2, nt, tok, tt) ||
            !add(d, tok, tt, nt, tt) || !ln(d, tt, nt, b.n1w, b.n1b, tok))
            return false;
    }
    // 2. token -> image
    if (!add(d, tok, d->qpe.as<float>(), nt, q2) || !add(d, keys, d->kpe.as<float>(), HH, k2) ||
        !attention(d, b.t2i, q2, nt, k2, HH, keys, tt) || !add(d, tok, tt, nt, tt) || !ln(d, tt, nt, b.n2w, b.n2b, tok))
        return false;
    // 3. MLP (ReLU)
    float *mh = d->mlp.as<float>();
    if (!lin(d, b.fc1, tok, d->D, nt, b.fc1b, mh, d->hp.mlp_dim) || !act(d, mh, static_cast<int64_t>(nt) * d->hp.mlp_dim, 1) ||
        !lin(d, b.fc2, mh, d->hp.mlp_dim, nt, b.fc2b, tt, d->D) || !add(d, tok, tt, nt, tt) ||
        !ln(d, tt, nt, b.n3w, b.n3b, tok))
        return false;
    // 4. image -> token (keys updated)
    float *tk = d->tmp_keys.as<float>();
    return add(d, tok, d->qpe.as<float>(), nt, q2) && add(d, keys, d->kpe.as<float>(), HH, k2) &&
           attention(d, b.i2t, k2, HH, q2, nt, tok, tk) && add(d, keys, tk, HH, tk) &&
           ln(d, tk, HH, b.n4w, b.n4b, keys);
}

// 1x1 convolution with an F32 kernel (ggml_conv_2d_sk_p0 on the high-resolution
// features, sam3.cpp:10658, 10678) in fp32: out[oc][p] = add[oc][p] + (sum_c w[oc][c]
// x[p][c] + bias[oc]), x token-major [P][D] as the encoder hands it over, out
// channel-major.  An f32 GEMM (one fma per channel in channel order, then the bias,
// then the upscaled map).
bool conv1x1(SamDec *d, const float *x_tok, int64_t P, int OC, const DevBuf &w, const DevBuf &b, const float *add_cm,
             float *out) {
    if (!dlaunched(d, sgemm_nt(w.as<float>(), d->D, 1, x_tok, d->D, 1, OC, static_cast<int>(P), d->D, b.as<float>(),
                               out, P, false, d->be->stream, false, true),
                   "sam_dec conv1x1"))
        return false;
    const int64_t n = static_cast<int64_t>(OC) * P;
    if (n % d->D != 0) return dlaunched(d, cudaErrorInvalidValue, "sam_dec conv1x1 add");
    return add(d, add_cm, out, n / d->D, out);
}

bool to_channels(SamDec *d, const float *x, int64_t P, int C, float *y) {
    dim3 grid(nblocks(P, 32), nblocks(C, 32));
    to_channels_kernel<<<grid, dim3(32, 8), 0, d->be->stream>>>(x, P, C, y);
    return dlaunched(d, cudaGetLastError(), "sam_dec transpose");
}

// add_no_mem: the PVS decode adds no_mem_embed to the image features (sam3.cpp:10926-10936); a
// propagated frame's memory-conditioned features go in without it (sam3.cpp:11296-11335).
bool decode(SamDec *d, const float *img, const float *fs0, const float *fs1, bool add_no_mem = true) {
    const int D = d->D, H = d->H, HH = H * H;
    const int64_t P1 = static_cast<int64_t>(2 * H) * 2 * H, P0 = static_cast<int64_t>(4 * H) * 4 * H;
    cudaStream_t s = d->be->stream;
    auto *hb = reinterpret_cast<sam3b200_backend *>(d->be);
    // keys = image features (+ no_mem_embed) + no-mask dense embedding; key PE = dense grid
    if (!add(d, img, nullptr, HH, d->keys.as<float>(), add_no_mem ? d->no_mem.as<float>() : nullptr,
             d->no_mask_dev.as<float>()) ||
        !cuda_ok(cudaMemcpyAsync(d->kpe.p, d->dense_pe.p, static_cast<size_t>(HH) * D * 4, cudaMemcpyDeviceToDevice, s),
                 "kpe"))
        return false;
    for (size_t i = 0; i < d->blk.size(); ++i)
        if (!twoway(d, d->blk[i], i == 0)) return false;
    // final token -> image attention
    const int nt = d->ntok;
    float *tok = d->tok.as<float>(), *tt = d->tmp_tok.as<float>();
    if (!add(d, tok, d->qpe.as<float>(), nt, d->q2.as<float>()) ||
        !add(d, d->keys.as<float>(), d->kpe.as<float>(), HH, d->k2.as<float>()) ||
        !attention(d, d->final_attn, d->q2.as<float>(), nt, d->k2.as<float>(), HH, d->keys.as<float>(), tt) ||
        !add(d, tok, tt, nt, tt) || !ln(d, tt, nt, d->final_nw, d->final_nb, tok))
        return false;
    // upscaling: keys (token-major) -> channel-major; ConvT (D -> 64) + bias + conv_s1(feat_s1); LN2d; GELU
    float *cm = d->cm.as<float>(), *up1 = d->up1.as<float>();
    if (!to_channels(d, d->keys.as<float>(), HH, D, cm) ||
        sam3b200_conv_transpose_2d(hb, d->up1_w16.p, cm, H, H, D, 64, 2, 2, 2, up1) != SAM3B200_STATUS_SUCCESS ||
        !act(d, up1, 64 * P1, 0, d->up1_b.as<float>(), P1) ||
        !conv1x1(d, fs1, P1, 64, d->cs1_w, d->cs1_b, up1, d->up1b.as<float>()))
        return false;
    ln_channels_kernel<<<nblocks(P1, 256), 256, 0, s>>>(d->up1b.as<float>(), 64, P1, d->up1_nw.as<float>(),
                                                        d->up1_nb.as<float>(), 1e-6f, up1);
    if (!dlaunched(d, cudaGetLastError(), "sam_dec ln2d") || !act(d, up1, 64 * P1, 2)) return false;
    // ConvT (64 -> 32) + bias + conv_s0(feat_s0); GELU
    float *up2 = d->up2.as<float>();
    if (sam3b200_conv_transpose_2d(hb, d->up2_w16.p, up1, 2 * H, 2 * H, 64, 32, 2, 2, 2, d->hs0.as<float>()) !=
            SAM3B200_STATUS_SUCCESS ||
        !act(d, d->hs0.as<float>(), 32 * P0, 0, d->up2_b.as<float>(), P0) ||
        !conv1x1(d, fs0, P0, 32, d->cs0_w, d->cs0_b, d->hs0.as<float>(), up2) || !act(d, up2, 32 * P0, 2))
        return false;
    // hypernetworks on the mask tokens, masks, IoU and object heads
    const int s0 = d->hp.pred_obj_scores ? 1 : 0;
    float *hyp = d->hyp.as<float>();
    for (int m = 0; m < d->nmask; ++m)
        if (!mlp3(d, d->hyper[m], tok + static_cast<int64_t>(s0 + 1 + m) * D, 32, hyp + m * 32, false)) return false;
    hyper_masks_kernel<<<nblocks(P0, 256), 256, 0, s>>>(hyp, d->nmask, up2, P0, d->masks.as<float>());
    if (!dlaunched(d, cudaGetLastError(), "sam_dec masks")) return false;
    float *heads_out = d->hyp.as<float>() + 4 * 32;  // iou [nmask], obj [1]
    if (!mlp3(d, d->iou_head, tok + static_cast<int64_t>(s0) * D, d->nmask, heads_out, true)) return false;
    if (d->hp.pred_obj_scores && !mlp3(d, d->obj_head, tok, 1, heads_out + 4, false)) return false;
    float hbuf[5] = {0, 0, 0, 0, 10.0f};  // no object-score head: logit 10 (sam3.cpp:10752-10758)
    if (!cuda_ok(cudaMemcpyAsync(hbuf, heads_out, (d->hp.pred_obj_scores ? 5 : 4) * sizeof(float),
                                 cudaMemcpyDeviceToHost, s),
                 "heads") ||
        !cuda_ok(cudaStreamSynchronize(s), "sam_dec sync"))
        return false;
    for (int m = 0; m < 4; ++m) d->iou[m] = m < d->nmask ? hbuf[m] : 0.f;
    d->obj = hbuf[4];
    return true;
}

// random Fourier encoding of a normalised point (sam3_pe_encode_coord, sam3.cpp:10273-10287)
void pe_encode(const std::vector<float> &g, float xn, float yn, float *out) {
    const int n = static_cast<int>(g.size() / 2);
    const float cx = 2.0f * xn - 1.0f, cy = 2.0f * yn - 1.0f;
    for (int i = 0; i < n; ++i) {
        float dot = cx * g[i] + cy * g[n + i];
        dot *= 2.0f * static_cast<float>(M_PI);
        out[i] = sinf(dot);
        out[i + n] = cosf(dot);
    }
}

bool make_dense(SamDec *d) {
    const int D = d->D, H = d->H;
    std::vector<float> grid(static_cast<size_t>(D) * H * H), pe(D);
    for (int r = 0; r < H; ++r)
        for (int c = 0; c < H; ++c) {
            pe_encode(d->pe_gauss, (c + 0.5f) / H, (r + 0.5f) / H, pe.data());
            for (int k = 0; k < D; ++k) grid[(static_cast<size_t>(r) * H + c) * D + k] = pe[k];
        }
    return upload(d->dense_pe, grid.data(), grid.size() * 4, d->be->stream);
}

bool check_ready(SamDec *d) {
    d->missing.clear();
    auto need = [&](bool ok, const std::string &n) {
        if (!ok) d->missing.push_back(n);
    };
    need(!d->tok_iou.empty() && !d->tok_masks.empty() && (!d->hp.pred_obj_scores || !d->tok_obj.empty()),
         "sam_dec.{iou_token,mask_tokens,obj_score_token}");
    need(d->dense_pe.p != nullptr, "sam_pe.pe_gaussian");
    need(!d->not_a_point.empty() && d->no_mask_dev.p, "sam_pe.{not_a_point,no_mask}_embed");
    for (int i = 0; i < 4; ++i) need(!d->point_emb[i].empty(), "sam_pe.point_embeddings." + std::to_string(i));
    need(d->no_mem.p != nullptr, "no_mem_embed");
    auto attn_ok = [](const DecAttn &a) { return a.q && a.k && a.v && a.o && a.qb.p && a.kb.p && a.vb.p && a.ob.p; };
    for (size_t i = 0; i < d->blk.size(); ++i) {
        const DecBlock &b = d->blk[i];
        const std::string p = "sam_dec.twoway." + std::to_string(i);
        need(attn_ok(b.sa) && attn_ok(b.t2i) && attn_ok(b.i2t), p + " attention");
        need(b.n1w.p && b.n1b.p && b.n2w.p && b.n2b.p && b.n3w.p && b.n3b.p && b.n4w.p && b.n4b.p, p + " norms");
        need(b.fc1 && b.fc2 && b.fc1b.p && b.fc2b.p, p + ".mlp");
    }
    need(attn_ok(d->final_attn) && d->final_nw.p && d->final_nb.p, "sam_dec.final_attn/final_norm");
    need(d->up1_w16.p && d->up1_b.p && d->up1_nw.p && d->up1_nb.p && d->up2_w16.p && d->up2_b.p, "sam_dec.upscale");
    need(d->cs0_w.p && d->cs0_b.p && d->cs1_w.p && d->cs1_b.p, "sam_dec.conv_s0/conv_s1");
    auto mlp_ok = [](const Mlp3 &m) { return m.w[0] && m.w[1] && m.w[2] && m.b[0].p && m.b[1].p && m.b[2].p; };
    for (int m = 0; m < d->nmask; ++m) need(mlp_ok(d->hyper[m]), "sam_dec.hyper." + std::to_string(m));
    need(mlp_ok(d->iou_head), "sam_dec.iou_prediction_head");
    if (d->hp.pred_obj_scores) need(mlp_ok(d->obj_head), "sam_dec.pred_obj_score_head");
    if (!d->missing.empty()) {
        set_error("sam_dec: %zu tensors missing (first: %s)", d->missing.size(), d->missing[0].c_str());
        return false;
    }
    return true;
}

void free_w(SamDec *d, sam3b200_weight *&w) {
    if (w) sam3b200_weight_free(reinterpret_cast<sam3b200_backend *>(d->be), w);
    w = nullptr;
}

}  // namespace
}  // namespace b200

using namespace b200;

sam3b200_sam_dec *sam3b200_sam_dec_create(sam3b200_backend *hb, const sam3b200_sam_dec_hparams *hp) {
    auto *be = reinterpret_cast<Backend *>(hb);
    if (!be || !hp) return nullptr;
    if (hp->feat_size <= 1 || hp->embed != 256 || hp->heads != 8 || hp->depth <= 0 || hp->mlp_dim <= 0 ||
        hp->mlp_dim % 32 != 0 || hp->n_multimask < 0 || hp->n_multimask > 3 || hp->max_points <= 0 ||
        hp->max_points > 64) {
        set_error("sam_dec_create: unsupported hyperparameters (embed 256, 8 heads, <= 4 mask tokens)");
        return nullptr;
    }
    cudaSetDevice(be->device);
    auto *d = new SamDec();
    d->be = be;
    d->hp = *hp;
    d->H = hp->feat_size;
    d->D = hp->embed;
    d->nmask = hp->n_multimask + 1;
    d->nspecial = (hp->pred_obj_scores ? 2 : 1) + d->nmask;
    d->ntok_max = d->nspecial + hp->max_points;
    d->blk.resize(hp->depth);
    for (auto &b : d->blk) {
        b.sa.id = 256;
        b.t2i.id = 128;
        b.i2t.id = 128;
    }
    d->final_attn.id = 128;
    const size_t D = d->D, HH = static_cast<size_t>(d->H) * d->H, NT = d->ntok_max;
    const size_t P1 = 4 * HH, P0 = 16 * HH;
    const bool ok = d->tok.alloc(NT * D * 4) && d->qpe.alloc(NT * D * 4) && d->q2.alloc(NT * D * 4) &&
                    d->keys.alloc(HH * D * 4) && d->kpe.alloc(HH * D * 4) && d->k2.alloc(HH * D * 4) &&
                    d->tq.alloc(HH * D * 4) && d->tk.alloc(HH * D * 4) && d->tv.alloc(HH * D * 4) &&
                    d->to.alloc(HH * D * 4) && d->tmp_tok.alloc(NT * D * 4) && d->tmp_keys.alloc(HH * D * 4) &&
                    d->mlp.alloc(NT * hp->mlp_dim * 4) && d->cm.alloc(HH * D * 4) && d->up1.alloc(64 * P1 * 4) &&
                    d->up1b.alloc(64 * P1 * 4) && d->up2.alloc(32 * P0 * 4) &&
                    d->hs0.alloc(32 * P0 * 4) && d->hyp.alloc((4 * 32 + 8) * 4) && d->masks.alloc(4 * P0 * 4) &&
                    d->heads_tmp.alloc(2 * D * 4) &&
                    d->part_o.alloc(static_cast<size_t>(DEC_SPLITS) * hp->heads * NT * 32 * 4) &&
                    d->part_ml.alloc(static_cast<size_t>(DEC_SPLITS) * hp->heads * NT * 8);
    if (!ok) {
        delete d;
        return nullptr;
    }
    return reinterpret_cast<sam3b200_sam_dec *>(d);
}

void sam3b200_sam_dec_free(sam3b200_sam_dec *hd) {
    auto *d = reinterpret_cast<SamDec *>(hd);
    if (!d) return;
    cudaSetDevice(d->be->device);
    cudaStreamSynchronize(d->be->stream);
    auto free_attn = [&](DecAttn &a) {
        free_w(d, a.q);
        free_w(d, a.k);
        free_w(d, a.v);
        free_w(d, a.o);
    };
    for (auto &b : d->blk) {
        free_attn(b.sa);
        free_attn(b.t2i);
        free_attn(b.i2t);
        free_w(d, b.fc1);
        free_w(d, b.fc2);
    }
    free_attn(d->final_attn);
    for (auto *m : {&d->hyper[0], &d->hyper[1], &d->hyper[2], &d->hyper[3], &d->iou_head, &d->obj_head})
        for (auto &w : m->w) free_w(d, w);
    delete d;
}

int sam3b200_sam_dec_set_tensor(sam3b200_sam_dec *hd, const char *name_c, int type, const void *data, const int64_t *ne) {
    auto *d = reinterpret_cast<SamDec *>(hd);
    if (!d || !name_c || !data || !ne) return SAM3B200_STATUS_FAILED;
    cudaSetDevice(d->be->device);
    auto *hb = reinterpret_cast<sam3b200_backend *>(d->be);
    cudaStream_t s = d->be->stream;
    const std::string name(name_c);
    const int64_t n = ne[0] * (ne[1] > 0 ? ne[1] : 1) * (ne[2] > 0 ? ne[2] : 1) * (ne[3] > 0 ? ne[3] : 1);
    std::vector<float> f;
    auto host = [&](std::vector<float> &dst, int64_t want) -> int {
        if (n != want || !to_f32(type, data, n, f)) {
            set_error("%s: %lld elements of type %d, expected %lld F32/F16", name_c, (long long)n, type,
                      (long long)want);
            return SAM3B200_STATUS_FAILED;
        }
        dst = f;
        return SAM3B200_STATUS_SUCCESS;
    };
    auto vec = [&](DevBuf &dst, int64_t want) -> int {
        std::vector<float> v;
        if (host(v, want) != SAM3B200_STATUS_SUCCESS) return SAM3B200_STATUS_FAILED;
        return upload(dst, v.data(), v.size() * 4, s) ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
    };
    auto f16 = [&](DevBuf &dst, int64_t want) -> int {
        std::vector<float> v;
        if (host(v, want) != SAM3B200_STATUS_SUCCESS) return SAM3B200_STATUS_FAILED;
        return upload_f16(dst, v, s) ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
    };
    auto weight = [&](sam3b200_weight *&w, int64_t K, int64_t N) -> int {
        if (ne[0] != K || ne[1] != N) {
            set_error("%s: shape [%lld, %lld], expected [%lld, %lld]", name_c, (long long)ne[0], (long long)ne[1],
                      (long long)K, (long long)N);
            return SAM3B200_STATUS_FAILED;
        }
        free_w(d, w);
        w = sam3b200_weight_upload(hb, type, data, K, N);
        return w ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
    };
    const int64_t D = d->D;
    auto attn = [&](DecAttn &a, const std::string &r) -> int {
        if (r == "q_proj.weight") return weight(a.q, D, a.id);
        if (r == "k_proj.weight") return weight(a.k, D, a.id);
        if (r == "v_proj.weight") return weight(a.v, D, a.id);
        if (r == "out_proj.weight") return weight(a.o, a.id, D);
        if (r == "q_proj.bias") return vec(a.qb, a.id);
        if (r == "k_proj.bias") return vec(a.kb, a.id);
        if (r == "v_proj.bias") return vec(a.vb, a.id);
        if (r == "out_proj.bias") return vec(a.ob, D);
        return -100;
    };
    auto mlp = [&](Mlp3 &m, const std::string &r, int last_out) -> int {
        if (r.size() < 9 || r.compare(0, 7, "layers.") != 0) return -100;
        const int j = r[7] - '0';
        if (j < 0 || j > 2) return -100;
        const std::string t = r.substr(8);
        const int out = j == 2 ? last_out : static_cast<int>(D);
        if (t == ".weight") return weight(m.w[j], D, out);
        if (t == ".bias") return vec(m.b[j], out);
        return -100;
    };
    int st = -100;
    if (name == "sam_dec.iou_token.weight") st = host(d->tok_iou, D);
    else if (name == "sam_dec.mask_tokens.weight") st = host(d->tok_masks, D * d->nmask);
    else if (name == "sam_dec.obj_score_token.weight") st = host(d->tok_obj, D);
    else if (name == "sam_dec.final_norm.weight") st = vec(d->final_nw, D);
    else if (name == "sam_dec.final_norm.bias") st = vec(d->final_nb, D);
    else if (name == "sam_dec.upscale.0.weight") st = f16(d->up1_w16, 2 * 2 * 64 * D);  // ggml_cast to F16
    else if (name == "sam_dec.upscale.0.bias") st = vec(d->up1_b, 64);
    else if (name == "sam_dec.upscale.1.weight") st = vec(d->up1_nw, 64);
    else if (name == "sam_dec.upscale.1.bias") st = vec(d->up1_nb, 64);
    else if (name == "sam_dec.upscale.3.weight") st = f16(d->up2_w16, 2 * 2 * 32 * 64);
    else if (name == "sam_dec.upscale.3.bias") st = vec(d->up2_b, 32);
    else if (name == "sam_dec.conv_s0.weight") st = vec(d->cs0_w, D * 32);
    else if (name == "sam_dec.conv_s0.bias") st = vec(d->cs0_b, 32);
    else if (name == "sam_dec.conv_s1.weight") st = vec(d->cs1_w, D * 64);
    else if (name == "sam_dec.conv_s1.bias") st = vec(d->cs1_b, 64);
    else if (name == "no_mem_embed") st = vec(d->no_mem, D);
    else if (name == "sam_pe.pe_gaussian") {
        st = host(d->pe_gauss, D);
        if (st == SAM3B200_STATUS_SUCCESS && !make_dense(d)) st = SAM3B200_STATUS_FAILED;
    } else if (name == "sam_pe.not_a_point_embed.weight") st = host(d->not_a_point, D);
    else if (name == "sam_pe.no_mask_embed.weight") {
        st = host(d->no_mask, D);
        if (st == SAM3B200_STATUS_SUCCESS && !upload(d->no_mask_dev, d->no_mask.data(), D * 4, s))
            st = SAM3B200_STATUS_FAILED;
    } else if (name.rfind("sam_pe.point_embeddings.", 0) == 0 && name.size() == 32 &&
               name.compare(25, 7, ".weight") == 0 && name[24] >= '0' && name[24] <= '3') {
        st = host(d->point_emb[name[24] - '0'], D);
    } else if (name.rfind("sam_dec.final_attn.", 0) == 0) {
        st = attn(d->final_attn, name.substr(19));
    } else if (name.rfind("sam_dec.hyper.", 0) == 0 && name.size() > 16) {
        const int m = name[14] - '0';
        if (m >= 0 && m < d->nmask && name[15] == '.') st = mlp(d->hyper[m], name.substr(16), 32);
    } else if (name.rfind("sam_dec.iou_prediction_head.", 0) == 0) {
        st = mlp(d->iou_head, name.substr(28), d->nmask);
    } else if (name.rfind("sam_dec.pred_obj_score_head.", 0) == 0) {
        st = mlp(d->obj_head, name.substr(28), 1);
    } else if (name.rfind("sam_dec.twoway.", 0) == 0) {
        const int i = atoi(name.c_str() + 15);
        if (i >= 0 && i < static_cast<int>(d->blk.size())) {
            DecBlock &b = d->blk[i];
            const std::string r = name.substr(name.find('.', 15) + 1);
            if (r.rfind("sa.", 0) == 0) st = attn(b.sa, r.substr(3));
            else if (r.rfind("cross_attn_token_to_image.", 0) == 0) st = attn(b.t2i, r.substr(26));
            else if (r.rfind("cross_attn_image_to_token.", 0) == 0) st = attn(b.i2t, r.substr(26));
            else if (r == "norm1.weight") st = vec(b.n1w, D);
            else if (r == "norm1.bias") st = vec(b.n1b, D);
            else if (r == "norm2.weight") st = vec(b.n2w, D);
            else if (r == "norm2.bias") st = vec(b.n2b, D);
            else if (r == "norm3.weight") st = vec(b.n3w, D);
            else if (r == "norm3.bias") st = vec(b.n3b, D);
            else if (r == "norm4.weight") st = vec(b.n4w, D);
            else if (r == "norm4.bias") st = vec(b.n4b, D);
            else if (r == "mlp.lin1.weight") st = weight(b.fc1, D, d->hp.mlp_dim);
            else if (r == "mlp.lin1.bias") st = vec(b.fc1b, d->hp.mlp_dim);
            else if (r == "mlp.lin2.weight") st = weight(b.fc2, d->hp.mlp_dim, D);
            else if (r == "mlp.lin2.bias") st = vec(b.fc2b, D);
        }
    }
    if (st == -100) {
        set_error("sam_dec: unknown tensor %s", name_c);
        return SAM3B200_STATUS_FAILED;
    }
    return st;
}

int sam3b200_sam_dec_missing(sam3b200_sam_dec *hd, char *buf, int cap) {
    auto *d = reinterpret_cast<SamDec *>(hd);
    if (!d) return -1;
    check_ready(d);
    std::string all;
    for (const auto &m : d->missing) all += m + "\n";
    if (buf && cap > 0) snprintf(buf, static_cast<size_t>(cap), "%s", all.c_str());
    return static_cast<int>(d->missing.size());
}

int sam3b200_sam_dec_run(sam3b200_sam_dec *hd, const float *img_feats_dev, const float *feat_s0_dev,
                         const float *feat_s1_dev, const float *coords, const int32_t *labels, int n_prompts,
                         int orig_w, int orig_h, int img_size) {
    auto *d = reinterpret_cast<SamDec *>(hd);
    if (!d || !img_feats_dev || !feat_s0_dev || !feat_s1_dev || (n_prompts > 0 && (!coords || !labels)) ||
        n_prompts < 1 || n_prompts + 1 > d->hp.max_points || orig_w <= 0 || orig_h <= 0 || img_size <= 0) {
        set_error("sam_dec_run: bad arguments (1 <= prompts < max_points)");
        return SAM3B200_STATUS_FAILED;
    }
    for (int p = 0; p < n_prompts; ++p)
        if (labels[p] < 0 || labels[p] > 3) {
            set_error("sam_dec_run: label %d (0 negative, 1 positive, 2/3 box corners)", labels[p]);
            return SAM3B200_STATUS_FAILED;
        }
    cudaSetDevice(d->be->device);
    if (!check_ready(d)) return SAM3B200_STATUS_FAILED;
    const int D = d->D, npts = n_prompts + 1;  // + the padding token (sam3_collect_pvs_prompt_tokens)
    d->ntok = d->nspecial + npts;
    std::vector<float> tok(static_cast<size_t>(d->ntok) * D), pe(D);
    size_t o = 0;
    if (d->hp.pred_obj_scores) std::copy(d->tok_obj.begin(), d->tok_obj.end(), tok.begin() + (o++) * D);
    std::copy(d->tok_iou.begin(), d->tok_iou.end(), tok.begin() + (o++) * D);
    std::copy(d->tok_masks.begin(), d->tok_masks.end(), tok.begin() + o * D);
    o += d->nmask;
    for (int p = 0; p < npts; ++p, ++o) {
        float *dst = tok.data() + o * D;
        if (p == n_prompts) {  // padding point: label -1
            std::copy(d->not_a_point.begin(), d->not_a_point.end(), dst);
            continue;
        }
        const float px = coords[2 * p] / static_cast<float>(orig_w) * static_cast<float>(img_size) + 0.5f;
        const float py = coords[2 * p + 1] / static_cast<float>(orig_h) * static_cast<float>(img_size) + 0.5f;
        pe_encode(d->pe_gauss, px / static_cast<float>(img_size), py / static_cast<float>(img_size), pe.data());
        for (int k = 0; k < D; ++k) dst[k] = pe[k] + d->point_emb[labels[p]][k];
    }
    const size_t bytes = tok.size() * 4;
    if (!cuda_ok(cudaMemcpyAsync(d->tok.p, tok.data(), bytes, cudaMemcpyHostToDevice, d->be->stream), "tokens") ||
        !cuda_ok(cudaMemcpyAsync(d->qpe.p, tok.data(), bytes, cudaMemcpyHostToDevice, d->be->stream), "tokens") ||
        !cuda_ok(cudaStreamSynchronize(d->be->stream), "tokens sync"))
        return SAM3B200_STATUS_FAILED;
    return decode(d, img_feats_dev, feat_s0_dev, feat_s1_dev) ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
}

int sam3b200_sam_dec_run_tracking(sam3b200_sam_dec *hd, const float *cond_feats_dev, const float *feat_s0_dev,
                                  const float *feat_s1_dev) {
    auto *d = reinterpret_cast<SamDec *>(hd);
    if (!d || !cond_feats_dev || !feat_s0_dev || !feat_s1_dev) {
        set_error("sam_dec_run_tracking: null argument");
        return SAM3B200_STATUS_FAILED;
    }
    cudaSetDevice(d->be->device);
    if (!check_ready(d)) return SAM3B200_STATUS_FAILED;
    // tokens: [obj_score?, iou, masks x n, not_a_point] -- the single padding token of sam3_propagate_single;
    // the same every frame, so they are formed once and kept on the device
    const int D = d->D;
    d->ntok = d->nspecial + 1;
    const size_t bytes = static_cast<size_t>(d->ntok) * D * 4;
    if (!d->track_tok.p) {
        std::vector<float> tok(static_cast<size_t>(d->ntok) * D);
        size_t o = 0;
        if (d->hp.pred_obj_scores) std::copy(d->tok_obj.begin(), d->tok_obj.end(), tok.begin() + (o++) * D);
        std::copy(d->tok_iou.begin(), d->tok_iou.end(), tok.begin() + (o++) * D);
        std::copy(d->tok_masks.begin(), d->tok_masks.end(), tok.begin() + o * D);
        o += d->nmask;
        std::copy(d->not_a_point.begin(), d->not_a_point.end(), tok.begin() + o * D);
        if (!upload(d->track_tok, tok.data(), bytes, d->be->stream)) return SAM3B200_STATUS_FAILED;
    }
    if (!cuda_ok(cudaMemcpyAsync(d->tok.p, d->track_tok.p, bytes, cudaMemcpyDeviceToDevice, d->be->stream), "tokens") ||
        !cuda_ok(cudaMemcpyAsync(d->qpe.p, d->track_tok.p, bytes, cudaMemcpyDeviceToDevice, d->be->stream), "tokens"))
        return SAM3B200_STATUS_FAILED;
    return decode(d, cond_feats_dev, feat_s0_dev, feat_s1_dev, false) ? SAM3B200_STATUS_SUCCESS
                                                                       : SAM3B200_STATUS_FAILED;
}

int sam3b200_sam_dec_mask_token(sam3b200_sam_dec *hd, int m, const float **dev) {
    auto *d = reinterpret_cast<SamDec *>(hd);
    if (!d || d->ntok == 0 || m < 0 || m >= d->nmask || !dev) {
        set_error("sam_dec_mask_token: no decode yet or token %d out of range", m);
        return SAM3B200_STATUS_FAILED;
    }
    *dev = d->tok.as<float>() + (d->hp.pred_obj_scores ? 2 + m : 1 + m) * d->D;
    return SAM3B200_STATUS_SUCCESS;
}

int sam3b200_sam_dec_outputs(sam3b200_sam_dec *hd, const float **masks_dev, float iou[4], float *obj_logit,
                             const float **sam_token_dev) {
    auto *d = reinterpret_cast<SamDec *>(hd);
    if (!d || d->ntok == 0) return SAM3B200_STATUS_FAILED;
    if (masks_dev) *masks_dev = d->masks.as<float>();
    if (iou)
        for (int m = 0; m < 4; ++m) iou[m] = d->iou[m];
    if (obj_logit) *obj_logit = d->obj;
    if (sam_token_dev) *sam_token_dev = d->tok.as<float>() + (d->hp.pred_obj_scores ? 2 : 1) * d->D;
    return SAM3B200_STATUS_SUCCESS;
}

int sam3b200_sam_dec_mask(sam3b200_sam_dec *hd, int m, int out_w, int out_h, uint8_t *dst_dev) {
    auto *d = reinterpret_cast<SamDec *>(hd);
    if (!d || d->ntok == 0 || m < 0 || m >= d->nmask || out_w <= 0 || out_h <= 0 || !dst_dev)
        return SAM3B200_STATUS_FAILED;
    cudaSetDevice(d->be->device);
    const int S = 4 * d->H;
    mask_resize_kernel<<<nblocks(static_cast<int64_t>(out_w) * out_h, 256), 256, 0, d->be->stream>>>(
        d->masks.as<float>() + static_cast<int64_t>(m) * S * S, S, S, out_w, out_h, dst_dev);
    return dlaunched(d, cudaGetLastError(), "sam_dec mask") ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
}
