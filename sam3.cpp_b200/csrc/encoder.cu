// encoder.cu -- the SAM3 visual encoder on the B200 backend: the graph that
// sam3_encode_image builds for a visual-only SAM3 model (sam3.cpp:6028-6149:
// preprocess, ViT prefix, 32 ViT blocks, tracker SimpleFPN neck) executed
// as a fixed sequence of fused kernels on the backend stream.
//
// Weights arrive by reference tensor name (sam3.cpp:2529-2600) in ggml
// layout and are stored in device layouts: the four linear weights of each
// block repacked for the MMQ (mmq.cuh), F32 convolution weights as fp16
// GEMM operands, the rest as f32.
#include "../../include/sam3_b200.h"
#include "attn.cuh"
#include "backend_impl.h"
#include "gemm_f16.cuh"
#include "mmq.cuh"
#include "vit_ops.cuh"

#include <cuda_fp16.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "model_util.h"

namespace b200 {

struct BlockW {
    DevBuf n1w, n1b, n2w, n2b, qkv_b, proj_b, fc1_b, fc2_b, freqs;
    QWeight qkv, proj, fc1, fc2;
};

struct NeckScaleW {
    DevBuf dc1, dc1_b, dc2, dc2_b, c1, c1_b, c3, c3_b;  // fp16 GEMM operands + f32 biases
};

struct Vit {
    Backend *be = nullptr;
    sam3b200_vit_hparams hp{};
    int G = 0, T = 0, Tpad = 0, KP = 0, MID = 512;
    DevBuf patch_w, pos, lnpre_w, lnpre_b;
    std::vector<BlockW> blk;
    NeckScaleW neck[4];
    NeckScaleW neck_det[4];  // detector neck (full SAM3 models): same graph, its own weights
    bool det_any = false;    // a neck.det tensor was set
    std::vector<std::string> missing;
    // activations
    DevBuf img_u8, img_rs, img_f32, a_patch, conv, x, codes_a, quads_a, codes_b, quads_b, q, k, v, rowmap;
    DevBuf a16, b16;  // DQ16 arithmetic: dequantised A operands, fp16 [T][E] and [T][mlp]
    DevBuf x16, mp16, n_a, n_c, n_d, n_col, out[4], out_det[4];
    int out_side[4] = {0, 0, 0, 0};
    int img_cap = 0;  // pixels of img_u8
    int bcap = 1;     // images the block-loop buffers (x, a16, b16, q, k, v, rowmap) hold, image-major
};

static bool is_global(const sam3b200_vit_hparams &hp, int i) {
    for (int j = 0; j < hp.n_global && j < 4; ++j)
        if (hp.global_idx[j] == i) return true;
    return false;
}

static bool alloc_activations(Vit *v) {
    const auto &hp = v->hp;
    const int E = hp.embed, T = v->T, D = hp.neck_dim, G = v->G;
    const size_t maxk = static_cast<size_t>(hp.mlp > E ? hp.mlp : E);
    bool ok = v->img_f32.alloc(static_cast<size_t>(3) * hp.img * hp.img * 4) &&
              v->a_patch.alloc(static_cast<size_t>(T) * v->KP * 2) && v->conv.alloc(static_cast<size_t>(T) * E * 4) &&
              v->x.alloc(static_cast<size_t>(T) * E * 4) && v->codes_a.alloc(static_cast<size_t>(T) * E) &&
              v->quads_a.alloc(act_quad_bytes(E, v->Tpad)) &&
              v->codes_b.alloc(static_cast<size_t>(T) * maxk) &&
              v->quads_b.alloc(act_quad_bytes(static_cast<int>(maxk), v->Tpad)) &&
              v->a16.alloc(static_cast<size_t>(T) * E * 2) && v->b16.alloc(static_cast<size_t>(T) * hp.mlp * 2) &&
              v->q.alloc(static_cast<size_t>(T) * E * 2) && v->k.alloc(static_cast<size_t>(T) * E * 2) &&
              v->v.alloc(static_cast<size_t>(T) * E * 2) &&
              v->rowmap.alloc(static_cast<size_t>(T) * 4) && v->x16.alloc(static_cast<size_t>(T) * E * 2) &&
              v->mp16.alloc(static_cast<size_t>(T / 4) * E * 2) &&
              v->n_a.alloc(static_cast<size_t>(4) * T * v->MID * 2) &&
              v->n_c.alloc(static_cast<size_t>(16) * T * D * 2) && v->n_d.alloc(static_cast<size_t>(16) * T * D * 2) &&
              v->n_col.alloc(static_cast<size_t>(16) * T * D * 9 * 2);
    const int side[4] = {4 * G, 2 * G, G, G / 2};
    for (int i = 0; i < 4 && ok; ++i) {
        v->out_side[i] = side[i];
        ok = v->out[i].alloc(static_cast<size_t>(side[i]) * side[i] * D * 4);
    }
    if (!ok) return false;
    if (!cuda_ok(cudaMemsetAsync(v->quads_a.p, 0, v->quads_a.n, v->be->stream), "memset") ||
        !cuda_ok(cudaMemsetAsync(v->quads_b.p, 0, v->quads_b.n, v->be->stream), "memset"))
        return false;
    if (hp.window > 0 && G % hp.window == 0)
        if (!cuda_ok(window_rowmap(G, hp.window, v->rowmap.as<int>(), v->be->stream), "rowmap")) return false;
    return cuda_ok(cudaStreamSynchronize(v->be->stream), "alloc sync");
}

// ---- forward pieces ---------------------------------------------------------------
// every kernel launch of the encoder goes through launched(), which counts it
static bool launched(Vit *v, cudaError_t e, const char *what, int n = 1) {
    v->be->count(n);
    return cuda_ok(e, what);
}

static bool mmq(Vit *v, const void *codes, const void *quads, const QWeight &w, int mode, const float *bias,
                float *y, int add, const int *rowmap, void *out_codes, void *out_quads, int gelu) {
    MmqArgs a;
    a.a = QMatrix{codes, quads, v->T, w.K, v->Tpad};
    a.b = QMatrix{w.codes.p, w.quads.p, w.N, w.K, w.ld, w.nib};
    a.bias = bias;
    a.y = y;
    a.ldy = w.N;
    a.dump = nullptr;
    a.err = v->be->err;
    a.add = add;
    a.rowmap = rowmap;
    a.gelu = gelu;
    a.out_codes = out_codes;
    a.out_quads = out_quads;
    a.out_ld = v->Tpad;
    v->be->prof_mark(0);
    const bool ok = launched(v, mmq_tc(a, mode, v->be->num_sms, v->be->stream, v->be->mmq_cvt, v->be->mmq_bn), "mmq");
    v->be->prof_mark(0);
    return ok;
}

// qkv projection with the attention-input epilogue: bias, RoPE, bf16 Q, K and V^T
static bool mmq_qkv(Vit *v, const BlockW &w, int win_tokens) {
    MmqArgs a;
    a.a = QMatrix{v->codes_a.p, v->quads_a.p, v->T, w.qkv.K, v->Tpad};
    a.b = QMatrix{w.qkv.codes.p, w.qkv.quads.p, w.qkv.N, w.qkv.K, w.qkv.ld, w.qkv.nib};
    a.bias = w.qkv_b.as<float>();
    a.y = nullptr;
    a.ldy = 0;
    a.dump = nullptr;
    a.err = v->be->err;
    a.q_out = v->q.p;
    a.k_out = v->k.p;
    a.vt_out = v->v.p;
    a.freqs = w.freqs.p ? w.freqs.as<float>() : nullptr;
    a.win_tokens = win_tokens;
    a.heads = v->hp.heads;
    v->be->prof_mark(0);
    const bool ok =
        launched(v, mmq_tc(a, MMQ_OUT_QKV, v->be->num_sms, v->be->stream, v->be->mmq_cvt, v->be->mmq_bn), "mmq qkv");
    v->be->prof_mark(0);
    return ok;
}

// DQ16 arithmetic (mmq.cuh): the dequantised A operand a16 [T][K] against the
// weight's fp16 copy, with the same epilogue modes
static bool mmq16(Vit *v, int rows, const void *a16, const QWeight &w, int mode, const float *bias, float *y, int add,
                  const int *rowmap, void *out16, int gelu) {
    MmqArgs a;
    a.a = QMatrix{nullptr, nullptr, rows, w.K, rows};
    a.b = QMatrix{nullptr, nullptr, w.N, w.K, w.ld, w.nib};
    a.bias = bias;
    a.y = y;
    a.ldy = w.N;
    a.dump = nullptr;
    a.err = v->be->err;
    a.add = add;
    a.rowmap = rowmap;
    a.gelu = gelu;
    a.out16 = out16;
    v->be->prof_mark(0);
    const bool ok = launched(v, mmq_dq16(a, a16, w.w16.p, mode, v->be->num_sms, v->be->stream), "mmq dq16");
    v->be->prof_mark(0);
    return ok;
}

static bool mmq16_qkv(Vit *v, int rows, const BlockW &w, int win_tokens) {
    MmqArgs a;
    a.a = QMatrix{nullptr, nullptr, rows, w.qkv.K, rows};
    a.b = QMatrix{nullptr, nullptr, w.qkv.N, w.qkv.K, w.qkv.ld, w.qkv.nib};
    a.bias = w.qkv_b.as<float>();
    a.y = nullptr;
    a.ldy = 0;
    a.dump = nullptr;
    a.err = v->be->err;
    a.q_out = v->q.p;
    a.k_out = v->k.p;
    a.vt_out = v->v.p;
    a.freqs = w.freqs.p ? w.freqs.as<float>() : nullptr;
    a.win_tokens = win_tokens;
    a.heads = v->hp.heads;
    v->be->prof_mark(0);
    const bool ok =
        launched(v, mmq_dq16(a, v->a16.p, w.qkv.w16.p, MMQ_OUT_QKV, v->be->num_sms, v->be->stream), "mmq dq16 qkv");
    v->be->prof_mark(0);
    return ok;
}

// LayerNorm + Q8_0 of the residual stream, written dequantised into a16 (one
// kernel for the supported widths, else layernorm_q8 and a dequantising pass)
static bool ln_dq16(Vit *v, int rows, const float *x, const DevBuf &w, const DevBuf &b, int win) {
    const int E = v->hp.embed;
    cudaStream_t s = v->be->stream;
    if (E % 256 == 0 && E <= 1536)
        return launched(v, layernorm_dq16(x, rows, E, w.as<float>(), b.as<float>(), 1e-5f, v->G, win, v->a16.p, s),
                        "ln dq16");
    if (rows != v->T) {
        set_error("vit: batched encode needs an embedding width in {256, 512, ..., 1536}");
        return false;
    }
    return launched(v, layernorm_q8(x, v->T, E, w.as<float>(), b.as<float>(), 1e-5f, v->G, win, v->codes_a.p,
                                    v->quads_a.p, v->Tpad, s),
                    "ln") &&
           launched(v, dequant_act_f16(v->codes_a.p, v->quads_a.p, v->T, E, v->Tpad, v->a16.p, s), "dequant_act_f16");
}

static bool gemm(Vit *v, const void *a, const DevBuf &b, int M, int N, int K, const DevBuf *bias, int gelu,
                 int out_f16, void *out, int store, int win, int cout) {
    GemmF16Args g;
    g.a = a;
    g.b = b.p;
    g.M = M;
    g.N = N;
    g.K = K;
    g.bias = bias ? bias->as<float>() : nullptr;
    g.gelu = gelu;
    g.out_f16 = out_f16;
    g.out = out;
    g.ldo = N;
    g.store = store;
    g.win = win;
    g.cout = cout;
    g.err = v->be->err;
    return launched(v, gemm_f16(g, v->be->num_sms, v->be->stream), "gemm_f16");
}

static bool run_prefix(Vit *v, const float *img_chw, float *x) {
    const auto &hp = v->hp;
    cudaStream_t s = v->be->stream;
    return launched(v, im2col_patch(img_chw, hp.img, hp.patch, v->KP, v->a_patch.p, s), "im2col_patch") &&
           gemm(v, v->a_patch.p, v->patch_w, v->T, hp.embed, v->KP, nullptr, 0, 0, v->conv.p, GEMM_STORE_ROWMAJOR, 0,
                0) &&
           launched(v, add_pos_layernorm(v->conv.as<float>(), v->pos.as<float>(), hp.pos_grid, v->G, hp.embed,
                                     v->lnpre_w.as<float>(), v->lnpre_b.as<float>(), 1e-5f, x, s),
                   "add_pos_layernorm");
}

// run_block with DQ16 linear layers: the same Q8_0 activations as the exact
// path (LayerNorm, attention and fc1's GELU epilogue quantise with ggml's
// rule), each written dequantised as the next fp16 MUL_MAT's operand.
// nimg images stacked image-major in x (nimg * T rows): every kernel of the
// block runs once over all of them (the windows and global blocks of image j
// follow those of image j - 1), so results per image are those of nimg = 1.
static bool run_block_dq16(Vit *v, int i, float *x, int nimg) {
    const auto &hp = v->hp;
    const BlockW &w = v->blk[i];
    cudaStream_t s = v->be->stream;
    const int E = hp.embed, G = v->G, T = v->T, ws = hp.window, rows = nimg * T;
    const bool glob = is_global(hp, i);
    const int B = nimg * (glob ? 1 : (G / ws) * (G / ws));
    const int N = glob ? T : ws * ws;
    AttnOut attn_dq;  // the proj MUL_MAT's operand (window order), written by the attention
    attn_dq.dq16 = v->a16.p;
    return ln_dq16(v, rows, x, w.n1w, w.n1b, glob ? 0 : ws) && mmq16_qkv(v, rows, w, N) &&
           launched(v, flash_attention(v->q.p, v->k.p, v->v.p, B, N, hp.heads,
                                       1.0f / sqrtf(static_cast<float>(E / hp.heads)), attn_dq, v->be->err, s),
                    "attention") &&
           mmq16(v, rows, v->a16.p, w.proj, MMQ_OUT_F32, w.proj_b.as<float>(), x, 1,
                 glob ? nullptr : v->rowmap.as<int>(), nullptr, 0) &&
           ln_dq16(v, rows, x, w.n2w, w.n2b, 0) &&
           mmq16(v, rows, v->a16.p, w.fc1, MMQ_OUT_DQ16, w.fc1_b.as<float>(), nullptr, 0, nullptr, v->b16.p, 1) &&
           mmq16(v, rows, v->b16.p, w.fc2, MMQ_OUT_F32, w.fc2_b.as<float>(), x, 1, nullptr, nullptr, 0);
}

static bool run_block(Vit *v, int i, float *x, int nimg = 1) {
    if (v->be->mmq_arith == SAM3B200_ARITH_DQ16) return run_block_dq16(v, i, x, nimg);
    if (nimg != 1) {
        set_error("vit: batched blocks need the DQ16 arithmetic");
        return false;
    }
    const auto &hp = v->hp;
    const BlockW &w = v->blk[i];
    cudaStream_t s = v->be->stream;
    const int E = hp.embed, G = v->G, T = v->T, ws = hp.window;
    const bool glob = is_global(hp, i);
    const int B = glob ? 1 : (G / ws) * (G / ws);
    const int N = glob ? T : ws * ws;
    AttnOut attn_q8;  // the proj MUL_MAT's quantised input (window order), written by the attention
    attn_q8.codes = v->codes_a.p;
    attn_q8.quads = v->quads_a.p;
    attn_q8.ld = v->Tpad;
    return launched(v, layernorm_q8(x, T, E, w.n1w.as<float>(), w.n1b.as<float>(), 1e-5f, G, glob ? 0 : ws,
                                v->codes_a.p, v->quads_a.p, v->Tpad, s),
                   "ln1") &&
           mmq_qkv(v, w, N) &&
           launched(v, flash_attention(v->q.p, v->k.p, v->v.p, B, N, hp.heads, 1.0f / sqrtf(static_cast<float>(E / hp.heads)),
                                   attn_q8, v->be->err, s),
                   "attention") &&
           mmq(v, v->codes_a.p, v->quads_a.p, w.proj, MMQ_OUT_F32, w.proj_b.as<float>(), x, 1,
               glob ? nullptr : v->rowmap.as<int>(), nullptr, nullptr, 0) &&
           launched(v, layernorm_q8(x, T, E, w.n2w.as<float>(), w.n2b.as<float>(), 1e-5f, G, 0, v->codes_a.p, v->quads_a.p,
                                v->Tpad, s),
                   "ln2") &&
           mmq(v, v->codes_a.p, v->quads_a.p, w.fc1, MMQ_OUT_Q8, w.fc1_b.as<float>(), nullptr, 0, nullptr,
               v->codes_b.p, v->quads_b.p, 1) &&
           mmq(v, v->codes_b.p, v->quads_b.p, w.fc2, MMQ_OUT_F32, w.fc2_b.as<float>(), x, 1, nullptr, nullptr, nullptr,
               0);
}

// sam3_build_neck_graph (sam3.cpp:3867-3925) with the scale weights n, writing outs[0..3]
static bool run_neck(Vit *v, const float *x, const NeckScaleW *n, DevBuf *outs) {
    const auto &hp = v->hp;
    cudaStream_t s = v->be->stream;
    const int E = hp.embed, G = v->G, T = v->T, D = hp.neck_dim, MID = v->MID;
    if (!launched(v, f32_to_f16(x, static_cast<int64_t>(T) * E, v->x16.p, s), "f32_to_f16")) return false;
    // scale 0: ConvT(E->512)+GELU, ConvT(512->D), conv1x1, conv3x3 at 4G
    if (!gemm(v, v->x16.p, n[0].dc1, T, 4 * MID, E, &n[0].dc1_b, 1, 1, v->n_a.p, GEMM_STORE_CONVT2X2, G, MID) ||
        !gemm(v, v->n_a.p, n[0].dc2, 4 * T, 4 * D, MID, &n[0].dc2_b, 0, 1, v->n_c.p, GEMM_STORE_CONVT2X2, 2 * G, D) ||
        !gemm(v, v->n_c.p, n[0].c1, 16 * T, D, D, &n[0].c1_b, 0, 1, v->n_d.p, GEMM_STORE_ROWMAJOR, 0, 0) ||
        !launched(v, im2col3x3_f16(v->n_d.p, 4 * G, 4 * G, D, v->n_col.p, s), "im2col") ||
        !gemm(v, v->n_col.p, n[0].c3, 16 * T, D, 9 * D, &n[0].c3_b, 0, 0, outs[0].p, GEMM_STORE_ROWMAJOR, 0, 0))
        return false;
    // scale 1: ConvT(E->512), conv1x1(512->D), conv3x3 at 2G
    if (!gemm(v, v->x16.p, n[1].dc1, T, 4 * MID, E, &n[1].dc1_b, 0, 1, v->n_a.p, GEMM_STORE_CONVT2X2, G, MID) ||
        !gemm(v, v->n_a.p, n[1].c1, 4 * T, D, MID, &n[1].c1_b, 0, 1, v->n_d.p, GEMM_STORE_ROWMAJOR, 0, 0) ||
        !launched(v, im2col3x3_f16(v->n_d.p, 2 * G, 2 * G, D, v->n_col.p, s), "im2col") ||
        !gemm(v, v->n_col.p, n[1].c3, 4 * T, D, 9 * D, &n[1].c3_b, 0, 0, outs[1].p, GEMM_STORE_ROWMAJOR, 0, 0))
        return false;
    // scale 2: conv1x1(E->D), conv3x3 at G
    if (!gemm(v, v->x16.p, n[2].c1, T, D, E, &n[2].c1_b, 0, 1, v->n_d.p, GEMM_STORE_ROWMAJOR, 0, 0) ||
        !launched(v, im2col3x3_f16(v->n_d.p, G, G, D, v->n_col.p, s), "im2col") ||
        !gemm(v, v->n_col.p, n[2].c3, T, D, 9 * D, &n[2].c3_b, 0, 0, outs[2].p, GEMM_STORE_ROWMAJOR, 0, 0))
        return false;
    // scale 3: maxpool 2x2, conv1x1(E->D), conv3x3 at G/2
    const int g = G / 2;
    return launched(v, maxpool2x2_f16(x, G, E, v->mp16.p, s), "maxpool") &&
           gemm(v, v->mp16.p, n[3].c1, g * g, D, E, &n[3].c1_b, 0, 1, v->n_d.p, GEMM_STORE_ROWMAJOR, 0, 0) &&
           launched(v, im2col3x3_f16(v->n_d.p, g, g, D, v->n_col.p, s), "im2col") &&
           gemm(v, v->n_col.p, n[3].c3, g * g, D, 9 * D, &n[3].c3_b, 0, 0, outs[3].p, GEMM_STORE_ROWMAJOR, 0, 0);
}

// both necks: the tracker's, then the detector's when its weights are set
static bool run_necks(Vit *v, const float *x) {
    return run_neck(v, x, v->neck, v->out) && (!v->det_any || run_neck(v, x, v->neck_det, v->out_det));
}

static bool check_ready(Vit *v) {
    v->missing.clear();
    auto need = [&](const DevBuf &d, const std::string &name) {
        if (!d.p) v->missing.push_back(name);
    };
    need(v->patch_w, "vit.patch_embed.proj.weight");
    need(v->pos, "vit.pos_embed");
    need(v->lnpre_w, "vit.ln_pre.weight");
    need(v->lnpre_b, "vit.ln_pre.bias");
    for (int i = 0; i < v->hp.depth; ++i) {
        const std::string p = "vit.blocks." + std::to_string(i);
        const BlockW &b = v->blk[i];
        need(b.n1w, p + ".norm1.weight");
        need(b.n1b, p + ".norm1.bias");
        need(b.n2w, p + ".norm2.weight");
        need(b.n2b, p + ".norm2.bias");
        need(b.qkv_b, p + ".attn.qkv.bias");
        need(b.proj_b, p + ".attn.proj.bias");
        need(b.fc1_b, p + ".mlp.lin1.bias");
        need(b.fc2_b, p + ".mlp.lin2.bias");
        if (!b.qkv.set) v->missing.push_back(p + ".attn.qkv.weight");
        if (!b.proj.set) v->missing.push_back(p + ".attn.proj.weight");
        if (!b.fc1.set) v->missing.push_back(p + ".mlp.lin1.weight");
        if (!b.fc2.set) v->missing.push_back(p + ".mlp.lin2.weight");
    }
    const char *sn[4][8] = {
        {"0.dconv_2x2_0.weight", "0.dconv_2x2_0.bias", "0.dconv_2x2_1.weight", "0.dconv_2x2_1.bias",
         "0.conv_1x1.weight", "0.conv_1x1.bias", "0.conv_3x3.weight", "0.conv_3x3.bias"},
        {"1.dconv_2x2.weight", "1.dconv_2x2.bias", nullptr, nullptr, "1.conv_1x1.weight", "1.conv_1x1.bias",
         "1.conv_3x3.weight", "1.conv_3x3.bias"},
        {nullptr, nullptr, nullptr, nullptr, "2.conv_1x1.weight", "2.conv_1x1.bias", "2.conv_3x3.weight",
         "2.conv_3x3.bias"},
        {nullptr, nullptr, nullptr, nullptr, "3.conv_1x1.weight", "3.conv_1x1.bias", "3.conv_3x3.weight",
         "3.conv_3x3.bias"}};
    for (int which = 0; which < (v->det_any ? 2 : 1); ++which) {
        const NeckScaleW *nk = which == 0 ? v->neck : v->neck_det;
        const std::string pre = which == 0 ? "neck.trk." : "neck.det.";
        for (int sc = 0; sc < 4; ++sc) {
            const DevBuf *bufs[8] = {&nk[sc].dc1, &nk[sc].dc1_b, &nk[sc].dc2, &nk[sc].dc2_b,
                                     &nk[sc].c1,  &nk[sc].c1_b,  &nk[sc].c3,  &nk[sc].c3_b};
            for (int j = 0; j < 8; ++j)
                if (sn[sc][j]) need(*bufs[j], pre + sn[sc][j]);
        }
    }
    if (!v->missing.empty()) {
        set_error("encoder weights missing: %zu tensors, first %s", v->missing.size(), v->missing[0].c_str());
        return false;
    }
    return true;
}

// preprocessing + prefix of one image into rows [0, T) of x
static bool prefix_image(Vit *v, const uint8_t *rgb_dev, int w, int h, float *x) {
    const auto &hp = v->hp;
    cudaStream_t s = v->be->stream;
    const uint8_t *src = rgb_dev;
    if (w != hp.img || h != hp.img) {
        if (!v->img_rs.p && !v->img_rs.alloc(static_cast<size_t>(hp.img) * hp.img * 3)) return false;
        if (!launched(v, resize_bilinear_u8(rgb_dev, w, h, v->img_rs.as<uint8_t>(), hp.img, hp.img, s), "resize"))
            return false;
        src = v->img_rs.as<uint8_t>();
    }
    return launched(v, preprocess_sam3(src, hp.img, v->img_f32.as<float>(), s), "preprocess") &&
           run_prefix(v, v->img_f32.as<float>(), x);
}

static bool ensure_batch(Vit *v, int n);

static bool encode(Vit *v, const uint8_t *rgb_dev, int w, int h) {
    // (a failed batch growth leaves no block-loop buffers: re-establish one image's)
    if (!ensure_batch(v, 1) || !prefix_image(v, rgb_dev, w, h, v->x.as<float>())) return false;
    for (int i = 0; i < v->hp.depth; ++i)
        if (!run_block(v, i, v->x.as<float>())) return false;
    return run_necks(v, v->x.as<float>());
}

// Block-loop buffers for n images stacked image-major (the batched encode);
// single-image encodes use the first image's part.  Grows only; contents are
// not kept across a growth.
static bool ensure_batch(Vit *v, int n) {
    if (n <= v->bcap) return true;
    const auto &hp = v->hp;
    const size_t T = static_cast<size_t>(v->T), E = static_cast<size_t>(hp.embed), nn = static_cast<size_t>(n);
    if (!cuda_ok(cudaStreamSynchronize(v->be->stream), "batch sync")) return false;
    v->bcap = 0;
    const bool ok = v->x.alloc(nn * T * E * 4) && v->a16.alloc(nn * T * E * 2) &&
                    v->b16.alloc(nn * T * static_cast<size_t>(hp.mlp) * 2) && v->q.alloc(nn * T * E * 2) &&
                    v->k.alloc(nn * T * E * 2) && v->v.alloc(nn * T * E * 2) && v->rowmap.alloc(nn * T * 4) &&
                    cuda_ok(window_rowmap(v->G, hp.window, v->rowmap.as<int>(), v->be->stream, n), "rowmap") &&
                    cuda_ok(cudaStreamSynchronize(v->be->stream), "rowmap sync");
    if (ok) v->bcap = n;
    return ok;
}

static bool copy_outputs(Vit *v, float *const *out_host) {
    for (int i = 0; i < 4; ++i) {
        if (!out_host || !out_host[i]) continue;
        const size_t ob = static_cast<size_t>(v->out_side[i]) * v->out_side[i] * v->hp.neck_dim * 4;
        if (!cuda_ok(cudaMemcpyAsync(out_host[i], v->out[i].p, ob, cudaMemcpyDeviceToHost, v->be->stream),
                     "output download"))
            return false;
    }
    return true;
}

// n images through the encoder: the prefix per image, the blocks once over
// all n images' tokens (DQ16; the exact arithmetic runs image by image), then
// each image's neck, whose outputs go to out_host[4 i .. 4 i + 3] (if given)
// before the next image's neck overwrites them.
static bool encode_batch(Vit *v, int n, const uint8_t *const *rgb_dev, int w, int h, float *const *out_host) {
    if (v->be->mmq_arith != SAM3B200_ARITH_DQ16 || n == 1) {
        for (int i = 0; i < n; ++i)
            if (!encode(v, rgb_dev[i], w, h) || !copy_outputs(v, out_host ? out_host + 4 * i : nullptr)) return false;
        return true;
    }
    if (!ensure_batch(v, n)) return false;
    const size_t img_elems = static_cast<size_t>(v->T) * v->hp.embed;
    for (int i = 0; i < n; ++i)
        if (!prefix_image(v, rgb_dev[i], w, h, v->x.as<float>() + i * img_elems)) return false;
    for (int b = 0; b < v->hp.depth; ++b)
        if (!run_block(v, b, v->x.as<float>(), n)) return false;
    for (int i = 0; i < n; ++i)
        if (!run_necks(v, v->x.as<float>() + i * img_elems) ||
            !copy_outputs(v, out_host ? out_host + 4 * i : nullptr))
            return false;
    return true;
}

}  // namespace b200

using namespace b200;

extern "C" {

sam3b200_vit *sam3b200_vit_create(sam3b200_backend *h, const sam3b200_vit_hparams *hp) {
    auto *be = reinterpret_cast<Backend *>(h);
    if (!be || !hp) {
        set_error("vit_create: null argument");
        return nullptr;
    }
    const int G = hp->patch > 0 ? hp->img / hp->patch : 0;
    if (hp->patch <= 0 || hp->img % hp->patch != 0 || hp->embed % 64 != 0 || hp->heads * 64 != hp->embed ||
        hp->mlp % 32 != 0 || hp->window <= 0 || G % hp->window != 0 || G % 2 != 0 ||
        hp->depth <= 0 || hp->depth > 64 || hp->pos_grid <= 0 || G % hp->pos_grid != 0 || hp->neck_dim % 32 != 0 ||
        hp->n_global < 0 || hp->n_global > 4 ||
        (hp->wtype != SAM3B200_TYPE_Q8_0 && hp->wtype != SAM3B200_TYPE_Q4_0)) {
        set_error("vit_create: unsupported hyper-parameters (need head_dim 64, grid divisible by window and 2, "
                  "Q8_0/Q4_0 linear weights)");
        return nullptr;
    }
    cudaSetDevice(be->device);
    auto *v = new Vit();
    v->be = be;
    v->hp = *hp;
    v->G = G;
    v->T = G * G;
    v->Tpad = (v->T + MMQ_ROW_ALIGN - 1) / MMQ_ROW_ALIGN * MMQ_ROW_ALIGN;
    v->KP = (3 * hp->patch * hp->patch + 15) / 16 * 16;
    v->blk.resize(hp->depth);
    if (!alloc_activations(v)) {
        delete v;
        return nullptr;
    }
    return reinterpret_cast<sam3b200_vit *>(v);
}

void sam3b200_vit_free(sam3b200_vit *hv) {
    auto *v = reinterpret_cast<Vit *>(hv);
    if (!v) return;
    cudaSetDevice(v->be->device);
    cudaStreamSynchronize(v->be->stream);
    delete v;  // every DevBuf member frees its device memory
}

int sam3b200_vit_set_tensor(sam3b200_vit *hv, const char *name_c, int type, const void *data, const int64_t *ne) {
    auto *v = reinterpret_cast<Vit *>(hv);
    if (!v || !name_c || !data || !ne) {
        set_error("vit_set_tensor: null argument");
        return SAM3B200_STATUS_FAILED;
    }
    cudaSetDevice(v->be->device);
    cudaStream_t s = v->be->stream;
    const std::string name(name_c);
    const auto &hp = v->hp;
    const int64_t n = ne[0] * ne[1] * ne[2] * ne[3];
    const int E = hp.embed, D = hp.neck_dim, MID = v->MID;
    std::vector<float> f;
    auto vec = [&](DevBuf &d, int64_t expect) -> int {
        if (n != expect) {
            set_error("%s: %lld elements, expected %lld", name_c, (long long)n, (long long)expect);
            return SAM3B200_STATUS_FAILED;
        }
        if (!to_f32(type, data, n, f) || !upload(d, f.data(), f.size() * 4, s)) return SAM3B200_STATUS_FAILED;
        return SAM3B200_STATUS_SUCCESS;
    };
    if (name == "vit.patch_embed.proj.weight") {  // ggml [p, p, 3, E]
        const int K = 3 * hp.patch * hp.patch;
        if (n != static_cast<int64_t>(K) * E || !to_f32(type, data, n, f)) {
            set_error("%s: bad shape or type", name_c);
            return SAM3B200_STATUS_FAILED;
        }
        std::vector<float> w(static_cast<size_t>(E) * v->KP, 0.f);
        for (int e = 0; e < E; ++e)
            for (int kk = 0; kk < K; ++kk) w[static_cast<size_t>(e) * v->KP + kk] = f[static_cast<size_t>(e) * K + kk];
        return upload_f16(v->patch_w, w, s) ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
    }
    if (name == "vit.pos_embed") return vec(v->pos, static_cast<int64_t>(E) * hp.pos_grid * hp.pos_grid);
    if (name == "vit.ln_pre.weight") return vec(v->lnpre_w, E);
    if (name == "vit.ln_pre.bias") return vec(v->lnpre_b, E);
    int bi = -1;
    char tail[128] = {0};
    if (sscanf(name_c, "vit.blocks.%d.%127s", &bi, tail) == 2) {
        if (bi < 0 || bi >= hp.depth) {
            set_error("%s: block index out of range", name_c);
            return SAM3B200_STATUS_FAILED;
        }
        BlockW &b = v->blk[bi];
        const std::string t(tail);
        const int N = is_global(hp, bi) ? v->T : hp.window * hp.window;
        if (t == "norm1.weight") return vec(b.n1w, E);
        if (t == "norm1.bias") return vec(b.n1b, E);
        if (t == "norm2.weight") return vec(b.n2w, E);
        if (t == "norm2.bias") return vec(b.n2b, E);
        if (t == "attn.qkv.bias") return vec(b.qkv_b, 3 * E);
        if (t == "attn.proj.bias") return vec(b.proj_b, E);
        if (t == "mlp.lin1.bias") return vec(b.fc1_b, hp.mlp);
        if (t == "mlp.lin2.bias") return vec(b.fc2_b, E);
        if (t == "attn.freqs_cis") return vec(b.freqs, static_cast<int64_t>(N) * 64);
        QWeight *qw = t == "attn.qkv.weight" ? &b.qkv
                      : t == "attn.proj.weight" ? &b.proj
                      : t == "mlp.lin1.weight" ? &b.fc1
                      : t == "mlp.lin2.weight" ? &b.fc2
                                                 : nullptr;
        if (qw) {
            const int64_t K = ne[0], NN = ne[1];
            const int64_t eK = qw == &b.fc2 ? hp.mlp : E;
            const int64_t eN = qw == &b.qkv ? 3 * E : qw == &b.fc1 ? hp.mlp : E;
            if (K != eK || NN != eN || ne[2] != 1 || ne[3] != 1) {
                set_error("%s: shape [%lld, %lld], expected [%lld, %lld]", name_c, (long long)K, (long long)NN,
                          (long long)eK, (long long)eN);
                return SAM3B200_STATUS_FAILED;
            }
            return upload_qweight(v->be, *qw, type, data, K, NN) && make_w16(v->be, *qw) ? SAM3B200_STATUS_SUCCESS
                                                                                         : SAM3B200_STATUS_FAILED;
        }
        set_error("%s: unknown block tensor", name_c);
        return SAM3B200_STATUS_FAILED;
    }
    int sc = -1;
    NeckScaleW *nwp = nullptr;
    if (sscanf(name_c, "neck.trk.%d.%127s", &sc, tail) == 2 && sc >= 0 && sc < 4) {
        nwp = &v->neck[sc];
    } else if (sscanf(name_c, "neck.det.%d.%127s", &sc, tail) == 2 && sc >= 0 && sc < 4) {
        if (!v->det_any) {  // first detector-neck tensor: its four outputs
            for (int i = 0; i < 4; ++i)
                if (!v->out_det[i].alloc(static_cast<size_t>(v->out_side[i]) * v->out_side[i] * D * 4))
                    return SAM3B200_STATUS_ALLOC_FAILED;
            v->det_any = true;
        }
        nwp = &v->neck_det[sc];
    }
    if (nwp) {
        NeckScaleW &nw = *nwp;
        const std::string t(tail);
        if (!to_f32(type, data, n, f)) return SAM3B200_STATUS_FAILED;
        auto bias = [&](DevBuf &d, int64_t expect) -> int {
            if (n != expect) {
                set_error("%s: bad size", name_c);
                return SAM3B200_STATUS_FAILED;
            }
            return upload(d, f.data(), f.size() * 4, s) ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
        };
        // ConvT ggml [2, 2, Cout, Cin] -> B[(ky*2+kx)*Cout + co][ci]
        auto convt = [&](DevBuf &d, int cout, int cin) -> int {
            if (n != 4LL * cout * cin) {
                set_error("%s: bad size", name_c);
                return SAM3B200_STATUS_FAILED;
            }
            std::vector<float> w(static_cast<size_t>(4) * cout * cin);
            for (int ci = 0; ci < cin; ++ci)
                for (int co = 0; co < cout; ++co)
                    for (int ky = 0; ky < 2; ++ky)
                        for (int kx = 0; kx < 2; ++kx)
                            w[(static_cast<size_t>(ky * 2 + kx) * cout + co) * cin + ci] =
                                f[kx + 2 * (ky + 2 * (co + static_cast<size_t>(cout) * ci))];
            return upload_f16(d, w, s) ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
        };
        // conv kxk ggml [k, k, Cin, Cout] -> B[co][(ky*k + kx)*Cin + ci]
        auto conv = [&](DevBuf &d, int ks, int cin, int cout) -> int {
            if (n != static_cast<int64_t>(ks) * ks * cin * cout) {
                set_error("%s: bad size", name_c);
                return SAM3B200_STATUS_FAILED;
            }
            std::vector<float> w(static_cast<size_t>(ks) * ks * cin * cout);
            for (int co = 0; co < cout; ++co)
                for (int ci = 0; ci < cin; ++ci)
                    for (int ky = 0; ky < ks; ++ky)
                        for (int kx = 0; kx < ks; ++kx)
                            w[static_cast<size_t>(co) * ks * ks * cin + static_cast<size_t>(ky * ks + kx) * cin + ci] =
                                f[kx + ks * (ky + ks * (ci + static_cast<size_t>(cin) * co))];
            return upload_f16(d, w, s) ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
        };
        const int c1_in = sc == 0 ? D : sc == 1 ? MID : E;
        if ((sc == 0 && t == "dconv_2x2_0.weight") || (sc == 1 && t == "dconv_2x2.weight")) return convt(nw.dc1, MID, E);
        if ((sc == 0 && t == "dconv_2x2_0.bias") || (sc == 1 && t == "dconv_2x2.bias")) return bias(nw.dc1_b, MID);
        if (sc == 0 && t == "dconv_2x2_1.weight") return convt(nw.dc2, D, MID);
        if (sc == 0 && t == "dconv_2x2_1.bias") return bias(nw.dc2_b, D);
        if (t == "conv_1x1.weight") return conv(nw.c1, 1, c1_in, D);
        if (t == "conv_1x1.bias") return bias(nw.c1_b, D);
        if (t == "conv_3x3.weight") return conv(nw.c3, 3, D, D);
        if (t == "conv_3x3.bias") return bias(nw.c3_b, D);
    }
    set_error("%s: not a tensor of the visual encoder", name_c);
    return SAM3B200_STATUS_FAILED;
}

int sam3b200_vit_missing(sam3b200_vit *hv, char *buf, int cap) {
    auto *v = reinterpret_cast<Vit *>(hv);
    if (!v) return -1;
    check_ready(v);
    if (buf && cap > 0) {
        std::string all;
        for (auto &m : v->missing) all += m + "\n";
        snprintf(buf, cap, "%s", all.c_str());
    }
    return static_cast<int>(v->missing.size());
}

int sam3b200_encode_image_device(sam3b200_vit *hv, const uint8_t *rgb_dev, int w, int h) {
    auto *v = reinterpret_cast<Vit *>(hv);
    if (!v || !rgb_dev || w <= 0 || h <= 0) {
        set_error("encode_image_device: bad argument");
        return SAM3B200_STATUS_FAILED;
    }
    cudaSetDevice(v->be->device);
    if (!check_ready(v)) return SAM3B200_STATUS_FAILED;
    return encode(v, rgb_dev, w, h) ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
}

int sam3b200_encode_image(sam3b200_vit *hv, const uint8_t *rgb, int w, int h, float *const out_host[4]) {
    auto *v = reinterpret_cast<Vit *>(hv);
    if (!v || !rgb || w <= 0 || h <= 0) {
        set_error("encode_image: bad argument");
        return SAM3B200_STATUS_FAILED;
    }
    cudaSetDevice(v->be->device);
    if (!check_ready(v)) return SAM3B200_STATUS_FAILED;
    const size_t bytes = static_cast<size_t>(w) * h * 3;
    if (v->img_u8.n < bytes && !v->img_u8.alloc(bytes)) return SAM3B200_STATUS_ALLOC_FAILED;
    cudaStream_t s = v->be->stream;
    if (!cuda_ok(cudaMemcpyAsync(v->img_u8.p, rgb, bytes, cudaMemcpyHostToDevice, s), "image upload") ||
        !encode(v, v->img_u8.as<uint8_t>(), w, h) || !copy_outputs(v, out_host))
        return SAM3B200_STATUS_FAILED;
    return sam3b200_backend_synchronize(reinterpret_cast<sam3b200_backend *>(v->be));
}

int sam3b200_encode_images_device(sam3b200_vit *hv, int n, const uint8_t *const *rgb_dev, int w, int h) {
    auto *v = reinterpret_cast<Vit *>(hv);
    if (!v || n <= 0 || !rgb_dev || w <= 0 || h <= 0) {
        set_error("encode_images_device: bad argument");
        return SAM3B200_STATUS_FAILED;
    }
    for (int i = 0; i < n; ++i)
        if (!rgb_dev[i]) {
            set_error("encode_images_device: image %d is null", i);
            return SAM3B200_STATUS_FAILED;
        }
    cudaSetDevice(v->be->device);
    if (!check_ready(v)) return SAM3B200_STATUS_FAILED;
    return encode_batch(v, n, rgb_dev, w, h, nullptr) ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
}

int sam3b200_encode_images(sam3b200_vit *hv, int n, const uint8_t *const *rgb, int w, int h,
                           float *const *out_host) {
    auto *v = reinterpret_cast<Vit *>(hv);
    if (!v || n <= 0 || !rgb || w <= 0 || h <= 0) {
        set_error("encode_images: bad argument");
        return SAM3B200_STATUS_FAILED;
    }
    cudaSetDevice(v->be->device);
    if (!check_ready(v)) return SAM3B200_STATUS_FAILED;
    const size_t bytes = static_cast<size_t>(w) * h * 3;
    if (v->img_u8.n < bytes * n && !v->img_u8.alloc(bytes * n)) return SAM3B200_STATUS_ALLOC_FAILED;
    cudaStream_t s = v->be->stream;
    std::vector<const uint8_t *> dev(static_cast<size_t>(n));
    for (int i = 0; i < n; ++i) {
        if (!rgb[i]) {
            set_error("encode_images: image %d is null", i);
            return SAM3B200_STATUS_FAILED;
        }
        dev[i] = v->img_u8.as<uint8_t>() + bytes * i;
        if (!cuda_ok(cudaMemcpyAsync(const_cast<uint8_t *>(dev[i]), rgb[i], bytes, cudaMemcpyHostToDevice, s),
                     "image upload"))
            return SAM3B200_STATUS_FAILED;
    }
    if (!encode_batch(v, n, dev.data(), w, h, out_host)) return SAM3B200_STATUS_FAILED;
    return sam3b200_backend_synchronize(reinterpret_cast<sam3b200_backend *>(v->be));
}

int sam3b200_vit_output_det(sam3b200_vit *hv, int i, const float **dev, int64_t *ne) {
    auto *v = reinterpret_cast<Vit *>(hv);
    if (!v || i < 0 || i > 3 || !dev) return SAM3B200_STATUS_FAILED;
    if (!v->det_any) {
        set_error("vit_output_det: the encoder has no detector neck (neck.det tensors not set)");
        return SAM3B200_STATUS_FAILED;
    }
    *dev = v->out_det[i].as<float>();
    if (ne) {
        ne[0] = v->hp.neck_dim;
        ne[1] = ne[2] = v->out_side[i];
        ne[3] = 1;
    }
    return SAM3B200_STATUS_SUCCESS;
}

int sam3b200_vit_output(sam3b200_vit *hv, int i, const float **dev, int64_t *ne) {
    auto *v = reinterpret_cast<Vit *>(hv);
    if (!v || i < -1 || i > 3 || !dev) return SAM3B200_STATUS_FAILED;
    if (i == -1) {  // ViT output [E, G, G]
        *dev = v->x.as<float>();
        if (ne) {
            ne[0] = v->hp.embed;
            ne[1] = ne[2] = v->G;
            ne[3] = 1;
        }
        return SAM3B200_STATUS_SUCCESS;
    }
    *dev = v->out[i].as<float>();
    if (ne) {
        ne[0] = v->hp.neck_dim;
        ne[1] = ne[2] = v->out_side[i];
        ne[3] = 1;
    }
    return SAM3B200_STATUS_SUCCESS;
}

static int preprocess_common(sam3b200_backend *hb, const uint8_t *rgb_dev, int w, int h, int img, float *out_dev,
                             bool sam2) {
    auto *be = reinterpret_cast<Backend *>(hb);
    if (!be || !rgb_dev || !out_dev || w <= 0 || h <= 0 || img <= 0) {
        set_error("preprocess: bad argument");
        return SAM3B200_STATUS_FAILED;
    }
    cudaSetDevice(be->device);
    const uint8_t *src = rgb_dev;
    uint8_t *tmp = nullptr;
    if (w != img || h != img) {
        if (!cuda_ok(cudaMallocAsync(reinterpret_cast<void **>(&tmp), static_cast<size_t>(img) * img * 3, be->stream),
                     "cudaMallocAsync") ||
            !cuda_ok(resize_bilinear_u8(rgb_dev, w, h, tmp, img, img, be->stream), "resize"))
            return SAM3B200_STATUS_FAILED;
        src = tmp;
    }
    const bool ok = cuda_ok(sam2 ? preprocess_sam2(src, img, out_dev, be->stream)
                                 : preprocess_sam3(src, img, out_dev, be->stream),
                            "preprocess");
    if (tmp) cudaFreeAsync(tmp, be->stream);
    return ok ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
}

int sam3b200_preprocess(sam3b200_backend *hb, const uint8_t *rgb_dev, int w, int h, int img, float *out_dev) {
    return preprocess_common(hb, rgb_dev, w, h, img, out_dev, false);
}

int sam3b200_preprocess_sam2(sam3b200_backend *hb, const uint8_t *rgb_dev, int w, int h, int img, float *out_dev) {
    return preprocess_common(hb, rgb_dev, w, h, img, out_dev, true);
}

int sam3b200_vit_run_prefix(sam3b200_vit *hv, const float *img_chw_dev, float *x_dev) {
    auto *v = reinterpret_cast<Vit *>(hv);
    if (!v || !img_chw_dev || !x_dev) return SAM3B200_STATUS_FAILED;
    cudaSetDevice(v->be->device);
    return run_prefix(v, img_chw_dev, x_dev) ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
}

int sam3b200_vit_run_block(sam3b200_vit *hv, int idx, float *x_dev) {
    auto *v = reinterpret_cast<Vit *>(hv);
    if (!v || !x_dev || idx < 0 || idx >= v->hp.depth) return SAM3B200_STATUS_FAILED;
    cudaSetDevice(v->be->device);
    return ensure_batch(v, 1) && run_block(v, idx, x_dev) ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
}

int sam3b200_vit_run_neck(sam3b200_vit *hv, const float *x_dev) {
    auto *v = reinterpret_cast<Vit *>(hv);
    if (!v || !x_dev) return SAM3B200_STATUS_FAILED;
    cudaSetDevice(v->be->device);
    return run_necks(v, x_dev) ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
}

}  // extern "C"
