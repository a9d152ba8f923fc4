// ddec.cu -- the DETR decoder of the SAM3 detector on the B200 backend: the
// graph sam3_build_ddec_graph builds (sam3.cpp:8749-8888) with its layer
// (sam3_ddec_layer_forward :8438-8632), query positions
// (sam3_build_query_pos / sam3_build_sine_pos_embed_4d :8200-8290), the
// box-relative attention bias (sam3_compute_box_rpb :8293-8436), the box
// refinement, the dot-product scoring (sam3_dot_product_scoring :8640-8739)
// and the presence head.
//
//   queries = [presence token; query_embed]     boxes = sigmoid(reference_points)
//   per layer: qpos = [0; ref_point_head(sine(boxes))]
//              rpb  = box-relative bias per head from boxes (log-spaced deltas, 2 MLPs)
//              queries = LN(queries + SA(queries + qpos, queries))                    norm2
//              queries = LN(queries + CA(queries + qpos, text; padding bias))          norm_ca_text
//              queries = LN(queries + CA(queries + qpos, enc + pos, enc; rpb))         norm1
//              queries = LN(queries + FFN(queries))                                    norm3
//              boxes = sigmoid(inverse_sigmoid(boxes) + bbox_embed(LN(queries[1:])))
//   outputs: [presence; LN(queries[1:])], boxes, clamp(score / 16), presence logit
//
// Every linear layer is run_mul_mat (the exact quantised MUL_MAT; fp16 GEMM for
// F16/F32), with the fused in_proj weights split by rows; attention is
// attention_simt (8 heads of 32) for the small self and text attention, the
// image cross-attention on the tensor cores (attn_mma.cu: fp16 q, k, v, fp32
// scores) with the f32 per-head bias the reference keeps in f32 (SOFT_MAX_EXT).
#include "../../include/sam3_b200.h"
#include "attn_mma.cuh"
#include "eltwise.cuh"
#include "model_util.h"
#include "row_norm.cuh"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

namespace b200 {
namespace {

__device__ __forceinline__ float sigmoid_f(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x))); }

// queries = [presence; query_embed] (rows of D), boxes = sigmoid(reference_points)
__global__ void dd_init_kernel(const float *__restrict__ pres, const float *__restrict__ qemb,
                               const float *__restrict__ refp, int NQ, int D, float *__restrict__ queries,
                               float *__restrict__ boxes) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t nq = static_cast<int64_t>(NQ + 1) * D;
    if (i < nq) queries[i] = i < D ? pres[i] : qemb[i - D];
    if (i < 4 * NQ) boxes[i] = sigmoid_f(refp[i]);
}

// sam3_build_sine_pos_embed_4d: per query, for the coordinates (cy, cx, w, h)
// in that order, 64 angles dim_t[i] * coord interleaved as (sin, cos) -> 512
__global__ void dd_sine_kernel(const float *__restrict__ boxes, const float *__restrict__ dim_t, int NQ,
                               float *__restrict__ out) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<int64_t>(NQ) * 256) return;
    const int q = static_cast<int>(i / 256), r = static_cast<int>(i % 256), c = r / 64, k = r % 64;
    const int coord = c == 0 ? 1 : c == 1 ? 0 : c;
    const float a = __fmul_rn(dim_t[k], boxes[q * 4 + coord]);
    float *o = out + static_cast<int64_t>(q) * 512 + c * 128 + 2 * k;
    o[0] = sinf(a);
    o[1] = cosf(a);
}

// Box-relative deltas (sam3_compute_box_rpb steps 1-3) for one axis: row
// q*S + s holds (coord[s] - lo[q], coord[s] - hi[q]) after the log transform
// sign(8d) * (log(|8d| + 1) * inv_ln2) * inv_log2_8, with lo/hi = c -/+ 0.5 e
// from the box's centre c and extent e (axis 0: cx, w; axis 1: cy, h).
__global__ void dd_deltas_kernel(const float *__restrict__ boxes, int axis, int NQ, int S, float inv_ln2,
                                 float inv_log2_8, float *__restrict__ out) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<int64_t>(NQ) * S) return;
    const int q = static_cast<int>(i / S), s = static_cast<int>(i % S);
    const float c = boxes[q * 4 + axis], e = boxes[q * 4 + 2 + axis];
    const float half = __fmul_rn(e, 0.5f);
    const float lo = __fsub_rn(c, half), hi = __fadd_rn(c, half);
    const float coord = __fdiv_rn(static_cast<float>(s), static_cast<float>(S));
    const float d[2] = {__fsub_rn(coord, lo), __fsub_rn(coord, hi)};
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const float d8 = __fmul_rn(d[j], 8.0f);
        const float sg = d8 > 0.f ? 1.f : d8 < 0.f ? -1.f : 0.f;
        float lv = logf(__fadd_rn(fabsf(d8), 1.0f));
        lv = __fmul_rn(__fmul_rn(lv, inv_ln2), inv_log2_8);
        out[i * 2 + j] = __fmul_rn(sg, lv);
    }
}

// First boxRPB layer (2 -> C, K = 2 is an F32 kernel in quantised files, F16
// in F16 files): relu(fl(fl(d0 w0) + fl(d1 w1)) + b); in_f16 rounds d to fp16
__global__ void dd_rpb0_kernel(const float *__restrict__ d, int64_t rows, const float *__restrict__ w,
                               const float *__restrict__ b, int C, int in_f16, float *__restrict__ out) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= rows * C) return;
    const int64_t r = i / C;
    const int c = static_cast<int>(i % C);
    float d0 = d[r * 2], d1 = d[r * 2 + 1];
    if (in_f16) {
        d0 = __half2float(__float2half_rn(d0));
        d1 = __half2float(__float2half_rn(d1));
    }
    const float v = __fadd_rn(__fadd_rn(__fmul_rn(d0, w[c * 2]), __fmul_rn(d1, w[c * 2 + 1])), b[c]);
    out[i] = fmaxf(v, 0.0f);
}

// The per-head f32 attention bias [NH][NQ+1][S*S]: row 0 (presence) zero,
// row 1+q at key (y, x) = rpb_y[q][y][h] + rpb_x[q][x][h]
__global__ void dd_rpb_mask_kernel(const float *__restrict__ rx, const float *__restrict__ ry, int NQ, int S, int NH,
                                   float *__restrict__ mask) {
    const int64_t N = static_cast<int64_t>(S) * S;
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<int64_t>(NH) * (NQ + 1) * N) return;
    const int64_t key = i % N;
    const int row = static_cast<int>((i / N) % (NQ + 1)), h = static_cast<int>(i / N / (NQ + 1));
    if (row == 0) {
        mask[i] = 0.0f;
        return;
    }
    const int q = row - 1, y = static_cast<int>(key / S), x = static_cast<int>(key % S);
    mask[i] = __fadd_rn(ry[(static_cast<int64_t>(q) * S + y) * NH + h], rx[(static_cast<int64_t>(q) * S + x) * NH + h]);
}

// boxes = sigmoid(inverse_sigmoid(boxes) + delta), inverse_sigmoid with the
// clamp to [1e-3, 1 - 1e-3] (sam3_inverse_sigmoid, sam3.cpp:8171-8181)
__global__ void dd_refine_kernel(float *boxes, const float *__restrict__ delta, int n, float lo, float hi) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float x = fminf(fmaxf(boxes[i], lo), hi);
    const float inv = __fsub_rn(logf(x), logf(__fadd_rn(-x, 1.0f)));
    boxes[i] = sigmoid_f(__fadd_rn(inv, delta[i]));
}

// mean over the T text rows of x[t][d] * valid[t] (pool_1d AVG over T of the
// masked rows; valid null: plain mean)
__global__ void dd_pool_kernel(const float *__restrict__ x, const float *__restrict__ valid, int T, int D,
                               float *__restrict__ out) {
    const int d = blockIdx.x * blockDim.x + threadIdx.x;
    if (d >= D) return;
    float s = 0.0f;
    for (int t = 0; t < T; ++t) {
        const float v = x[static_cast<int64_t>(t) * D + d];
        s = __fadd_rn(s, valid ? __fmul_rn(v, valid[t]) : v);
    }
    out[d] = __fdiv_rn(s, static_cast<float>(T));
}

// scores[q] = clamp(dot(p, h[q]) * scale, -12, 12), one warp per query
__global__ void dd_score_kernel(const float *__restrict__ p, const float *__restrict__ h, int NQ, int D, float scale,
                                float *__restrict__ scores) {
    const int q = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (q >= NQ) return;
    float s = 0.0f;
    for (int d = lane; d < D; d += 32) s = fmaf(p[d], h[static_cast<int64_t>(q) * D + d], s);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) scores[q] = fminf(fmaxf(__fmul_rn(s, scale), -12.0f), 12.0f);
}

struct Lin {  // a linear layer: weight + f32 bias
    sam3b200_weight *w = nullptr;
    DevBuf b;
    bool set() const { return w && b.p; }
};

struct DdecLayer {
    Lin sa_qk, sa_v, sa_o, ct_q, ct_kv, ct_o, ca_q, ca_k, ca_v, ca_o, f1, f2;
    DevBuf n1w, n1b, n2w, n2b, nctw, nctb, n3w, n3b;
};

}  // namespace

struct Ddec {
    Backend *be = nullptr;
    sam3b200_ddec_hparams hp{};
    std::vector<DdecLayer> ly;
    DevBuf qemb, pres, refp, normw, normb, pnw, pnb, sm_nw, sm_nb, dim_t, rpb0w[2], rpb0b[2];
    bool rpb0_f16[2] = {false, false};
    Lin bbox[3], rph[2], rpb1[2], phead[3], sm0, sm1, spp, shs;
    // activations
    DevBuf q, qpos, qin, qk, v, att, tmp, ffn, kvt, kin, kimg, vimg, tmask, rmask, sine, hid, dxy, rhid, rpbx, rpby;
    DevBuf boxes, bd, objn, bh1, bh2, tm, tm2, pooled, ppool, phs, scores, pr1, pr2, prout, seg;
    // host-run staging
    DevBuf in_enc, in_pos, in_text, in_bias, in_valid;
    std::vector<std::string> missing;
};

namespace {

bool dok(Ddec *d, cudaError_t e, const char *what) {
    d->be->count(1);
    return cuda_ok(e, what);
}

bool dlin(Ddec *d, const Lin &l, const float *x, int64_t ldx, int64_t rows, float *y, int64_t ldy) {
    return run_mul_mat(d->be, reinterpret_cast<const Weight *>(l.w), x, ldx, rows, l.b.as<float>(), y, ldy,
                       nullptr) == SAM3B200_STATUS_SUCCESS;
}

bool dln(Ddec *d, const float *x, int rows, const DevBuf &w, const DevBuf &b, float *y) {
    ln_rows_kernel<<<ew_blocks(static_cast<int64_t>(rows) * 32), 256, 0, d->be->stream>>>(
        x, rows, d->hp.d_model, w.as<float>(), b.as<float>(), 1e-5f, y);
    return dok(d, cudaGetLastError(), "ddec layer norm");
}

bool dadd(Ddec *d, const float *a, const float *b, int64_t n, float *c) {
    ew_add_kernel<<<ew_blocks(n), 256, 0, d->be->stream>>>(a, b, n, c);
    return dok(d, cudaGetLastError(), "ddec add");
}

bool drelu(Ddec *d, float *x, int64_t n) {
    ew_relu_kernel<<<ew_blocks(n), 256, 0, d->be->stream>>>(x, n);
    return dok(d, cudaGetLastError(), "ddec relu");
}

// 3-layer MLP with ReLU between (bbox_embed, presence_token_head)
bool mlp3(Ddec *d, const Lin (&l)[3], const float *x, int rows, float *out, int nout) {
    const int D = d->hp.d_model;
    float *h1 = d->bh1.as<float>(), *h2 = d->bh2.as<float>();
    return dlin(d, l[0], x, D, rows, h1, D) && drelu(d, h1, static_cast<int64_t>(rows) * D) &&
           dlin(d, l[1], h1, D, rows, h2, D) && drelu(d, h2, static_cast<int64_t>(rows) * D) &&
           dlin(d, l[2], h2, D, rows, out, nout);
}

// the box-relative bias of the current boxes into rmask
bool box_rpb(Ddec *d) {
    const int NQ = d->hp.num_queries, S = d->hp.feat, NH = d->hp.heads, D = d->hp.d_model;
    cudaStream_t s = d->be->stream;
    const int64_t rows = static_cast<int64_t>(NQ) * S;
    const float inv_ln2 = 1.0f / logf(2.0f), inv_log2_8 = 1.0f / log2f(8.0f);
    float *out[2] = {d->rpbx.as<float>(), d->rpby.as<float>()};
    for (int axis = 0; axis < 2; ++axis) {
        dd_deltas_kernel<<<ew_blocks(rows), 256, 0, s>>>(d->boxes.as<float>(), axis, NQ, S, inv_ln2, inv_log2_8,
                                                         d->dxy.as<float>());
        dd_rpb0_kernel<<<ew_blocks(rows * D), 256, 0, s>>>(d->dxy.as<float>(), rows, d->rpb0w[axis].as<float>(),
                                                           d->rpb0b[axis].as<float>(), D, d->rpb0_f16[axis] ? 1 : 0,
                                                           d->rhid.as<float>());
        if (!dok(d, cudaGetLastError(), "ddec box bias hidden") ||
            !dlin(d, d->rpb1[axis], d->rhid.as<float>(), D, rows, out[axis], NH))
            return false;
    }
    const int64_t n = static_cast<int64_t>(NH) * (NQ + 1) * S * S;
    dd_rpb_mask_kernel<<<ew_blocks(n), 256, 0, s>>>(out[0], out[1], NQ, S, NH, d->rmask.as<float>());
    return dok(d, cudaGetLastError(), "ddec box bias");
}

bool forward(Ddec *d, const float *enc, const float *enc_pos, const float *text, const float *bias,
             const float *valid, int T) {
    const int D = d->hp.d_model, NQ = d->hp.num_queries, NQ1 = NQ + 1, NH = d->hp.heads, HD = D / NH;
    const int F = d->hp.ffn_dim, N = d->hp.feat * d->hp.feat;
    const int64_t qd = static_cast<int64_t>(NQ1) * D;
    cudaStream_t s = d->be->stream;
    float *q = d->q.as<float>(), *qpos = d->qpos.as<float>(), *qin = d->qin.as<float>(), *qk = d->qk.as<float>();
    float *v = d->v.as<float>(), *att = d->att.as<float>(), *tmp = d->tmp.as<float>(), *kvt = d->kvt.as<float>();
    float *boxes = d->boxes.as<float>();
    const float scale = 1.0f / sqrtf(static_cast<float>(HD));
    const AttnStrides s1{0, HD, D}, s2{0, HD, 2 * D};
    dd_init_kernel<<<ew_blocks(qd), 256, 0, s>>>(d->pres.as<float>(), d->qemb.as<float>(), d->refp.as<float>(), NQ, D,
                                                 q, boxes);
    if (!dok(d, cudaGetLastError(), "ddec init") ||
        !dok(d, cudaMemsetAsync(qpos, 0, static_cast<size_t>(D) * 4, s), "ddec presence position"))
        return false;
    const __half *tmask = nullptr;
    if (bias) {
        ew_bias_mask_kernel<<<ew_blocks(static_cast<int64_t>(NQ1) * T), 256, 0, s>>>(bias, NQ1, T,
                                                                                     d->tmask.as<__half>());
        if (!dok(d, cudaGetLastError(), "ddec text mask")) return false;
        tmask = d->tmask.as<__half>();
    }
    // keys of the image cross-attention: enc + pos (the same for every layer)
    if (!dadd(d, enc, enc_pos, static_cast<int64_t>(N) * D, d->kin.as<float>())) return false;
    for (const DdecLayer &L : d->ly) {
        // query positions from the current boxes; the box-relative bias
        dd_sine_kernel<<<ew_blocks(static_cast<int64_t>(NQ) * 256), 256, 0, s>>>(boxes, d->dim_t.as<float>(), NQ,
                                                                                  d->sine.as<float>());
        if (!dok(d, cudaGetLastError(), "ddec sine") || !dlin(d, d->rph[0], d->sine.as<float>(), 512, NQ,
                                                              d->hid.as<float>(), D) ||
            !drelu(d, d->hid.as<float>(), static_cast<int64_t>(NQ) * D) ||
            !dlin(d, d->rph[1], d->hid.as<float>(), D, NQ, qpos + D, D) || !box_rpb(d))
            return false;
        // 1. self-attention (post-norm: norm2)
        if (!dadd(d, q, qpos, qd, qin) || !dlin(d, L.sa_qk, qin, D, NQ1, qk, 2 * D) ||
            !dlin(d, L.sa_v, q, D, NQ1, v, D) ||
            !dok(d, attention_simt(HD, qk, s2, NQ1, qk + D, s2, v, s1, NQ1, 1, NH, nullptr, 0, scale, att, s1, s),
                 "ddec self attention") ||
            !dlin(d, L.sa_o, att, D, NQ1, tmp, D) || !dadd(d, q, tmp, qd, qin) || !dln(d, qin, NQ1, L.n2w, L.n2b, q))
            return false;
        // 2. text cross-attention (norm_ca_text)
        if (!dadd(d, q, qpos, qd, qin) || !dlin(d, L.ct_q, qin, D, NQ1, att, D) ||
            !dlin(d, L.ct_kv, text, D, T, kvt, 2 * D) ||
            !dok(d, attention_simt(HD, att, s1, NQ1, kvt, s2, kvt + D, s2, T, 1, NH, tmask, T, scale, v, s1, s),
                 "ddec text attention") ||
            !dlin(d, L.ct_o, v, D, NQ1, tmp, D) || !dadd(d, q, tmp, qd, qin) || !dln(d, qin, NQ1, L.nctw, L.nctb, q))
            return false;
        // 3. image cross-attention with the box-relative bias (norm1)
        if (!dadd(d, q, qpos, qd, qin) || !dlin(d, L.ca_q, qin, D, NQ1, att, D) ||
            !dlin(d, L.ca_k, d->kin.as<float>(), D, N, d->kimg.as<float>(), D) ||
            !dlin(d, L.ca_v, enc, D, N, d->vimg.as<float>(), D) ||
            !dok(d, attention_mma_f32mask(HD, att, s1, NQ1, d->kimg.as<float>(), s1, d->vimg.as<float>(), s1, N, 1,
                                          NH, d->rmask.as<float>(), N, static_cast<int64_t>(NQ1) * N, scale, v, s1,
                                          s),
                 "ddec image attention") ||
            !dlin(d, L.ca_o, v, D, NQ1, tmp, D) || !dadd(d, q, tmp, qd, qin) || !dln(d, qin, NQ1, L.n1w, L.n1b, q))
            return false;
        // 4. feed-forward (norm3)
        if (!dlin(d, L.f1, q, D, NQ1, d->ffn.as<float>(), F) || !drelu(d, d->ffn.as<float>(),
                                                                        static_cast<int64_t>(NQ1) * F) ||
            !dlin(d, L.f2, d->ffn.as<float>(), F, NQ1, tmp, D) || !dadd(d, q, tmp, qd, qin) ||
            !dln(d, qin, NQ1, L.n3w, L.n3b, q))
            return false;
        // box refinement on the normed object queries
        if (!dln(d, q + D, NQ, d->normw, d->normb, d->objn.as<float>()) ||
            !mlp3(d, d->bbox, d->objn.as<float>(), NQ, d->bd.as<float>(), 4))
            return false;
        dd_refine_kernel<<<ew_blocks(4 * NQ), 256, 0, s>>>(boxes, d->bd.as<float>(), 4 * NQ, 1e-3f, 1.0f - 1e-3f);
        if (!dok(d, cudaGetLastError(), "ddec box refinement")) return false;
    }
    // outputs for the segmentation head: [last presence; LN(object queries)]
    float *seg = d->seg.as<float>();
    if (!dok(d, cudaMemcpyAsync(seg, q, static_cast<size_t>(D) * 4, cudaMemcpyDeviceToDevice, s), "ddec presence") ||
        !dln(d, q + D, NQ, d->normw, d->normb, seg + D))
        return false;
    // dot-product scoring against the pooled text
    float *tm = d->tm.as<float>(), *tm2 = d->tm2.as<float>();
    if (!dlin(d, d->sm0, text, D, T, tm, F) || !drelu(d, tm, static_cast<int64_t>(T) * F) ||
        !dlin(d, d->sm1, tm, F, T, tm2, D) || !dadd(d, tm2, text, static_cast<int64_t>(T) * D, tm) ||
        !dln(d, tm, T, d->sm_nw, d->sm_nb, tm2))
        return false;
    dd_pool_kernel<<<ew_blocks(D), 256, 0, s>>>(tm2, valid, T, D, d->pooled.as<float>());
    if (!dok(d, cudaGetLastError(), "ddec text pool") ||
        !dlin(d, d->spp, d->pooled.as<float>(), D, 1, d->ppool.as<float>(), D) ||
        !dlin(d, d->shs, seg + D, D, NQ, d->phs.as<float>(), D))
        return false;
    dd_score_kernel<<<ew_blocks(static_cast<int64_t>(NQ) * 32), 256, 0, s>>>(
        d->ppool.as<float>(), d->phs.as<float>(), NQ, D, 1.0f / sqrtf(static_cast<float>(D)), d->scores.as<float>());
    if (!dok(d, cudaGetLastError(), "ddec scores")) return false;
    // presence logit
    return dln(d, q, 1, d->pnw, d->pnb, d->pr1.as<float>()) &&
           mlp3(d, d->phead, d->pr1.as<float>(), 1, d->prout.as<float>(), 1);
}

bool check_ready(Ddec *d) {
    d->missing.clear();
    auto need = [&](bool ok, const std::string &n) {
        if (!ok) d->missing.push_back(n);
    };
    need(d->qemb.p && d->pres.p && d->refp.p, "ddec.query_embed / presence_token / reference_points");
    need(d->normw.p && d->normb.p && d->pnw.p && d->pnb.p, "ddec.norm / presence_token_out_norm");
    for (int j = 0; j < 3; ++j) need(d->bbox[j].set() && d->phead[j].set(), "ddec.bbox_embed / presence_token_head");
    for (int j = 0; j < 2; ++j)
        need(d->rph[j].set() && d->rpb1[j].set() && d->rpb0w[j].p && d->rpb0b[j].p, "ddec.ref_point_head / boxRPB");
    need(d->sm0.set() && d->sm1.set() && d->spp.set() && d->shs.set() && d->sm_nw.p && d->sm_nb.p, "scoring.*");
    for (size_t i = 0; i < d->ly.size(); ++i) {
        const DdecLayer &L = d->ly[i];
        need(L.sa_qk.set() && L.sa_v.set() && L.sa_o.set() && L.ct_q.set() && L.ct_kv.set() && L.ct_o.set() &&
                 L.ca_q.set() && L.ca_k.set() && L.ca_v.set() && L.ca_o.set() && L.f1.set() && L.f2.set() &&
                 L.n1w.p && L.n1b.p && L.n2w.p && L.n2b.p && L.nctw.p && L.nctb.p && L.n3w.p && L.n3b.p,
             "ddec.layers." + std::to_string(i));
    }
    if (!d->missing.empty()) {
        set_error("ddec: %zu tensors missing (first: %s)", d->missing.size(), d->missing[0].c_str());
        return false;
    }
    return true;
}

void dfree(Ddec *d, sam3b200_weight *&w) {
    if (w) sam3b200_weight_free(reinterpret_cast<sam3b200_backend *>(d->be), w);
    w = nullptr;
}

bool check_run(Ddec *d, int T) {
    if (T <= 0 || T > d->hp.max_prompt) {
        set_error("ddec_run: %d prompt tokens (max %d)", T, d->hp.max_prompt);
        return false;
    }
    return check_ready(d);
}

}  // namespace
}  // namespace b200

using namespace b200;

sam3b200_ddec *sam3b200_ddec_create(sam3b200_backend *hb, const sam3b200_ddec_hparams *hp) {
    auto *be = reinterpret_cast<Backend *>(hb);
    if (!be || !hp) return nullptr;
    const int D = hp->d_model;
    if (D != 256 || hp->heads != 8 || hp->layers <= 0 || hp->ffn_dim <= 0 || hp->ffn_dim % 32 != 0 ||
        hp->num_queries <= 0 || hp->feat <= 0 || hp->feat > 256 || hp->max_prompt <= 0) {
        set_error("ddec_create: unsupported hyperparameters (d_model 256, 8 heads, feat <= 256)");
        return nullptr;
    }
    cudaSetDevice(be->device);
    auto *d = new Ddec();
    d->be = be;
    d->hp = *hp;
    d->ly.resize(hp->layers);
    const size_t NQ = hp->num_queries, NQ1 = NQ + 1, N = static_cast<size_t>(hp->feat) * hp->feat;
    const size_t T = hp->max_prompt, F = hp->ffn_dim, S = hp->feat, dd = D;
    // angle multipliers of the query sine code, as the reference fills its sine_dim_t input
    std::vector<float> dim_t(64);
    for (int i = 0; i < 64; ++i)
        dim_t[i] = 2.0f * static_cast<float>(M_PI) / powf(10000.0f, 2.0f * static_cast<float>(i) / 128.0f);
    const bool ok =
        upload(d->dim_t, dim_t.data(), 64 * 4, be->stream) && d->q.alloc(NQ1 * dd * 4) && d->qpos.alloc(NQ1 * dd * 4) &&
        d->qin.alloc(NQ1 * dd * 4) && d->qk.alloc(2 * NQ1 * dd * 4) && d->v.alloc(NQ1 * dd * 4) &&
        d->att.alloc(NQ1 * dd * 4) && d->tmp.alloc(NQ1 * dd * 4) && d->ffn.alloc(NQ1 * F * 4) &&
        d->kvt.alloc(2 * T * dd * 4) && d->kin.alloc(N * dd * 4) && d->kimg.alloc(N * dd * 4) &&
        d->vimg.alloc(N * dd * 4) && d->tmask.alloc(NQ1 * T * 2) && d->rmask.alloc(8 * NQ1 * N * 4) &&
        d->sine.alloc(NQ * 512 * 4) && d->hid.alloc(NQ * dd * 4) && d->dxy.alloc(NQ * S * 2 * 4) &&
        d->rhid.alloc(NQ * S * dd * 4) && d->rpbx.alloc(NQ * S * 8 * 4) && d->rpby.alloc(NQ * S * 8 * 4) &&
        d->boxes.alloc(NQ * 4 * 4) && d->bd.alloc(NQ * 4 * 4) && d->objn.alloc(NQ * dd * 4) &&
        d->bh1.alloc(NQ * dd * 4) && d->bh2.alloc(NQ * dd * 4) && d->tm.alloc(T * F * 4) && d->tm2.alloc(T * dd * 4) &&
        d->pooled.alloc(dd * 4) && d->ppool.alloc(dd * 4) && d->phs.alloc(NQ * dd * 4) && d->scores.alloc(NQ * 4) &&
        d->pr1.alloc(dd * 4) && d->pr2.alloc(dd * 4) && d->prout.alloc(16) && d->seg.alloc(NQ1 * dd * 4) &&
        d->in_enc.alloc(N * dd * 4) && d->in_pos.alloc(N * dd * 4) && d->in_text.alloc(T * dd * 4) &&
        d->in_bias.alloc(T * 4) && d->in_valid.alloc(T * 4);
    if (!ok) {
        delete d;
        return nullptr;
    }
    return reinterpret_cast<sam3b200_ddec *>(d);
}

void sam3b200_ddec_free(sam3b200_ddec *hd) {
    auto *d = reinterpret_cast<Ddec *>(hd);
    if (!d) return;
    cudaSetDevice(d->be->device);
    cudaStreamSynchronize(d->be->stream);
    for (auto &L : d->ly)
        for (Lin *l : {&L.sa_qk, &L.sa_v, &L.sa_o, &L.ct_q, &L.ct_kv, &L.ct_o, &L.ca_q, &L.ca_k, &L.ca_v, &L.ca_o,
                       &L.f1, &L.f2})
            dfree(d, l->w);
    for (int j = 0; j < 3; ++j) {
        dfree(d, d->bbox[j].w);
        dfree(d, d->phead[j].w);
    }
    for (int j = 0; j < 2; ++j) {
        dfree(d, d->rph[j].w);
        dfree(d, d->rpb1[j].w);
    }
    for (Lin *l : {&d->sm0, &d->sm1, &d->spp, &d->shs}) dfree(d, l->w);
    delete d;
}

int sam3b200_ddec_set_tensor(sam3b200_ddec *hd, const char *name_c, int type, const void *data, const int64_t *ne) {
    auto *d = reinterpret_cast<Ddec *>(hd);
    if (!d || !name_c || !data || !ne) return SAM3B200_STATUS_FAILED;
    cudaSetDevice(d->be->device);
    auto *hb = reinterpret_cast<sam3b200_backend *>(d->be);
    const std::string name(name_c);
    const int64_t D = d->hp.d_model, F = d->hp.ffn_dim, NQ = d->hp.num_queries, NH = d->hp.heads;
    const int64_t n = ne[0] * (ne[1] > 0 ? ne[1] : 1) * (ne[2] > 0 ? ne[2] : 1) * (ne[3] > 0 ? ne[3] : 1);
    std::vector<float> v;
    const int OK = SAM3B200_STATUS_SUCCESS, BAD = SAM3B200_STATUS_FAILED;
    auto vec_part = [&](DevBuf &b, int64_t want, int64_t off, int64_t len) -> int {
        if (n != want || !to_f32(type, data, n, v)) {
            set_error("%s: %lld elements of type %d, expected %lld F32/F16", name_c, (long long)n, type,
                      (long long)want);
            return BAD;
        }
        return upload(b, v.data() + off, static_cast<size_t>(len) * 4, d->be->stream) ? OK : BAD;
    };
    auto vec = [&](DevBuf &b, int64_t want) { return vec_part(b, want, 0, want); };
    auto shape_ok = [&](int64_t K, int64_t N) {
        if (ne[0] == K && ne[1] == N) return true;
        set_error("%s: shape [%lld, %lld], expected [%lld, %lld]", name_c, (long long)ne[0], (long long)ne[1],
                  (long long)K, (long long)N);
        return false;
    };
    auto weight = [&](Lin &l, int64_t K, int64_t N) -> int {
        if (!shape_ok(K, N)) return BAD;
        dfree(d, l.w);
        l.w = sam3b200_weight_upload(hb, type, data, K, N);
        return l.w ? OK : BAD;
    };
    auto rows = [&](Lin &l, int64_t r0, int64_t nr) -> bool {
        dfree(d, l.w);
        l.w = upload_weight_rows(d->be, type, data, D, r0, nr);
        return l.w != nullptr;
    };
    // "<prefix>.weight" / ".bias" of a plain linear layer
    auto linear = [&](const std::string &pfx, Lin &l, int64_t K, int64_t N, int &st) -> bool {
        if (name == pfx + ".weight") return st = weight(l, K, N), true;
        if (name == pfx + ".bias") return st = vec(l.b, N), true;
        return false;
    };
    int st = BAD;
    if (name == "ddec.query_embed.weight") return vec(d->qemb, D * NQ);
    if (name == "ddec.presence_token.weight") return vec(d->pres, D);
    if (name == "ddec.reference_points.weight") return vec(d->refp, 4 * NQ);
    if (name == "ddec.norm.weight") return vec(d->normw, D);
    if (name == "ddec.norm.bias") return vec(d->normb, D);
    if (name == "ddec.presence_token_out_norm.weight") return vec(d->pnw, D);
    if (name == "ddec.presence_token_out_norm.bias") return vec(d->pnb, D);
    if (name == "scoring.prompt_mlp.out_norm.weight") return vec(d->sm_nw, D);
    if (name == "scoring.prompt_mlp.out_norm.bias") return vec(d->sm_nb, D);
    for (int j = 0; j < 3; ++j) {
        const std::string jj = std::to_string(j);
        if (linear("ddec.bbox_embed.layers." + jj, d->bbox[j], D, j == 2 ? 4 : D, st)) return st;
        if (linear("ddec.presence_token_head.layers." + jj, d->phead[j], D, j == 2 ? 1 : D, st)) return st;
    }
    if (linear("ddec.ref_point_head.layers.0", d->rph[0], 512, D, st)) return st;
    if (linear("ddec.ref_point_head.layers.1", d->rph[1], D, D, st)) return st;
    for (int a = 0; a < 2; ++a) {
        const std::string p = std::string("ddec.boxRPB_embed_") + (a == 0 ? "x" : "y") + ".layers.";
        if (name == p + "0.weight") {  // [2, D]: kept in f32 for dd_rpb0_kernel
            if (!shape_ok(2, D)) return BAD;
            d->rpb0_f16[a] = type == SAM3B200_TYPE_F16;
            return vec(d->rpb0w[a], 2 * D);
        }
        if (name == p + "0.bias") return vec(d->rpb0b[a], D);
        if (linear(p + "1", d->rpb1[a], D, NH, st)) return st;
    }
    if (linear("scoring.prompt_mlp.layers.0", d->sm0, D, F, st)) return st;
    if (linear("scoring.prompt_mlp.layers.1", d->sm1, F, D, st)) return st;
    if (linear("scoring.prompt_proj", d->spp, D, D, st)) return st;
    if (linear("scoring.hs_proj", d->shs, D, D, st)) return st;
    int li = -1;
    char tail[64] = {0};
    if (sscanf(name_c, "ddec.layers.%d.%63s", &li, tail) == 2 && li >= 0 && li < static_cast<int>(d->ly.size())) {
        DdecLayer &L = d->ly[li];
        const std::string t(tail);
        if (t == "sa.in_proj_weight")
            return shape_ok(D, 3 * D) && rows(L.sa_qk, 0, 2 * D) && rows(L.sa_v, 2 * D, D) ? OK : BAD;
        if (t == "sa.in_proj_bias") return vec_part(L.sa_qk.b, 3 * D, 0, 2 * D) == OK ? vec_part(L.sa_v.b, 3 * D, 2 * D, D) : BAD;
        if (t == "ca_text.in_proj_weight")
            return shape_ok(D, 3 * D) && rows(L.ct_q, 0, D) && rows(L.ct_kv, D, 2 * D) ? OK : BAD;
        if (t == "ca_text.in_proj_bias") return vec_part(L.ct_q.b, 3 * D, 0, D) == OK ? vec_part(L.ct_kv.b, 3 * D, D, 2 * D) : BAD;
        if (t == "ca.in_proj_weight")
            return shape_ok(D, 3 * D) && rows(L.ca_q, 0, D) && rows(L.ca_k, D, D) && rows(L.ca_v, 2 * D, D) ? OK : BAD;
        if (t == "ca.in_proj_bias")
            return vec_part(L.ca_q.b, 3 * D, 0, D) == OK && vec_part(L.ca_k.b, 3 * D, D, D) == OK
                       ? vec_part(L.ca_v.b, 3 * D, 2 * D, D)
                       : BAD;
        const std::string p = "ddec.layers." + std::to_string(li) + ".";
        if (linear(p + "sa.out_proj", L.sa_o, D, D, st)) return st;
        if (linear(p + "ca_text.out_proj", L.ct_o, D, D, st)) return st;
        if (linear(p + "ca.out_proj", L.ca_o, D, D, st)) return st;
        if (linear(p + "linear1", L.f1, D, F, st)) return st;
        if (linear(p + "linear2", L.f2, F, D, st)) return st;
        if (t == "norm1.weight") return vec(L.n1w, D);
        if (t == "norm1.bias") return vec(L.n1b, D);
        if (t == "norm2.weight") return vec(L.n2w, D);
        if (t == "norm2.bias") return vec(L.n2b, D);
        if (t == "norm_ca_text.weight") return vec(L.nctw, D);
        if (t == "norm_ca_text.bias") return vec(L.nctb, D);
        if (t == "norm3.weight") return vec(L.n3w, D);
        if (t == "norm3.bias") return vec(L.n3b, D);
    }
    set_error("ddec: unknown tensor %s", name_c);
    return BAD;
}

int sam3b200_ddec_missing(sam3b200_ddec *hd, char *buf, int cap) {
    auto *d = reinterpret_cast<Ddec *>(hd);
    if (!d) return -1;
    check_ready(d);
    std::string all;
    for (const auto &s : d->missing) all += s + "\n";
    if (buf && cap > 0) snprintf(buf, static_cast<size_t>(cap), "%s", all.c_str());
    return static_cast<int>(d->missing.size());
}

int sam3b200_ddec_run_device(sam3b200_ddec *hd, const float *enc_feats, const float *enc_pos, const float *text,
                             const float *text_bias, const float *text_valid, int n_text) {
    auto *d = reinterpret_cast<Ddec *>(hd);
    if (!d || !enc_feats || !enc_pos || !text) {
        set_error("ddec_run: null argument");
        return SAM3B200_STATUS_FAILED;
    }
    cudaSetDevice(d->be->device);
    if (!check_run(d, n_text)) return SAM3B200_STATUS_FAILED;
    return forward(d, enc_feats, enc_pos, text, text_bias, text_valid, n_text) ? SAM3B200_STATUS_SUCCESS
                                                                               : SAM3B200_STATUS_FAILED;
}

int sam3b200_ddec_run(sam3b200_ddec *hd, const float *enc_feats, const float *enc_pos, const float *text,
                      const float *text_bias, const float *text_valid, int n_text) {
    auto *d = reinterpret_cast<Ddec *>(hd);
    if (!d || !enc_feats || !enc_pos || !text) {
        set_error("ddec_run: null argument");
        return SAM3B200_STATUS_FAILED;
    }
    cudaSetDevice(d->be->device);
    if (!check_run(d, n_text)) return SAM3B200_STATUS_FAILED;
    const size_t nd = static_cast<size_t>(d->hp.feat) * d->hp.feat * d->hp.d_model * 4;
    const size_t td = static_cast<size_t>(n_text) * d->hp.d_model * 4, tb = static_cast<size_t>(n_text) * 4;
    cudaStream_t s = d->be->stream;
    if (!cuda_ok(cudaMemcpyAsync(d->in_enc.p, enc_feats, nd, cudaMemcpyHostToDevice, s), "ddec enc") ||
        !cuda_ok(cudaMemcpyAsync(d->in_pos.p, enc_pos, nd, cudaMemcpyHostToDevice, s), "ddec pos") ||
        !cuda_ok(cudaMemcpyAsync(d->in_text.p, text, td, cudaMemcpyHostToDevice, s), "ddec text") ||
        (text_bias && !cuda_ok(cudaMemcpyAsync(d->in_bias.p, text_bias, tb, cudaMemcpyHostToDevice, s), "bias")) ||
        (text_valid && !cuda_ok(cudaMemcpyAsync(d->in_valid.p, text_valid, tb, cudaMemcpyHostToDevice, s), "valid")))
        return SAM3B200_STATUS_FAILED;
    return forward(d, d->in_enc.as<float>(), d->in_pos.as<float>(), d->in_text.as<float>(),
                   text_bias ? d->in_bias.as<float>() : nullptr, text_valid ? d->in_valid.as<float>() : nullptr,
                   n_text)
               ? SAM3B200_STATUS_SUCCESS
               : SAM3B200_STATUS_FAILED;
}

int sam3b200_ddec_outputs(sam3b200_ddec *hd, const float **queries, const float **boxes, const float **scores,
                          const float **presence) {
    auto *d = reinterpret_cast<Ddec *>(hd);
    if (!d) return SAM3B200_STATUS_FAILED;
    if (queries) *queries = d->seg.as<float>();
    if (boxes) *boxes = d->boxes.as<float>();
    if (scores) *scores = d->scores.as<float>();
    if (presence) *presence = d->prout.as<float>();
    return SAM3B200_STATUS_SUCCESS;
}
