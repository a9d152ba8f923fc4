// geom.cu -- the geometry (exemplar-prompt) encoder of the SAM3 detector on
// the B200 backend: the transformer of sam3_build_geom_enc_graph
// (sam3.cpp:7677-7800) over the prompt's geometry tokens (box embeddings + CLS,
// prepared on the host by sam3_precompute_geom_input as in the reference):
//
//   per layer: x += sa_out(attn(LN1(x)))                       q = k = v, no position
//              x += ca_out(attn(LN2(x); k from img + pe, v from img))
//              x += fc2(relu(fc1(LN3(x))))
//   out = LN(x)                                                 encode_norm
//
// Fused in_proj weights are split by rows at load (self-attention: one
// [D, 3D] GEMM over LN1(x); cross-attention: q rows, then k and v rows as
// separate GEMMs over img + pe and img).  Attention is attention_simt (fp32;
// at most a few geometry tokens per call).
#include "../../include/sam3_b200.h"
#include "attn_simt.cuh"
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

struct GeomLayer {
    DevBuf n1w, n1b, n2w, n2b, n3w, n3b;
    DevBuf sqkv_b, so_b, cq_b, ck_b, cv_b, co_b, f1_b, f2_b;
    sam3b200_weight *sqkv = nullptr, *so = nullptr, *cq = nullptr, *ck = nullptr, *cv = nullptr, *co = nullptr;
    sam3b200_weight *f1 = nullptr, *f2 = nullptr;
};

}  // namespace

struct Geom {
    Backend *be = nullptr;
    sam3b200_geom_hparams hp{};
    std::vector<GeomLayer> ly;
    DevBuf encw, encb;
    DevBuf x, xn, qkv, att, tmp, ffn, kin, kimg, vimg, out, in_x, in_img, in_pe;
    std::vector<std::string> missing;
};

namespace {

bool gok(Geom *g, cudaError_t e, const char *what) {
    g->be->count(1);
    return cuda_ok(e, what);
}

bool glin(Geom *g, const sam3b200_weight *w, const float *x, int64_t ldx, int64_t rows, const DevBuf &b, float *y,
          int64_t ldy) {
    return run_mul_mat(g->be, reinterpret_cast<const Weight *>(w), x, ldx, rows, b.as<float>(), y, ldy, nullptr) ==
           SAM3B200_STATUS_SUCCESS;
}

bool forward(Geom *g, const float *x_in, const float *img, const float *pe, int S, int N) {
    const int D = g->hp.d_model, H = g->hp.heads, HD = D / H, F = g->hp.ffn_dim;
    const int64_t sd = static_cast<int64_t>(S) * D, nd = static_cast<int64_t>(N) * D;
    cudaStream_t s = g->be->stream;
    float *x = g->x.as<float>(), *xn = g->xn.as<float>(), *qkv = g->qkv.as<float>(), *att = g->att.as<float>();
    float *tmp = g->tmp.as<float>(), *kin = g->kin.as<float>(), *kimg = g->kimg.as<float>(), *vimg = g->vimg.as<float>();
    const float scale = 1.0f / sqrtf(static_cast<float>(HD));
    const AttnStrides s1{0, HD, D}, s3{0, HD, 3 * D};
    auto ln = [&](const float *src, const DevBuf &w, const DevBuf &b, float *dst) {
        ln_rows_kernel<<<ew_blocks(static_cast<int64_t>(S) * 32), 256, 0, s>>>(src, S, D, w.as<float>(),
                                                                              b.as<float>(), 1e-5f, dst);
        return gok(g, cudaGetLastError(), "geom layer norm");
    };
    auto add = [&](const float *a, const float *b, int64_t n, float *c) {
        ew_add_kernel<<<ew_blocks(n), 256, 0, s>>>(a, b, n, c);
        return gok(g, cudaGetLastError(), "geom add");
    };
    if (!gok(g, cudaMemcpyAsync(x, x_in, sd * 4, cudaMemcpyDeviceToDevice, s), "geom input") ||
        !add(img, pe, nd, kin))
        return false;
    for (const GeomLayer &L : g->ly) {
        if (!ln(x, L.n1w, L.n1b, xn) || !glin(g, L.sqkv, xn, D, S, L.sqkv_b, qkv, 3 * D) ||
            !gok(g, attention_simt(HD, qkv, s3, S, qkv + D, s3, qkv + 2 * D, s3, S, 1, H, nullptr, 0, scale, att, s1, s),
                 "geom self attention") ||
            !glin(g, L.so, att, D, S, L.so_b, tmp, D) || !add(x, tmp, sd, x))
            return false;
        if (!ln(x, L.n2w, L.n2b, xn) || !glin(g, L.cq, xn, D, S, L.cq_b, qkv, D) ||
            !glin(g, L.ck, kin, D, N, L.ck_b, kimg, D) || !glin(g, L.cv, img, D, N, L.cv_b, vimg, D) ||
            !gok(g, attention_simt(HD, qkv, s1, S, kimg, s1, vimg, s1, N, 1, H, nullptr, 0, scale, att, s1, s),
                 "geom cross attention") ||
            !glin(g, L.co, att, D, S, L.co_b, tmp, D) || !add(x, tmp, sd, x))
            return false;
        if (!ln(x, L.n3w, L.n3b, xn) || !glin(g, L.f1, xn, D, S, L.f1_b, g->ffn.as<float>(), F)) return false;
        ew_relu_kernel<<<ew_blocks(static_cast<int64_t>(S) * F), 256, 0, s>>>(g->ffn.as<float>(),
                                                                              static_cast<int64_t>(S) * F);
        if (!gok(g, cudaGetLastError(), "geom relu") || !glin(g, L.f2, g->ffn.as<float>(), F, S, L.f2_b, tmp, D) ||
            !add(x, tmp, sd, x))
            return false;
    }
    return ln(x, g->encw, g->encb, g->out.as<float>());
}

bool check_ready(Geom *g) {
    g->missing.clear();
    if (!g->encw.p || !g->encb.p) g->missing.push_back("geom.encode_norm");
    for (size_t i = 0; i < g->ly.size(); ++i) {
        const GeomLayer &L = g->ly[i];
        const bool ok = L.sqkv && L.so && L.cq && L.ck && L.cv && L.co && L.f1 && L.f2 && L.sqkv_b.p && L.so_b.p &&
                        L.cq_b.p && L.ck_b.p && L.cv_b.p && L.co_b.p && L.f1_b.p && L.f2_b.p && L.n1w.p && L.n1b.p &&
                        L.n2w.p && L.n2b.p && L.n3w.p && L.n3b.p;
        if (!ok) g->missing.push_back("geom.layers." + std::to_string(i));
    }
    if (!g->missing.empty()) {
        set_error("geom: %zu tensors missing (first: %s)", g->missing.size(), g->missing[0].c_str());
        return false;
    }
    return true;
}

void gfree(Geom *g, sam3b200_weight *&w) {
    if (w) sam3b200_weight_free(reinterpret_cast<sam3b200_backend *>(g->be), w);
    w = nullptr;
}

bool check_run(Geom *g, int S, int N) {
    if (S <= 0 || S > g->hp.max_tokens || N <= 0 || N > g->hp.max_image_tokens) {
        set_error("geom_run: %d geometry tokens (max %d), %d image tokens (max %d)", S, g->hp.max_tokens, N,
                  g->hp.max_image_tokens);
        return false;
    }
    return check_ready(g);
}

}  // namespace
}  // namespace b200

using namespace b200;

sam3b200_geom *sam3b200_geom_create(sam3b200_backend *hb, const sam3b200_geom_hparams *hp) {
    auto *be = reinterpret_cast<Backend *>(hb);
    if (!be || !hp) return nullptr;
    const int D = hp->d_model;
    const int HD = hp->heads > 0 && D % hp->heads == 0 ? D / hp->heads : 0;
    if (D <= 0 || D % 32 != 0 || (HD != 16 && HD != 32 && HD != 64 && HD != 128) || hp->layers <= 0 ||
        hp->ffn_dim <= 0 || hp->ffn_dim % 32 != 0 || hp->max_tokens <= 0 || hp->max_image_tokens <= 0) {
        set_error("geom_create: unsupported hyperparameters (head dim 16/32/64/128, widths multiples of 32)");
        return nullptr;
    }
    cudaSetDevice(be->device);
    auto *g = new Geom();
    g->be = be;
    g->hp = *hp;
    g->ly.resize(hp->layers);
    const size_t S = hp->max_tokens, N = hp->max_image_tokens, d = D;
    const bool ok = g->x.alloc(S * d * 4) && g->xn.alloc(S * d * 4) && g->qkv.alloc(3 * S * d * 4) &&
                    g->att.alloc(S * d * 4) && g->tmp.alloc(S * d * 4) && g->ffn.alloc(S * hp->ffn_dim * 4) &&
                    g->kin.alloc(N * d * 4) && g->kimg.alloc(N * d * 4) && g->vimg.alloc(N * d * 4) &&
                    g->out.alloc(S * d * 4) && g->in_x.alloc(S * d * 4) && g->in_img.alloc(N * d * 4) &&
                    g->in_pe.alloc(N * d * 4);
    if (!ok) {
        delete g;
        return nullptr;
    }
    return reinterpret_cast<sam3b200_geom *>(g);
}

void sam3b200_geom_free(sam3b200_geom *hg) {
    auto *g = reinterpret_cast<Geom *>(hg);
    if (!g) return;
    cudaSetDevice(g->be->device);
    cudaStreamSynchronize(g->be->stream);
    for (auto &L : g->ly)
        for (sam3b200_weight **w : {&L.sqkv, &L.so, &L.cq, &L.ck, &L.cv, &L.co, &L.f1, &L.f2}) gfree(g, *w);
    delete g;
}

int sam3b200_geom_set_tensor(sam3b200_geom *hg, const char *name_c, int type, const void *data, const int64_t *ne) {
    auto *g = reinterpret_cast<Geom *>(hg);
    if (!g || !name_c || !data || !ne) return SAM3B200_STATUS_FAILED;
    cudaSetDevice(g->be->device);
    auto *hb = reinterpret_cast<sam3b200_backend *>(g->be);
    const std::string name(name_c);
    const int64_t D = g->hp.d_model, F = g->hp.ffn_dim;
    const int64_t n = ne[0] * (ne[1] > 0 ? ne[1] : 1) * (ne[2] > 0 ? ne[2] : 1) * (ne[3] > 0 ? ne[3] : 1);
    const int OK = SAM3B200_STATUS_SUCCESS, BAD = SAM3B200_STATUS_FAILED;
    std::vector<float> v;
    auto vec_part = [&](DevBuf &b, int64_t want, int64_t off, int64_t len) -> int {
        if (n != want || !to_f32(type, data, n, v)) {
            set_error("%s: %lld elements of type %d, expected %lld F32/F16", name_c, (long long)n, type,
                      (long long)want);
            return BAD;
        }
        return upload(b, v.data() + off, static_cast<size_t>(len) * 4, g->be->stream) ? OK : BAD;
    };
    auto vec = [&](DevBuf &b, int64_t want) { return vec_part(b, want, 0, want); };
    auto shape_ok = [&](int64_t K, int64_t N) {
        if (ne[0] == K && ne[1] == N) return true;
        set_error("%s: shape [%lld, %lld], expected [%lld, %lld]", name_c, (long long)ne[0], (long long)ne[1],
                  (long long)K, (long long)N);
        return false;
    };
    auto rows = [&](sam3b200_weight *&w, int64_t r0, int64_t nr) -> bool {
        gfree(g, w);
        w = upload_weight_rows(g->be, type, data, D, r0, nr);
        return w != nullptr;
    };
    auto weight = [&](sam3b200_weight *&w, int64_t K, int64_t N) -> int {
        if (!shape_ok(K, N)) return BAD;
        gfree(g, w);
        w = sam3b200_weight_upload(hb, type, data, K, N);
        return w ? OK : BAD;
    };
    if (name == "geom.encode_norm.weight") return vec(g->encw, D);
    if (name == "geom.encode_norm.bias") return vec(g->encb, D);
    int li = -1;
    char tail[64] = {0};
    if (sscanf(name_c, "geom.layers.%d.%63s", &li, tail) == 2 && li >= 0 && li < static_cast<int>(g->ly.size())) {
        GeomLayer &L = g->ly[li];
        const std::string t(tail);
        if (t == "sa.in_proj_weight") return shape_ok(D, 3 * D) && rows(L.sqkv, 0, 3 * D) ? OK : BAD;
        if (t == "sa.in_proj_bias") return vec(L.sqkv_b, 3 * D);
        if (t == "ca.in_proj_weight")
            return shape_ok(D, 3 * D) && rows(L.cq, 0, D) && rows(L.ck, D, D) && rows(L.cv, 2 * D, D) ? OK : BAD;
        if (t == "ca.in_proj_bias")
            return vec_part(L.cq_b, 3 * D, 0, D) == OK && vec_part(L.ck_b, 3 * D, D, D) == OK
                       ? vec_part(L.cv_b, 3 * D, 2 * D, D)
                       : BAD;
        if (t == "sa.out_proj.weight") return weight(L.so, D, D);
        if (t == "sa.out_proj.bias") return vec(L.so_b, D);
        if (t == "ca.out_proj.weight") return weight(L.co, D, D);
        if (t == "ca.out_proj.bias") return vec(L.co_b, D);
        if (t == "linear1.weight") return weight(L.f1, D, F);
        if (t == "linear1.bias") return vec(L.f1_b, F);
        if (t == "linear2.weight") return weight(L.f2, F, D);
        if (t == "linear2.bias") return vec(L.f2_b, D);
        if (t == "norm1.weight") return vec(L.n1w, D);
        if (t == "norm1.bias") return vec(L.n1b, D);
        if (t == "norm2.weight") return vec(L.n2w, D);
        if (t == "norm2.bias") return vec(L.n2b, D);
        if (t == "norm3.weight") return vec(L.n3w, D);
        if (t == "norm3.bias") return vec(L.n3b, D);
    }
    set_error("geom: unknown tensor %s", name_c);
    return BAD;
}

int sam3b200_geom_missing(sam3b200_geom *hg, char *buf, int cap) {
    auto *g = reinterpret_cast<Geom *>(hg);
    if (!g) return -1;
    check_ready(g);
    std::string all;
    for (const auto &s : g->missing) all += s + "\n";
    if (buf && cap > 0) snprintf(buf, static_cast<size_t>(cap), "%s", all.c_str());
    return static_cast<int>(g->missing.size());
}

int sam3b200_geom_run_device(sam3b200_geom *hg, const float *tokens, int n_tokens, const float *img_feats,
                             const float *img_pe, int n_image) {
    auto *g = reinterpret_cast<Geom *>(hg);
    if (!g || !tokens || !img_feats || !img_pe) {
        set_error("geom_run: null argument");
        return SAM3B200_STATUS_FAILED;
    }
    cudaSetDevice(g->be->device);
    if (!check_run(g, n_tokens, n_image)) return SAM3B200_STATUS_FAILED;
    return forward(g, tokens, img_feats, img_pe, n_tokens, n_image) ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
}

int sam3b200_geom_run(sam3b200_geom *hg, const float *tokens, int n_tokens, const float *img_feats,
                      const float *img_pe, int n_image) {
    auto *g = reinterpret_cast<Geom *>(hg);
    if (!g || !tokens || !img_feats || !img_pe) {
        set_error("geom_run: null argument");
        return SAM3B200_STATUS_FAILED;
    }
    cudaSetDevice(g->be->device);
    if (!check_run(g, n_tokens, n_image)) return SAM3B200_STATUS_FAILED;
    const size_t D = g->hp.d_model;
    cudaStream_t s = g->be->stream;
    if (!cuda_ok(cudaMemcpyAsync(g->in_x.p, tokens, n_tokens * D * 4, cudaMemcpyHostToDevice, s), "geom tokens") ||
        !cuda_ok(cudaMemcpyAsync(g->in_img.p, img_feats, n_image * D * 4, cudaMemcpyHostToDevice, s), "geom img") ||
        !cuda_ok(cudaMemcpyAsync(g->in_pe.p, img_pe, n_image * D * 4, cudaMemcpyHostToDevice, s), "geom pe"))
        return SAM3B200_STATUS_FAILED;
    return forward(g, g->in_x.as<float>(), g->in_img.as<float>(), g->in_pe.as<float>(), n_tokens, n_image)
               ? SAM3B200_STATUS_SUCCESS
               : SAM3B200_STATUS_FAILED;
}

int sam3b200_geom_output(sam3b200_geom *hg, const float **dev) {
    auto *g = reinterpret_cast<Geom *>(hg);
    if (!g || !dev) return SAM3B200_STATUS_FAILED;
    *dev = g->out.as<float>();
    return SAM3B200_STATUS_SUCCESS;
}
