// fenc.cu -- the fusion encoder of the SAM3 detector on the B200 backend: the
// graph sam3_build_fenc_graph builds (sam3.cpp:8146-8165; layer
// sam3_fenc_layer_forward :8033-8139), conditioning the detector's image
// tokens on the prompt tokens:
//
//   per layer: x += sa_out(attn(q, k from LN1(x) + pos; v from LN1(x)))
//              x += ca_out(attn(q from LN2(x); k, v from prompt; padding bias))
//              x += fc2(relu(fc1(LN3(x))))
//
// The fused in_proj weights [D, 3D] are split by rows when they are set: the
// self-attention's q and k rows form one [D, 2D] weight (both read LN1(x) +
// pos), its v rows another; the cross-attention's q rows one, its k and v
// rows one [D, 2D] weight over the prompt.  Every output element is the same
// row dot as in the reference's per-view MUL_MATs.  Attention is
// attention_mma on the strided q/k/v (tensor cores, 8 heads of 32 channels); the padding
// bias is cast to the fp16 mask of FLASH_ATTN_EXT.
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

struct FencLayer {
    DevBuf n1w, n1b, n2w, n2b, n3w, n3b;
    DevBuf sqk_b, sv_b, so_b, cq_b, ckv_b, co_b, f1_b, f2_b;
    sam3b200_weight *sqk = nullptr, *sv = nullptr, *so = nullptr, *cq = nullptr, *ckv = nullptr, *co = nullptr;
    sam3b200_weight *f1 = nullptr, *f2 = nullptr;
};

}  // namespace

struct Fenc {
    Backend *be = nullptr;
    sam3b200_fenc_hparams hp{};
    std::vector<FencLayer> ly;
    DevBuf x, xn, qin, qk, v, att, tmp, ffn, kv, mask, in_img, in_prompt, in_pos, in_bias;
    std::vector<std::string> missing;
};

namespace {

bool fok(Fenc *f, cudaError_t e, const char *what) {
    f->be->count(1);
    return cuda_ok(e, what);
}

bool flin(Fenc *f, const sam3b200_weight *w, const float *x, int64_t ldx, int64_t rows, const DevBuf &b, float *y,
          int64_t ldy) {
    return run_mul_mat(f->be, reinterpret_cast<const Weight *>(w), x, ldx, rows, b.as<float>(), y, ldy, nullptr) ==
           SAM3B200_STATUS_SUCCESS;
}

bool forward(Fenc *f, const float *img, const float *prompt, const float *pos, const float *bias, int N, int T) {
    const int D = f->hp.d_model, H = f->hp.heads, HD = D / H, F = f->hp.ffn_dim;
    const int64_t nd = static_cast<int64_t>(N) * D;
    cudaStream_t s = f->be->stream;
    float *x = f->x.as<float>(), *xn = f->xn.as<float>(), *qin = f->qin.as<float>(), *qk = f->qk.as<float>();
    float *v = f->v.as<float>(), *att = f->att.as<float>(), *tmp = f->tmp.as<float>(), *kv = f->kv.as<float>();
    const float scale = 1.0f / sqrtf(static_cast<float>(HD));
    const __half *mask = nullptr;
    if (bias) {
        ew_bias_mask_kernel<<<ew_blocks(static_cast<int64_t>(N) * T), 256, 0, s>>>(bias, N, T, f->mask.as<__half>());
        if (!fok(f, cudaGetLastError(), "fenc prompt mask")) return false;
        mask = f->mask.as<__half>();
    }
    if (!fok(f, cudaMemcpyAsync(x, img, nd * 4, cudaMemcpyDeviceToDevice, s), "fenc input")) return false;
    const AttnStrides s2{0, HD, 2 * D}, s1{0, HD, D};
    auto ln = [&](const DevBuf &w, const DevBuf &b) {
        ln_rows_kernel<<<ew_blocks(static_cast<int64_t>(N) * 32), 256, 0, s>>>(x, N, D, w.as<float>(), b.as<float>(),
                                                                              1e-5f, xn);
        return fok(f, cudaGetLastError(), "fenc layer norm");
    };
    auto add = [&](float *a, const float *b, int64_t n, float *c) {
        ew_add_kernel<<<ew_blocks(n), 256, 0, s>>>(a, b, n, c);
        return fok(f, cudaGetLastError(), "fenc add");
    };
    for (const FencLayer &L : f->ly) {
        // self-attention: q, k from LN1(x) + pos, v from LN1(x)
        if (!ln(L.n1w, L.n1b) || !add(xn, pos, nd, qin) || !flin(f, L.sqk, qin, D, N, L.sqk_b, qk, 2 * D) ||
            !flin(f, L.sv, xn, D, N, L.sv_b, v, D) ||
            !fok(f, attention_mma(HD, qk, s2, N, qk + D, s2, v, s1, N, 1, H, nullptr, 0, scale, att, s1, s),
                 "fenc self attention") ||
            !flin(f, L.so, att, D, N, L.so_b, tmp, D) || !add(x, tmp, nd, x))
            return false;
        // cross-attention to the prompt tokens
        if (!ln(L.n2w, L.n2b) || !flin(f, L.cq, xn, D, N, L.cq_b, qin, D) ||
            !flin(f, L.ckv, prompt, D, T, L.ckv_b, kv, 2 * D) ||
            !fok(f, attention_mma(HD, qin, s1, N, kv, s2, kv + D, s2, T, 1, H, mask, T, scale, att, s1, s),
                 "fenc cross attention") ||
            !flin(f, L.co, att, D, N, L.co_b, tmp, D) || !add(x, tmp, nd, x))
            return false;
        // feed-forward
        if (!ln(L.n3w, L.n3b) || !flin(f, L.f1, xn, D, N, L.f1_b, f->ffn.as<float>(), F)) return false;
        ew_relu_kernel<<<ew_blocks(static_cast<int64_t>(N) * F), 256, 0, s>>>(f->ffn.as<float>(),
                                                                              static_cast<int64_t>(N) * F);
        if (!fok(f, cudaGetLastError(), "fenc relu") || !flin(f, L.f2, f->ffn.as<float>(), F, N, L.f2_b, tmp, D) ||
            !add(x, tmp, nd, x))
            return false;
    }
    return true;
}

bool check_ready(Fenc *f) {
    f->missing.clear();
    for (size_t i = 0; i < f->ly.size(); ++i) {
        const FencLayer &L = f->ly[i];
        const bool ok = L.sqk && L.sv && L.so && L.cq && L.ckv && L.co && L.f1 && L.f2 && L.sqk_b.p && L.sv_b.p &&
                        L.so_b.p && L.cq_b.p && L.ckv_b.p && L.co_b.p && L.f1_b.p && L.f2_b.p && L.n1w.p &&
                        L.n1b.p && L.n2w.p && L.n2b.p && L.n3w.p && L.n3b.p;
        if (!ok) f->missing.push_back("fenc.layers." + std::to_string(i));
    }
    if (!f->missing.empty()) {
        set_error("fenc: %zu tensors missing (first: %s)", f->missing.size(), f->missing[0].c_str());
        return false;
    }
    return true;
}

void ffree(Fenc *f, sam3b200_weight *&w) {
    if (w) sam3b200_weight_free(reinterpret_cast<sam3b200_backend *>(f->be), w);
    w = nullptr;
}

bool check_run(Fenc *f, int N, int T) {
    if (N <= 0 || N > f->hp.max_tokens || T <= 0 || T > f->hp.max_prompt) {
        set_error("fenc_run: %d image tokens (max %d), %d prompt tokens (max %d)", N, f->hp.max_tokens, T,
                  f->hp.max_prompt);
        return false;
    }
    return check_ready(f);
}

}  // namespace

}  // namespace b200

using namespace b200;

sam3b200_fenc *sam3b200_fenc_create(sam3b200_backend *hb, const sam3b200_fenc_hparams *hp) {
    auto *be = reinterpret_cast<Backend *>(hb);
    if (!be || !hp) return nullptr;
    const int D = hp->d_model;
    const int HD = hp->heads > 0 && D % hp->heads == 0 ? D / hp->heads : 0;
    if (D <= 0 || D % 32 != 0 || !attention_mma_supported(HD) || hp->layers <= 0 ||
        hp->ffn_dim <= 0 || hp->ffn_dim % 32 != 0 || hp->max_tokens <= 0 || hp->max_prompt <= 0) {
        set_error("fenc_create: unsupported hyperparameters (head dim 32/64/128/256, widths multiples of 32)");
        return nullptr;
    }
    cudaSetDevice(be->device);
    auto *f = new Fenc();
    f->be = be;
    f->hp = *hp;
    f->ly.resize(hp->layers);
    const size_t N = hp->max_tokens, T = hp->max_prompt, d = D;
    const bool ok = f->x.alloc(N * d * 4) && f->xn.alloc(N * d * 4) && f->qin.alloc(N * d * 4) &&
                    f->qk.alloc(2 * N * d * 4) && f->v.alloc(N * d * 4) && f->att.alloc(N * d * 4) &&
                    f->tmp.alloc(N * d * 4) && f->ffn.alloc(N * hp->ffn_dim * 4) && f->kv.alloc(2 * T * d * 4) &&
                    f->mask.alloc(N * T * 2) && f->in_img.alloc(N * d * 4) && f->in_prompt.alloc(T * d * 4) &&
                    f->in_pos.alloc(N * d * 4) && f->in_bias.alloc(T * 4);
    if (!ok) {
        delete f;
        return nullptr;
    }
    return reinterpret_cast<sam3b200_fenc *>(f);
}

void sam3b200_fenc_free(sam3b200_fenc *hf) {
    auto *f = reinterpret_cast<Fenc *>(hf);
    if (!f) return;
    cudaSetDevice(f->be->device);
    cudaStreamSynchronize(f->be->stream);
    for (auto &L : f->ly)
        for (sam3b200_weight **w : {&L.sqk, &L.sv, &L.so, &L.cq, &L.ckv, &L.co, &L.f1, &L.f2}) ffree(f, *w);
    delete f;
}

int sam3b200_fenc_set_tensor(sam3b200_fenc *hf, const char *name_c, int type, const void *data, const int64_t *ne) {
    auto *f = reinterpret_cast<Fenc *>(hf);
    if (!f || !name_c || !data || !ne) return SAM3B200_STATUS_FAILED;
    cudaSetDevice(f->be->device);
    auto *hb = reinterpret_cast<sam3b200_backend *>(f->be);
    const int64_t D = f->hp.d_model, F = f->hp.ffn_dim;
    const int64_t n = ne[0] * (ne[1] > 0 ? ne[1] : 1) * (ne[2] > 0 ? ne[2] : 1) * (ne[3] > 0 ? ne[3] : 1);
    std::vector<float> v;
    auto vec_part = [&](DevBuf &d, int64_t want, int64_t off, int64_t len) -> int {
        if (n != want || !to_f32(type, data, n, v)) {
            set_error("%s: %lld elements of type %d, expected %lld F32/F16", name_c, (long long)n, type,
                      (long long)want);
            return SAM3B200_STATUS_FAILED;
        }
        return upload(d, v.data() + off, static_cast<size_t>(len) * 4, f->be->stream) ? SAM3B200_STATUS_SUCCESS
                                                                                      : SAM3B200_STATUS_FAILED;
    };
    auto vec = [&](DevBuf &d, int64_t want) { return vec_part(d, want, 0, want); };
    auto shape_ok = [&](int64_t K, int64_t N) {
        if (ne[0] == K && ne[1] == N) return true;
        set_error("%s: shape [%lld, %lld], expected [%lld, %lld]", name_c, (long long)ne[0], (long long)ne[1],
                  (long long)K, (long long)N);
        return false;
    };
    auto rows = [&](sam3b200_weight *&w, int64_t r0, int64_t nr) -> bool {
        ffree(f, w);
        w = upload_weight_rows(f->be, type, data, D, r0, nr);
        return w != nullptr;
    };
    auto weight = [&](sam3b200_weight *&w, int64_t K, int64_t N) -> int {
        if (!shape_ok(K, N)) return SAM3B200_STATUS_FAILED;
        ffree(f, w);
        w = sam3b200_weight_upload(hb, type, data, K, N);
        return w ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
    };
    int li = -1;
    char tail[64] = {0};
    if (sscanf(name_c, "fenc.layers.%d.%63s", &li, tail) == 2 && li >= 0 && li < static_cast<int>(f->ly.size())) {
        FencLayer &L = f->ly[li];
        const std::string t(tail);
        if (t == "sa.in_proj_weight")
            return shape_ok(D, 3 * D) && rows(L.sqk, 0, 2 * D) && rows(L.sv, 2 * D, D) ? SAM3B200_STATUS_SUCCESS
                                                                                      : SAM3B200_STATUS_FAILED;
        if (t == "sa.in_proj_bias") {
            const int st = vec_part(L.sqk_b, 3 * D, 0, 2 * D);
            return st == SAM3B200_STATUS_SUCCESS ? vec_part(L.sv_b, 3 * D, 2 * D, D) : st;
        }
        if (t == "ca.in_proj_weight")
            return shape_ok(D, 3 * D) && rows(L.cq, 0, D) && rows(L.ckv, D, 2 * D) ? SAM3B200_STATUS_SUCCESS
                                                                                 : SAM3B200_STATUS_FAILED;
        if (t == "ca.in_proj_bias") {
            const int st = vec_part(L.cq_b, 3 * D, 0, D);
            return st == SAM3B200_STATUS_SUCCESS ? vec_part(L.ckv_b, 3 * D, D, 2 * D) : st;
        }
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
    set_error("fenc: unknown tensor %s", name_c);
    return SAM3B200_STATUS_FAILED;
}

int sam3b200_fenc_missing(sam3b200_fenc *hf, char *buf, int cap) {
    auto *f = reinterpret_cast<Fenc *>(hf);
    if (!f) return -1;
    check_ready(f);
    std::string all;
    for (const auto &s : f->missing) all += s + "\n";
    if (buf && cap > 0) snprintf(buf, static_cast<size_t>(cap), "%s", all.c_str());
    return static_cast<int>(f->missing.size());
}

int sam3b200_fenc_run_device(sam3b200_fenc *hf, const float *image_feats, const float *prompt, const float *pos,
                             const float *prompt_bias, int n_tokens, int n_prompt) {
    auto *f = reinterpret_cast<Fenc *>(hf);
    if (!f || !image_feats || !prompt || !pos) {
        set_error("fenc_run: null argument");
        return SAM3B200_STATUS_FAILED;
    }
    cudaSetDevice(f->be->device);
    if (!check_run(f, n_tokens, n_prompt)) return SAM3B200_STATUS_FAILED;
    return forward(f, image_feats, prompt, pos, prompt_bias, n_tokens, n_prompt) ? SAM3B200_STATUS_SUCCESS
                                                                                 : SAM3B200_STATUS_FAILED;
}

int sam3b200_fenc_run(sam3b200_fenc *hf, const float *image_feats, const float *prompt, const float *pos,
                      const float *prompt_bias, int n_tokens, int n_prompt) {
    auto *f = reinterpret_cast<Fenc *>(hf);
    if (!f || !image_feats || !prompt || !pos) {
        set_error("fenc_run: null argument");
        return SAM3B200_STATUS_FAILED;
    }
    cudaSetDevice(f->be->device);
    if (!check_run(f, n_tokens, n_prompt)) return SAM3B200_STATUS_FAILED;
    const size_t nd = static_cast<size_t>(n_tokens) * f->hp.d_model * 4;
    const size_t td = static_cast<size_t>(n_prompt) * f->hp.d_model * 4;
    cudaStream_t s = f->be->stream;
    if (!cuda_ok(cudaMemcpyAsync(f->in_img.p, image_feats, nd, cudaMemcpyHostToDevice, s), "fenc image") ||
        !cuda_ok(cudaMemcpyAsync(f->in_prompt.p, prompt, td, cudaMemcpyHostToDevice, s), "fenc prompt") ||
        !cuda_ok(cudaMemcpyAsync(f->in_pos.p, pos, nd, cudaMemcpyHostToDevice, s), "fenc pos") ||
        (prompt_bias && !cuda_ok(cudaMemcpyAsync(f->in_bias.p, prompt_bias, static_cast<size_t>(n_prompt) * 4,
                                                 cudaMemcpyHostToDevice, s),
                                 "fenc bias")))
        return SAM3B200_STATUS_FAILED;
    return forward(f, f->in_img.as<float>(), f->in_prompt.as<float>(), f->in_pos.as<float>(),
                   prompt_bias ? f->in_bias.as<float>() : nullptr, n_tokens, n_prompt)
               ? SAM3B200_STATUS_SUCCESS
               : SAM3B200_STATUS_FAILED;
}

int sam3b200_fenc_output(sam3b200_fenc *hf, const float **dev) {
    auto *f = reinterpret_cast<Fenc *>(hf);
    if (!f || !dev) return SAM3B200_STATUS_FAILED;
    *dev = f->x.as<float>();
    return SAM3B200_STATUS_SUCCESS;
}
