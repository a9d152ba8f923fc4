// text_enc.cu -- the SAM3 text encoder on the B200 backend: the graph
// sam3_build_text_encoder_graph builds (sam3.cpp:4039-4066; block
// sam3_text_block_forward :3958-4032, causal mask :3934-3951):
//
//   x = token_embed[ids] + pos_embed                          GET_ROWS + add
//   per block: x += out_proj(attn(LN1(x)))                     causal 16-head attention
//              x += fc2(GELU_erf(fc1(LN2(x))))
//   features = resizer(LN_final(x))                            [ctx_len][out_dim]
//
// The 32-token rows make every MUL_MAT a skinny one: run_mul_mat (the exact
// quantised MUL_MAT, its SIMT kernel below 64 rows; fp16 GEMM for F16/F32
// weights); the attention is attention_simt with the F16 causal mask.
#include "../../include/sam3_b200.h"
#include "attn_simt.cuh"
#include "model_util.h"
#include "row_norm.cuh"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

namespace b200 {
namespace {

// c = a + b elementwise
// (in place: c may alias a or b)
__global__ void text_add_kernel(const float *a, const float *b, int64_t n, float *c) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) c[i] = __fadd_rn(a[i], b[i]);
}

// ggml_gelu_erf (f32): 0.5 x (1 + erf(x / sqrt(2))), in place
__global__ void text_gelu_kernel(float *__restrict__ x, int64_t n) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float v = x[i];
    x[i] = __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, erff(__fmul_rn(v, 0.70710678118654752440f))));
}

struct TextBlock {
    DevBuf ln1w, ln1b, ln2w, ln2b, qkv_b, out_b, fc1_b, fc2_b;
    sam3b200_weight *qkv = nullptr, *out = nullptr, *fc1 = nullptr, *fc2 = nullptr;
};

inline unsigned tblocks(int64_t n) { return static_cast<unsigned>((n + 255) / 256); }

}  // namespace

struct TextEnc {
    Backend *be = nullptr;
    sam3b200_text_hparams hp{};
    std::vector<TextBlock> blk;
    DevBuf tok_emb, pos, lnf_w, lnf_b, res_b, mask, ids, x, xn, qkv, att, tmp, mlp, out;
    sam3b200_weight *res = nullptr;
    std::vector<std::string> missing;
};

namespace {

bool tok(TextEnc *t, cudaError_t e, const char *what) {
    t->be->count(1);
    return cuda_ok(e, what);
}

bool tlin(TextEnc *t, const sam3b200_weight *w, const float *x, int64_t ldx, const DevBuf &b, float *y, int64_t ldy) {
    return run_mul_mat(t->be, reinterpret_cast<const Weight *>(w), x, ldx, t->hp.ctx_len, b.as<float>(), y, ldy,
                       nullptr) == SAM3B200_STATUS_SUCCESS;
}

bool forward(TextEnc *t) {
    const int E = t->hp.width, L = t->hp.ctx_len, H = t->hp.heads, HD = E / H, F = 4 * E;
    cudaStream_t s = t->be->stream;
    auto *hb = reinterpret_cast<sam3b200_backend *>(t->be);
    float *x = t->x.as<float>(), *xn = t->xn.as<float>(), *tmp = t->tmp.as<float>();
    const int64_t n = static_cast<int64_t>(L) * E;
    if (sam3b200_get_rows(hb, SAM3B200_TYPE_F32, t->tok_emb.p, E, t->hp.vocab, t->ids.as<int32_t>(), L, x) !=
        SAM3B200_STATUS_SUCCESS)
        return false;
    text_add_kernel<<<tblocks(n), 256, 0, s>>>(x, t->pos.as<float>(), n, x);
    if (!tok(t, cudaGetLastError(), "text pos")) return false;
    const AttnStrides qs{0, HD, 3 * E}, os{0, HD, E};
    for (const TextBlock &b : t->blk) {
        ln_rows_kernel<<<tblocks(static_cast<int64_t>(L) * 32), 256, 0, s>>>(x, L, E, b.ln1w.as<float>(),
                                                                             b.ln1b.as<float>(), 1e-5f, xn);
        if (!tok(t, cudaGetLastError(), "text ln1") || !tlin(t, b.qkv, xn, E, b.qkv_b, t->qkv.as<float>(), 3 * E))
            return false;
        const float *q = t->qkv.as<float>();
        if (!tok(t,
                 attention_simt(HD, q, qs, L, q + E, qs, q + 2 * E, qs, L, 1, H, t->mask.as<__half>(), L,
                                1.0f / sqrtf(static_cast<float>(HD)), t->att.as<float>(), os, s),
                 "text attention") ||
            !tlin(t, b.out, t->att.as<float>(), E, b.out_b, tmp, E))
            return false;
        text_add_kernel<<<tblocks(n), 256, 0, s>>>(x, tmp, n, x);
        ln_rows_kernel<<<tblocks(static_cast<int64_t>(L) * 32), 256, 0, s>>>(x, L, E, b.ln2w.as<float>(),
                                                                             b.ln2b.as<float>(), 1e-5f, xn);
        if (!tok(t, cudaGetLastError(), "text ln2") || !tlin(t, b.fc1, xn, E, b.fc1_b, t->mlp.as<float>(), F))
            return false;
        text_gelu_kernel<<<tblocks(static_cast<int64_t>(L) * F), 256, 0, s>>>(t->mlp.as<float>(),
                                                                              static_cast<int64_t>(L) * F);
        if (!tok(t, cudaGetLastError(), "text gelu") || !tlin(t, b.fc2, t->mlp.as<float>(), F, b.fc2_b, tmp, E))
            return false;
        text_add_kernel<<<tblocks(n), 256, 0, s>>>(x, tmp, n, x);
        if (!tok(t, cudaGetLastError(), "text residual")) return false;
    }
    ln_rows_kernel<<<tblocks(static_cast<int64_t>(L) * 32), 256, 0, s>>>(x, L, E, t->lnf_w.as<float>(),
                                                                         t->lnf_b.as<float>(), 1e-5f, xn);
    return tok(t, cudaGetLastError(), "text ln_final") && tlin(t, t->res, xn, E, t->res_b, t->out.as<float>(),
                                                               t->hp.out_dim);
}

bool check_ready(TextEnc *t) {
    t->missing.clear();
    auto need = [&](bool ok, const std::string &n) {
        if (!ok) t->missing.push_back(n);
    };
    need(t->tok_emb.p && t->pos.p, "text.token_embed.weight / text.pos_embed");
    need(t->lnf_w.p && t->lnf_b.p && t->res && t->res_b.p, "text.ln_final / text.resizer");
    for (size_t i = 0; i < t->blk.size(); ++i) {
        const TextBlock &b = t->blk[i];
        need(b.qkv && b.out && b.fc1 && b.fc2 && b.qkv_b.p && b.out_b.p && b.fc1_b.p && b.fc2_b.p && b.ln1w.p &&
                 b.ln1b.p && b.ln2w.p && b.ln2b.p,
             "text.blocks." + std::to_string(i));
    }
    if (!t->missing.empty()) {
        set_error("text: %zu tensors missing (first: %s)", t->missing.size(), t->missing[0].c_str());
        return false;
    }
    return true;
}

void tfree(TextEnc *t, sam3b200_weight *&w) {
    if (w) sam3b200_weight_free(reinterpret_cast<sam3b200_backend *>(t->be), w);
    w = nullptr;
}

}  // namespace
}  // namespace b200

using namespace b200;

sam3b200_text *sam3b200_text_create(sam3b200_backend *hb, const sam3b200_text_hparams *hp) {
    auto *be = reinterpret_cast<Backend *>(hb);
    if (!be || !hp) return nullptr;
    if (hp->width <= 0 || hp->width % 32 != 0 || hp->heads <= 0 || hp->width % hp->heads != 0 ||
        hp->width / hp->heads != 64 || hp->layers <= 0 || hp->ctx_len <= 0 || hp->ctx_len > 1024 ||
        hp->vocab <= 0 || hp->out_dim <= 0) {
        set_error("text_create: unsupported hyperparameters (head dim 64, width a multiple of 32)");
        return nullptr;
    }
    cudaSetDevice(be->device);
    auto *t = new TextEnc();
    t->be = be;
    t->hp = *hp;
    t->blk.resize(hp->layers);
    const size_t L = hp->ctx_len, E = hp->width;
    // causal mask [q][kv]: 0 where kv <= q, -inf above (sam3_fill_causal_mask)
    std::vector<__half> m(L * L);
    for (size_t q = 0; q < L; ++q)
        for (size_t k = 0; k < L; ++k) m[q * L + k] = __float2half_rn(k <= q ? 0.0f : -INFINITY);
    const bool ok = upload(t->mask, m.data(), m.size() * 2, be->stream) && t->ids.alloc(L * 4) &&
                    t->x.alloc(L * E * 4) && t->xn.alloc(L * E * 4) && t->qkv.alloc(3 * L * E * 4) &&
                    t->att.alloc(L * E * 4) && t->tmp.alloc(L * E * 4) && t->mlp.alloc(4 * L * E * 4) &&
                    t->out.alloc(L * hp->out_dim * 4);
    if (!ok) {
        delete t;
        return nullptr;
    }
    return reinterpret_cast<sam3b200_text *>(t);
}

void sam3b200_text_free(sam3b200_text *ht) {
    auto *t = reinterpret_cast<TextEnc *>(ht);
    if (!t) return;
    cudaSetDevice(t->be->device);
    cudaStreamSynchronize(t->be->stream);
    for (auto &b : t->blk) {
        tfree(t, b.qkv);
        tfree(t, b.out);
        tfree(t, b.fc1);
        tfree(t, b.fc2);
    }
    tfree(t, t->res);
    delete t;
}

int sam3b200_text_set_tensor(sam3b200_text *ht, const char *name_c, int type, const void *data, const int64_t *ne) {
    auto *t = reinterpret_cast<TextEnc *>(ht);
    if (!t || !name_c || !data || !ne) return SAM3B200_STATUS_FAILED;
    cudaSetDevice(t->be->device);
    auto *hb = reinterpret_cast<sam3b200_backend *>(t->be);
    const std::string name(name_c);
    const int64_t E = t->hp.width, n = ne[0] * (ne[1] > 0 ? ne[1] : 1) * (ne[2] > 0 ? ne[2] : 1) * (ne[3] > 0 ? ne[3] : 1);
    std::vector<float> f;
    auto vec = [&](DevBuf &d, int64_t want) -> int {
        if (n != want || !to_f32(type, data, n, f)) {
            set_error("%s: %lld elements of type %d, expected %lld F32/F16", name_c, (long long)n, type,
                      (long long)want);
            return SAM3B200_STATUS_FAILED;
        }
        return upload(d, f.data(), f.size() * 4, t->be->stream) ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
    };
    auto weight = [&](sam3b200_weight *&w, int64_t K, int64_t N) -> int {
        if (ne[0] != K || ne[1] != N) {
            set_error("%s: shape [%lld, %lld], expected [%lld, %lld]", name_c, (long long)ne[0], (long long)ne[1],
                      (long long)K, (long long)N);
            return SAM3B200_STATUS_FAILED;
        }
        tfree(t, w);
        w = sam3b200_weight_upload(hb, type, data, K, N);
        return w ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
    };
    if (name == "text.token_embed.weight") return vec(t->tok_emb, E * t->hp.vocab);
    if (name == "text.pos_embed") return vec(t->pos, E * t->hp.ctx_len);
    if (name == "text.ln_final.weight") return vec(t->lnf_w, E);
    if (name == "text.ln_final.bias") return vec(t->lnf_b, E);
    if (name == "text.resizer.weight") return weight(t->res, E, t->hp.out_dim);
    if (name == "text.resizer.bias") return vec(t->res_b, t->hp.out_dim);
    if (name.rfind("text.blocks.", 0) == 0) {
        const int i = atoi(name.c_str() + 12);
        if (i >= 0 && i < static_cast<int>(t->blk.size())) {
            TextBlock &b = t->blk[i];
            const std::string r = name.substr(name.find('.', 12) + 1);
            if (r == "attn.in_proj.weight") return weight(b.qkv, E, 3 * E);
            if (r == "attn.in_proj.bias") return vec(b.qkv_b, 3 * E);
            if (r == "attn.out_proj.weight") return weight(b.out, E, E);
            if (r == "attn.out_proj.bias") return vec(b.out_b, E);
            if (r == "ln_1.weight") return vec(b.ln1w, E);
            if (r == "ln_1.bias") return vec(b.ln1b, E);
            if (r == "ln_2.weight") return vec(b.ln2w, E);
            if (r == "ln_2.bias") return vec(b.ln2b, E);
            if (r == "mlp.fc1.weight") return weight(b.fc1, E, 4 * E);
            if (r == "mlp.fc1.bias") return vec(b.fc1_b, 4 * E);
            if (r == "mlp.fc2.weight") return weight(b.fc2, 4 * E, E);
            if (r == "mlp.fc2.bias") return vec(b.fc2_b, E);
        }
    }
    set_error("text: unknown tensor %s", name_c);
    return SAM3B200_STATUS_FAILED;
}

int sam3b200_text_missing(sam3b200_text *ht, char *buf, int cap) {
    auto *t = reinterpret_cast<TextEnc *>(ht);
    if (!t) return -1;
    check_ready(t);
    std::string all;
    for (const auto &m : t->missing) all += m + "\n";
    if (buf && cap > 0) snprintf(buf, static_cast<size_t>(cap), "%s", all.c_str());
    return static_cast<int>(t->missing.size());
}

int sam3b200_text_encode(sam3b200_text *ht, const int32_t *ids, int n_ids) {
    auto *t = reinterpret_cast<TextEnc *>(ht);
    if (!t || !ids || n_ids <= 0 || n_ids > t->hp.ctx_len) {
        set_error("text_encode: 1..ctx_len token ids expected");
        return SAM3B200_STATUS_FAILED;
    }
    for (int i = 0; i < n_ids; ++i)
        if (ids[i] < 0 || ids[i] >= t->hp.vocab) {
            set_error("text_encode: token id %d outside the vocabulary", ids[i]);
            return SAM3B200_STATUS_FAILED;
        }
    cudaSetDevice(t->be->device);
    if (!check_ready(t)) return SAM3B200_STATUS_FAILED;
    std::vector<int32_t> padded(t->hp.ctx_len, 0);  // padded with id 0 to the context length
    std::copy(ids, ids + n_ids, padded.begin());
    if (!cuda_ok(cudaMemcpyAsync(t->ids.p, padded.data(), padded.size() * 4, cudaMemcpyHostToDevice, t->be->stream),
                 "text ids") ||
        !cuda_ok(cudaStreamSynchronize(t->be->stream), "text ids sync"))
        return SAM3B200_STATUS_FAILED;
    return forward(t) ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
}

int sam3b200_text_output(sam3b200_text *ht, const float **dev, int64_t *ne) {
    auto *t = reinterpret_cast<TextEnc *>(ht);
    if (!t || !dev || !ne) return SAM3B200_STATUS_FAILED;
    *dev = t->out.as<float>();
    ne[0] = t->hp.out_dim;
    ne[1] = t->hp.ctx_len;
    return SAM3B200_STATUS_SUCCESS;
}
