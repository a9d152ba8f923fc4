// mem_attn.cu -- the memory attention of the video tracker on the B200
// backend: the graph sam3_build_mem_attn_graph builds (sam3.cpp:9228-9341),
// fed as sam3_propagate_single feeds it (:11175-11310):
//
//   x = curr + 0.1 * src_pos                                  pos_enc_at_input
//   per layer: x += sa_out(attn(rope(q(LN1 x)), rope(k(LN1 x)), v(LN1 x)))
//              x += ca_out(attn(rope(q(LN2 x)), rope_spatial(k(prompt + prompt_pos)), v(prompt)))
//              x += fc2(relu(fc1(LN3 x)))
//   out = LN(x)                                               mem_attn.norm
//
// Single-head attention over the d_model (256) channels; the cross-attention
// keys and values are projected up from mem_dim (64) channels, and only the
// first M_total - n_obj_ptr_tokens keys (the spatial memories) are rotated.
// Linear layers are run_mul_mat (the exact quantised MUL_MAT; fp16 GEMM for
// F16/F32 weights); attention runs on the tensor cores (attn_mma.cu: head dim
// 256, fp16 k and v, the keys split across CTAs).
#include "../../include/sam3_b200.h"
#include "attn_mma.cuh"
#include "attn_tc256.cuh"
#include "model_util.h"
#include "eltwise.cuh"
#include "row_norm.cuh"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <algorithm>
#include <vector>

namespace b200 {
namespace {

inline unsigned mblocks(int64_t n) { return static_cast<unsigned>((n + 255) / 256); }

// c = a + b (c may alias a or b)
__global__ void ma_add_kernel(const float *a, const float *b, int64_t n, float *c) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) c[i] = __fadd_rn(a[i], b[i]);
}

// c = a + (b * s), the product rounded first (ggml_scale then ggml_add)
__global__ void ma_add_scaled_kernel(const float *__restrict__ a, const float *__restrict__ b, float s, int64_t n,
                                     float *__restrict__ c) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) c[i] = __fadd_rn(a[i], __fmul_rn(b[i], s));
}

__global__ void ma_relu_kernel(float *x, int64_t n) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) x[i] = fmaxf(x[i], 0.0f);
}

// sam3_apply_rope (sam3.cpp:3671-3710) on rows of 2*half channels: the pair
// (x[2j], x[2j+1]) times (cos, sin) = table[row][j][0..1]; every product is
// rounded before the sum, as the ggml mul/sub/add nodes round them.
__global__ void ma_rope_kernel(float *x, const float *__restrict__ cs, int64_t rows, int half) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= rows * half) return;
    float2 *p = reinterpret_cast<float2 *>(x) + i;
    const float2 t = reinterpret_cast<const float2 *>(cs)[i];
    const float2 v = *p;
    float2 r;
    r.x = __fsub_rn(__fmul_rn(v.x, t.x), __fmul_rn(v.y, t.y));
    r.y = __fadd_rn(__fmul_rn(v.x, t.y), __fmul_rn(v.y, t.x));
    *p = r;
}

struct MemLayer {
    DevBuf n1w, n1b, n2w, n2b, n3w, n3b;
    DevBuf sqb, skb, svb, sob, cqb, ckb, cvb, cob, f1b, f2b;
    sam3b200_weight *sq = nullptr, *sk = nullptr, *sv = nullptr, *so = nullptr;
    sam3b200_weight *cq = nullptr, *ck = nullptr, *cv = nullptr, *co = nullptr;
    sam3b200_weight *f1 = nullptr, *f2 = nullptr;
};

}  // namespace

struct MemAttn {
    Backend *be = nullptr;
    sam3b200_mem_attn_hparams hp{};
    std::vector<MemLayer> ly;
    DevBuf normw, normb;
    // activations
    DevBuf x, xn, q, k, v, att, tmp, ffn, kvpos, out;
    // attention operands in fp16 and the split-KV partial results
    DevBuf k16, v16, q16, part_o, part_ml;
    int splits = 1;
    bool tc = true;  // d_model 256: tcgen05 flash attention (env SAM3B200_MEM_ATTN_TC=0: the mma.sync kernel)
    // host-run staging of the inputs
    DevBuf in_curr, in_spos, in_prompt, in_ppos, in_rq, in_rk;
    std::vector<std::string> missing;
};

namespace {

bool mok(MemAttn *m, cudaError_t e, const char *what, int n = 1) {
    m->be->count(n);
    return cuda_ok(e, what);
}

bool mlin(MemAttn *m, const sam3b200_weight *w, const float *x, int64_t ldx, int64_t rows, const DevBuf &b, float *y,
          int64_t ldy) {
    return run_mul_mat(m->be, reinterpret_cast<const Weight *>(w), x, ldx, rows, b.as<float>(), y, ldy, nullptr) ==
           SAM3B200_STATUS_SUCCESS;
}

bool mln(MemAttn *m, const float *x, int rows, const DevBuf &w, const DevBuf &b, float *y) {
    ln_rows_kernel<<<mblocks(static_cast<int64_t>(rows) * 32), 256, 0, m->be->stream>>>(
        x, rows, m->hp.d_model, w.as<float>(), b.as<float>(), 1e-5f, y);
    return mok(m, cudaGetLastError(), "mem_attn layer norm");
}

bool madd(MemAttn *m, float *x, const float *y, int64_t n) {
    ma_add_kernel<<<mblocks(n), 256, 0, m->be->stream>>>(x, y, n, x);
    return mok(m, cudaGetLastError(), "mem_attn residual");
}

bool mrope(MemAttn *m, float *x, const float *table, int64_t rows) {
    if (rows <= 0) return true;
    const int half = m->hp.d_model / 2;
    ma_rope_kernel<<<mblocks(rows * half), 256, 0, m->be->stream>>>(x, table, rows, half);
    return mok(m, cudaGetLastError(), "mem_attn rope");
}

// single-head attention of N queries over NK keys on the tensor cores: k, v
// rounded to fp16 once, the keys split across CTAs so 4096 queries fill the GPU
bool attend(MemAttn *m, const float *q, const float *k, const float *v, int N, int NK, float scale, float *out) {
    const int D = m->hp.d_model;
    const int64_t n = static_cast<int64_t>(NK) * D;
    cudaStream_t s = m->be->stream;
    if (D == 256 && m->tc) {
        // tcgen05 flash attention: q, k fp16 row-major, v transposed to fp16 [256][keys]
        const int ldt = (NK + 63) / 64 * 64;
        const int64_t nq = static_cast<int64_t>(N) * D;
        ew_to_half_kernel<<<ew_blocks(nq), 256, 0, s>>>(q, nq, m->q16.as<__half>());
        ew_to_half_kernel<<<ew_blocks(n), 256, 0, s>>>(k, n, m->k16.as<__half>());
        if (!mok(m, cudaGetLastError(), "mem_attn fp16 q, k", 2) ||
            !mok(m, v_to_half_transposed(v, NK, D, m->v16.as<__half>(), ldt, s), "mem_attn fp16 v^T"))
            return false;
        // no more key ranges than part_o / part_ml hold rows of N queries for
        const int room = static_cast<int>(std::min(m->part_o.n / (static_cast<size_t>(N) * D * 4),
                                                   m->part_ml.n / (static_cast<size_t>(N) * 8)));
        const int splits = std::max(1, std::min(attention_tc256_splits(N, NK, m->be->num_sms), room));
        m->be->prof_mark(1);  // profile class 1: the memory attention's attention kernels
        const bool ok = mok(m, attention_tc256(m->q16.as<__half>(), N, m->k16.as<__half>(), NK, m->v16.as<__half>(), ldt,
                                               scale, splits, m->part_o.as<float>(), m->part_ml.as<float2>(), out,
                                               m->be->err, s),
                            "mem_attn attention", 2);
        m->be->prof_mark(1);
        return ok;
    }
    ew_to_half_kernel<<<ew_blocks(n), 256, 0, s>>>(k, n, m->k16.as<__half>());
    ew_to_half_kernel<<<ew_blocks(n), 256, 0, s>>>(v, n, m->v16.as<__half>());
    const AttnStrides rs{0, 0, D};
    if (!mok(m, cudaGetLastError(), "mem_attn fp16 k, v")) return false;
    m->be->prof_mark(1);  // profile class 1: the memory attention's attention kernels
    const bool ok = mok(m, attention_mma_f16kv_split(D, q, rs, N, m->k16.as<__half>(), rs, m->v16.as<__half>(), rs, NK,
                                                     1, 1, scale, out, rs, m->splits, m->part_o.as<float>(),
                                                     m->part_ml.as<float2>(), s),
                        "mem_attn attention");
    m->be->prof_mark(1);
    return ok;
}

bool forward(MemAttn *m, const float *curr, const float *spos, const float *prompt, const float *ppos,
             const float *rope_q, const float *rope_k, int N, int M, int n_ptr) {
    const int D = m->hp.d_model, MD = m->hp.mem_dim, F = m->hp.ffn_dim;
    const int64_t nd = static_cast<int64_t>(N) * D;
    const int Ms = M - n_ptr;
    cudaStream_t s = m->be->stream;
    float *x = m->x.as<float>(), *xn = m->xn.as<float>(), *q = m->q.as<float>(), *k = m->k.as<float>();
    float *v = m->v.as<float>(), *att = m->att.as<float>(), *tmp = m->tmp.as<float>(), *kvpos = m->kvpos.as<float>();
    const float scale = 1.0f / sqrtf(static_cast<float>(D));
    ma_add_scaled_kernel<<<mblocks(nd), 256, 0, s>>>(curr, spos, 0.1f, nd, x);
    if (!mok(m, cudaGetLastError(), "mem_attn input")) return false;
    // the keys' positional sum prompt + prompt_pos is the same for every layer
    ma_add_kernel<<<mblocks(static_cast<int64_t>(M) * MD), 256, 0, s>>>(prompt, ppos, static_cast<int64_t>(M) * MD,
                                                                        kvpos);
    if (!mok(m, cudaGetLastError(), "mem_attn prompt + pos")) return false;
    for (const MemLayer &L : m->ly) {
        // self-attention with RoPE on q and k
        if (!mln(m, x, N, L.n1w, L.n1b, xn) || !mlin(m, L.sq, xn, D, N, L.sqb, q, D) ||
            !mlin(m, L.sk, xn, D, N, L.skb, k, D) || !mlin(m, L.sv, xn, D, N, L.svb, v, D) ||
            !mrope(m, q, rope_q, N) || !mrope(m, k, rope_q, N) ||
            !attend(m, q, k, v, N, N, scale, att) ||
            !mlin(m, L.so, att, D, N, L.sob, tmp, D) || !madd(m, x, tmp, nd))
            return false;
        // cross-attention to the memories: k from prompt + pos, v from prompt
        if (!mln(m, x, N, L.n2w, L.n2b, xn) || !mlin(m, L.cq, xn, D, N, L.cqb, q, D) ||
            !mlin(m, L.ck, kvpos, MD, M, L.ckb, k, D) || !mlin(m, L.cv, prompt, MD, M, L.cvb, v, D) ||
            !mrope(m, q, rope_q, N) || (rope_k && !mrope(m, k, rope_k, Ms)) ||
            !attend(m, q, k, v, N, M, scale, att) ||
            !mlin(m, L.co, att, D, N, L.cob, tmp, D) || !madd(m, x, tmp, nd))
            return false;
        // feed-forward
        if (!mln(m, x, N, L.n3w, L.n3b, xn) || !mlin(m, L.f1, xn, D, N, L.f1b, m->ffn.as<float>(), F))
            return false;
        ma_relu_kernel<<<mblocks(static_cast<int64_t>(N) * F), 256, 0, s>>>(m->ffn.as<float>(),
                                                                            static_cast<int64_t>(N) * F);
        if (!mok(m, cudaGetLastError(), "mem_attn relu") || !mlin(m, L.f2, m->ffn.as<float>(), F, N, L.f2b, tmp, D) ||
            !madd(m, x, tmp, nd))
            return false;
    }
    return mln(m, x, N, m->normw, m->normb, m->out.as<float>());
}

bool check_ready(MemAttn *m) {
    m->missing.clear();
    if (!m->normw.p || !m->normb.p) m->missing.push_back("mem_attn.norm");
    for (size_t i = 0; i < m->ly.size(); ++i) {
        const MemLayer &L = m->ly[i];
        const bool ok = L.sq && L.sk && L.sv && L.so && L.cq && L.ck && L.cv && L.co && L.f1 && L.f2 && L.sqb.p &&
                        L.skb.p && L.svb.p && L.sob.p && L.cqb.p && L.ckb.p && L.cvb.p && L.cob.p && L.f1b.p &&
                        L.f2b.p && L.n1w.p && L.n1b.p && L.n2w.p && L.n2b.p && L.n3w.p && L.n3b.p;
        if (!ok) m->missing.push_back("mem_attn.layers." + std::to_string(i));
    }
    if (!m->missing.empty()) {
        set_error("mem_attn: %zu tensors missing (first: %s)", m->missing.size(), m->missing[0].c_str());
        return false;
    }
    return true;
}

void mfree(MemAttn *m, sam3b200_weight *&w) {
    if (w) sam3b200_weight_free(reinterpret_cast<sam3b200_backend *>(m->be), w);
    w = nullptr;
}

bool check_run(MemAttn *m, int N, int M, int n_ptr) {
    if (N <= 0 || N > m->hp.max_tokens || M <= 0 || M > m->hp.max_mem_tokens || n_ptr < 0 || n_ptr > M) {
        set_error("mem_attn_run: N=%d (max %d), M_total=%d (max %d), obj-ptr tokens %d out of range", N,
                  m->hp.max_tokens, M, m->hp.max_mem_tokens, n_ptr);
        return false;
    }
    return check_ready(m);
}

}  // namespace
}  // namespace b200

using namespace b200;

sam3b200_mem_attn *sam3b200_mem_attn_create(sam3b200_backend *hb, const sam3b200_mem_attn_hparams *hp) {
    auto *be = reinterpret_cast<Backend *>(hb);
    if (!be || !hp) return nullptr;
    const int D = hp->d_model;
    if ((D != 64 && D != 128 && D != 256) || hp->mem_dim <= 0 || hp->mem_dim % 32 != 0 ||
        hp->layers <= 0 || hp->ffn_dim <= 0 || hp->ffn_dim % 32 != 0 || hp->max_tokens <= 0 ||
        hp->max_mem_tokens <= 0) {
        set_error("mem_attn_create: unsupported hyperparameters (d_model in {64,128,256}, mem_dim and "
                  "ffn_dim multiples of 32)");
        return nullptr;
    }
    cudaSetDevice(be->device);
    auto *m = new MemAttn();
    m->be = be;
    m->hp = *hp;
    m->ly.resize(hp->layers);
    const size_t N = hp->max_tokens, M = hp->max_mem_tokens, NM = N > M ? N : M;
    const size_t d = D, md = hp->mem_dim;
    // split-KV: about two CTAs per SM for the 64-query tiles of max_tokens
    const int qtiles = static_cast<int>((N + 63) / 64);
    m->splits = std::min(8, std::max(1, (2 * be->num_sms + qtiles - 1) / qtiles));
    const char *tc_env = std::getenv("SAM3B200_MEM_ATTN_TC");
    m->tc = D == 256 && !(tc_env && tc_env[0] == '0');
    // the tcgen05 path splits keys into up to num_sms / (query tiles of 128) ranges
    const int tc_splits = std::max(1, be->num_sms / static_cast<int>((N + 127) / 128));
    const size_t sp = static_cast<size_t>(std::max(m->splits, m->tc ? tc_splits : 1));
    const size_t NMp = (NM + 63) / 64 * 64;  // v^T rows padded to whole 64-key tiles
    const bool ok = m->k16.alloc(NM * d * 2) && m->v16.alloc(NMp * d * 2) && m->q16.alloc(N * d * 2) &&
                    m->part_o.alloc(sp * N * d * 4) &&
                    m->part_ml.alloc(sp * N * 8) && m->x.alloc(N * d * 4) && m->xn.alloc(N * d * 4) &&
                    m->q.alloc(N * d * 4) &&
                    m->k.alloc(NM * d * 4) && m->v.alloc(NM * d * 4) && m->att.alloc(N * d * 4) &&
                    m->tmp.alloc(N * d * 4) && m->ffn.alloc(N * hp->ffn_dim * 4) && m->kvpos.alloc(M * md * 4) &&
                    m->out.alloc(N * d * 4);
    if (!ok) {
        delete m;
        return nullptr;
    }
    return reinterpret_cast<sam3b200_mem_attn *>(m);
}

void sam3b200_mem_attn_free(sam3b200_mem_attn *hm) {
    auto *m = reinterpret_cast<MemAttn *>(hm);
    if (!m) return;
    cudaSetDevice(m->be->device);
    cudaStreamSynchronize(m->be->stream);
    for (auto &L : m->ly)
        for (sam3b200_weight **w : {&L.sq, &L.sk, &L.sv, &L.so, &L.cq, &L.ck, &L.cv, &L.co, &L.f1, &L.f2}) mfree(m, *w);
    delete m;
}

int sam3b200_mem_attn_set_tensor(sam3b200_mem_attn *hm, const char *name_c, int type, const void *data,
                                 const int64_t *ne) {
    auto *m = reinterpret_cast<MemAttn *>(hm);
    if (!m || !name_c || !data || !ne) return SAM3B200_STATUS_FAILED;
    cudaSetDevice(m->be->device);
    auto *hb = reinterpret_cast<sam3b200_backend *>(m->be);
    const std::string name(name_c);
    const int64_t D = m->hp.d_model, MD = m->hp.mem_dim, F = m->hp.ffn_dim;
    const int64_t n = ne[0] * (ne[1] > 0 ? ne[1] : 1) * (ne[2] > 0 ? ne[2] : 1) * (ne[3] > 0 ? ne[3] : 1);
    std::vector<float> f;
    auto vec = [&](DevBuf &d, int64_t want) -> int {
        if (n != want || !to_f32(type, data, n, f)) {
            set_error("%s: %lld elements of type %d, expected %lld F32/F16", name_c, (long long)n, type,
                      (long long)want);
            return SAM3B200_STATUS_FAILED;
        }
        return upload(d, f.data(), f.size() * 4, m->be->stream) ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
    };
    auto weight = [&](sam3b200_weight *&w, int64_t K, int64_t N) -> int {
        if (ne[0] != K || ne[1] != N) {
            set_error("%s: shape [%lld, %lld], expected [%lld, %lld]", name_c, (long long)ne[0], (long long)ne[1],
                      (long long)K, (long long)N);
            return SAM3B200_STATUS_FAILED;
        }
        mfree(m, w);
        w = sam3b200_weight_upload(hb, type, data, K, N);
        return w ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
    };
    if (name == "mem_attn.norm.weight") return vec(m->normw, D);
    if (name == "mem_attn.norm.bias") return vec(m->normb, D);
    int li = -1;
    char tail[96] = {0};
    if (sscanf(name_c, "mem_attn.layers.%d.%95s", &li, tail) == 2 && li >= 0 && li < static_cast<int>(m->ly.size())) {
        MemLayer &L = m->ly[li];
        const std::string t(tail);
        struct Proj {
            const char *pfx;
            sam3b200_weight **w;
            DevBuf *b;
            int64_t K, N;
        };
        const Proj projs[] = {
            {"sa.q_proj.", &L.sq, &L.sqb, D, D},   {"sa.k_proj.", &L.sk, &L.skb, D, D},
            {"sa.v_proj.", &L.sv, &L.svb, D, D},   {"sa.out_proj.", &L.so, &L.sob, D, D},
            {"ca.q_proj.", &L.cq, &L.cqb, D, D},   {"ca.k_proj.", &L.ck, &L.ckb, MD, D},
            {"ca.v_proj.", &L.cv, &L.cvb, MD, D},  {"ca.out_proj.", &L.co, &L.cob, D, D},
            {"linear1.", &L.f1, &L.f1b, D, F},     {"linear2.", &L.f2, &L.f2b, F, D},
        };
        for (const Proj &p : projs) {
            const std::string pf(p.pfx);
            if (t == pf + "weight") return weight(*p.w, p.K, p.N);
            if (t == pf + "bias") return vec(*p.b, p.N);
        }
        if (t == "norm1.weight") return vec(L.n1w, D);
        if (t == "norm1.bias") return vec(L.n1b, D);
        if (t == "norm2.weight") return vec(L.n2w, D);
        if (t == "norm2.bias") return vec(L.n2b, D);
        if (t == "norm3.weight") return vec(L.n3w, D);
        if (t == "norm3.bias") return vec(L.n3b, D);
    }
    set_error("mem_attn: unknown tensor %s", name_c);
    return SAM3B200_STATUS_FAILED;
}

int sam3b200_mem_attn_missing(sam3b200_mem_attn *hm, char *buf, int cap) {
    auto *m = reinterpret_cast<MemAttn *>(hm);
    if (!m) return -1;
    check_ready(m);
    std::string all;
    for (const auto &s : m->missing) all += s + "\n";
    if (buf && cap > 0) snprintf(buf, static_cast<size_t>(cap), "%s", all.c_str());
    return static_cast<int>(m->missing.size());
}

int sam3b200_mem_attn_run_device(sam3b200_mem_attn *hm, const float *curr, const float *src_pos,
                                 const float *prompt, const float *prompt_pos, const float *rope_q,
                                 const float *rope_k, int n_tokens, int n_mem_tokens, int n_obj_ptr_tokens) {
    auto *m = reinterpret_cast<MemAttn *>(hm);
    if (!m || !curr || !src_pos || !prompt || !prompt_pos || !rope_q) {
        set_error("mem_attn_run: null argument");
        return SAM3B200_STATUS_FAILED;
    }
    cudaSetDevice(m->be->device);
    if (!check_run(m, n_tokens, n_mem_tokens, n_obj_ptr_tokens)) return SAM3B200_STATUS_FAILED;
    return forward(m, curr, src_pos, prompt, prompt_pos, rope_q, rope_k, n_tokens, n_mem_tokens, n_obj_ptr_tokens)
               ? SAM3B200_STATUS_SUCCESS
               : SAM3B200_STATUS_FAILED;
}

int sam3b200_mem_attn_run(sam3b200_mem_attn *hm, const float *curr, const float *src_pos, const float *prompt,
                          const float *prompt_pos, const float *rope_q, const float *rope_k, int n_tokens,
                          int n_mem_tokens, int n_obj_ptr_tokens) {
    auto *m = reinterpret_cast<MemAttn *>(hm);
    if (!m || !curr || !src_pos || !prompt || !prompt_pos || !rope_q) {
        set_error("mem_attn_run: null argument");
        return SAM3B200_STATUS_FAILED;
    }
    cudaSetDevice(m->be->device);
    if (!check_run(m, n_tokens, n_mem_tokens, n_obj_ptr_tokens)) return SAM3B200_STATUS_FAILED;
    const size_t nd = static_cast<size_t>(n_tokens) * m->hp.d_model * 4;
    const size_t mm = static_cast<size_t>(n_mem_tokens) * m->hp.mem_dim * 4;
    const size_t mk = static_cast<size_t>(n_mem_tokens - n_obj_ptr_tokens) * m->hp.d_model * 4;
    const bool with_k = rope_k && mk > 0;
    // the staging buffers keep their size across calls; a larger call grows them
    auto stage = [&](DevBuf &d, const void *h, size_t bytes) {
        return (d.n >= bytes || d.alloc(bytes)) &&
               cuda_ok(cudaMemcpyAsync(d.p, h, bytes, cudaMemcpyHostToDevice, m->be->stream), "mem_attn input");
    };
    if (!stage(m->in_curr, curr, nd) || !stage(m->in_spos, src_pos, nd) || !stage(m->in_prompt, prompt, mm) ||
        !stage(m->in_ppos, prompt_pos, mm) || !stage(m->in_rq, rope_q, nd) ||
        (with_k && !stage(m->in_rk, rope_k, mk)))
        return SAM3B200_STATUS_FAILED;
    return forward(m, m->in_curr.as<float>(), m->in_spos.as<float>(), m->in_prompt.as<float>(),
                   m->in_ppos.as<float>(), m->in_rq.as<float>(), with_k ? m->in_rk.as<float>() : nullptr, n_tokens,
                   n_mem_tokens, n_obj_ptr_tokens)
               ? SAM3B200_STATUS_SUCCESS
               : SAM3B200_STATUS_FAILED;
}

int sam3b200_mem_attn_output(sam3b200_mem_attn *hm, const float **dev) {
    auto *m = reinterpret_cast<MemAttn *>(hm);
    if (!m || !dev) return SAM3B200_STATUS_FAILED;
    *dev = m->out.as<float>();
    return SAM3B200_STATUS_SUCCESS;
}
