// seghead.cu -- the segmentation head of the SAM3 detector on the B200
// backend: the graph sam3_build_seg_head_graph builds (sam3.cpp:8975-9058)
// with its pixel decoder (sam3_pixel_decoder, :8899-8960):
//
//   enc = enc + MHA(LN(enc), prompt; padding bias)            cross_attend_prompt
//   p0  = relu(GN(conv3x3(fpn1 + up2(enc))))                  144 x 144 (2 * feat)
//   p1  = relu(GN(conv3x3(fpn0 + up2(p0))))                   288 x 288 (4 * feat)
//   emb = conv1x1(p1)                                         instance_seg_head
//   masks[q][pixel] = mask_embed(queries[q]) . emb[pixel]     mask_predictor
//
// Maps are token-major [H][W][C].  The 3x3 convolutions run as im2col + the
// fp16 tensor-core GEMM (fp16 input and kernel, fp32 accumulation): ggml's
// own arithmetic for F16 kernels (its im2col of an F16 kernel is F16), within
// the 1e-2 bound for the F32 kernels of quantised files, as the tracker neck's
// convolutions.  GroupNorm(8) follows ggml's
// group_norm (double sums, then scale, weight, bias); the 1x1 convolution and
// the mask product are f32 tiled GEMMs.
#include "../../include/sam3_b200.h"
#include "attn_mma.cuh"
#include "eltwise.cuh"
#include "gemm_f16.cuh"
#include "model_util.h"
#include "row_norm.cuh"
#include "vit_ops.cuh"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

namespace b200 {
namespace {

constexpr int kGroups = 8;

// merged[(y, x)][c] = fpn[(y, x)][c] + prev[(y / 2, x / 2)][c] (nearest 2x upsample)
__global__ void sh_up_add_kernel(const float *__restrict__ fpn, const float *__restrict__ prev, int S, int C,
                                 float *__restrict__ out) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t n = static_cast<int64_t>(S) * S * C;
    if (i >= n) return;
    const int c = static_cast<int>(i % C);
    const int64_t p = i / C;
    const int y = static_cast<int>(p / S), x = static_cast<int>(p % S);
    const int64_t q = static_cast<int64_t>(y / 2) * (S / 2) + x / 2;
    out[i] = __fadd_rn(fpn[i], prev[q * C + c]);
}

// f32 C[m][n] = sum_k A[m][k] B[n][k] (+ bias[n]); A, B row-major with K
// contiguous; 64 x 64 tiles, 256 threads of 4 x 4 outputs, K staged 16 at a time.
__global__ void __launch_bounds__(256) sh_gemm_nt_kernel(const float *__restrict__ A, const float *__restrict__ B,
                                                         int64_t M, int64_t N, int K, const float *__restrict__ bias,
                                                         float *__restrict__ Cm, int64_t ldc) {
    __shared__ float as[16][64 + 4], bs[16][64 + 4];
    const int64_t m0 = static_cast<int64_t>(blockIdx.y) * 64, n0 = static_cast<int64_t>(blockIdx.x) * 64;
    const int tm = threadIdx.x / 16, tn = threadIdx.x % 16;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += 16) {
        __syncthreads();
        for (int e = threadIdx.x; e < 16 * 64; e += blockDim.x) {
            const int r = e / 16, kk = e % 16;
            const int k = k0 + kk;
            as[kk][r] = (m0 + r < M && k < K) ? A[(m0 + r) * K + k] : 0.0f;
            bs[kk][r] = (n0 + r < N && k < K) ? B[(n0 + r) * K + k] : 0.0f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                a[i] = as[kk][tm + 16 * i];
                b[i] = bs[kk][tn + 16 * i];
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t m = m0 + tm + 16 * i;
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int64_t n = n0 + tn + 16 * j;
            if (n < N) Cm[m * ldc + n] = bias ? __fadd_rn(acc[i][j], bias[n]) : acc[i][j];
        }
    }
}

// GroupNorm statistics over token-major [P][C] in kGroups groups of C/kGroups
// consecutive channels: per (group, block) partial double sums of x (pass 0)
// or of (x - mean)^2 rounded in f32 (pass 1), reduced in a fixed order.
constexpr int GN_BLOCKS = 64;

__global__ void sh_gn_partial_kernel(const float *__restrict__ x, int64_t P, int C, const float *__restrict__ mean,
                                     double *__restrict__ part) {
    const int g = blockIdx.y, cg = C / kGroups;
    const int64_t n = P * cg;
    double s = 0.0;
    for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < n;
         e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float v = x[(e / cg) * C + g * cg + e % cg];
        if (mean) {
            const float d = __fsub_rn(v, mean[g]);
            s += static_cast<double>(__fmul_rn(d, d));
        } else {
            s += static_cast<double>(v);
        }
    }
    __shared__ double red[256];
    red[threadIdx.x] = s;
    __syncthreads();
    for (int o = blockDim.x / 2; o > 0; o >>= 1) {
        if (threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
        __syncthreads();
    }
    if (threadIdx.x == 0) part[g * gridDim.x + blockIdx.x] = red[0];
}

// pass 0: mean[g] = sum / n; pass 1: scale[g] = 1 / sqrt(sum / n + eps)
__global__ void sh_gn_final_kernel(const double *__restrict__ part, int nparts, int64_t n, float eps, int pass,
                                   float *__restrict__ out) {
    const int g = threadIdx.x;
    if (g >= kGroups) return;
    double s = 0.0;
    for (int i = 0; i < nparts; ++i) s += part[g * nparts + i];
    const float v = static_cast<float>(s / static_cast<double>(n));
    out[g] = pass == 0 ? v : __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(v, eps)));
}

// x = fp16(x) in place (the im2col of an F16 1x1 kernel)
__global__ void sh_round_f16_kernel(float *x, int64_t n) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) x[i] = __half2float(__float2half_rn(x[i]));
}

// y = relu(((x - mean) * scale) * w[c] + b[c])
__global__ void sh_gn_apply_kernel(float *x, int64_t P, int C, const float *__restrict__ mean,
                                   const float *__restrict__ scale, const float *__restrict__ w,
                                   const float *__restrict__ b) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= P * C) return;
    const int c = static_cast<int>(i % C), g = c / (C / kGroups);
    const float v = __fmul_rn(__fsub_rn(x[i], mean[g]), scale[g]);
    x[i] = fmaxf(__fadd_rn(__fmul_rn(v, w[c]), b[c]), 0.0f);
}

struct Lin {
    sam3b200_weight *w = nullptr;
    DevBuf b;
    bool set() const { return w && b.p; }
};

}  // namespace

struct SegHead {
    Backend *be = nullptr;
    sam3b200_seg_hparams hp{};
    Lin ca_q, ca_kv, ca_o, me[3];
    DevBuf canw, canb, convw[2], convb[2], gnw[2], gnb[2], instw, instb;  // convw: fp16 [O][(ky*3+kx)*C + c]
    bool inst_f16 = false;
    // activations
    DevBuf enc, xn, q, kv, att, tmp, mask, m0, m1, emb, h1, h2, mev, out, gn_part, gn_stat;
    DevBuf x16, col;  // the 3x3 convolutions' fp16 input and im2col operand
    // host-run staging
    DevBuf in_enc, in_fpn0, in_fpn1, in_q, in_text, in_bias;
    std::vector<std::string> missing;
};

namespace {

bool sok(SegHead *h, cudaError_t e, const char *what) {
    h->be->count(1);
    return cuda_ok(e, what);
}

bool slin(SegHead *h, const Lin &l, const float *x, int64_t ldx, int64_t rows, float *y, int64_t ldy) {
    return run_mul_mat(h->be, reinterpret_cast<const Weight *>(l.w), x, ldx, rows, l.b.as<float>(), y, ldy,
                       nullptr) == SAM3B200_STATUS_SUCCESS;
}

bool gemm_nt(SegHead *h, const float *A, const float *B, int64_t M, int64_t N, int K, const float *bias, float *C) {
    dim3 grid(static_cast<unsigned>((N + 63) / 64), static_cast<unsigned>((M + 63) / 64));
    sh_gemm_nt_kernel<<<grid, 256, 0, h->be->stream>>>(A, B, M, N, K, bias, C, N);
    return sok(h, cudaGetLastError(), "seg gemm");
}

// relu(GN(conv3x3(merged))) in place of `out`
bool conv_gn(SegHead *h, int stage, const float *merged, int S, float *out) {
    const int D = h->hp.d_model;
    cudaStream_t s = h->be->stream;
    const int64_t P = static_cast<int64_t>(S) * S;
    GemmF16Args g{};
    g.a = h->col.p;
    g.b = h->convw[stage].p;
    g.M = static_cast<int>(P);
    g.N = D;
    g.K = 9 * D;
    g.bias = h->convb[stage].as<float>();
    g.out = out;
    g.ldo = D;
    g.store = GEMM_STORE_ROWMAJOR;
    g.err = h->be->err;
    h->be->count(3);
    if (!cuda_ok(f32_to_f16(merged, P * D, h->x16.p, s), "seg conv input") ||
        !cuda_ok(im2col3x3_f16(h->x16.p, S, S, D, h->col.p, s), "seg im2col") ||
        !cuda_ok(gemm_f16(g, h->be->num_sms, s), "seg conv3x3"))
        return false;
    double *part = h->gn_part.as<double>();
    float *mean = h->gn_stat.as<float>(), *scale = mean + kGroups;
    const int64_t n = P * (D / kGroups);
    sh_gn_partial_kernel<<<dim3(GN_BLOCKS, kGroups), 256, 0, s>>>(out, P, D, nullptr, part);
    sh_gn_final_kernel<<<1, 32, 0, s>>>(part, GN_BLOCKS, n, 1e-5f, 0, mean);
    sh_gn_partial_kernel<<<dim3(GN_BLOCKS, kGroups), 256, 0, s>>>(out, P, D, mean, part);
    sh_gn_final_kernel<<<1, 32, 0, s>>>(part, GN_BLOCKS, n, 1e-5f, 1, scale);
    sh_gn_apply_kernel<<<ew_blocks(P * D), 256, 0, s>>>(out, P, D, mean, scale, h->gnw[stage].as<float>(),
                                                         h->gnb[stage].as<float>());
    return sok(h, cudaGetLastError(), "seg group norm");
}

bool forward(SegHead *h, const float *enc_in, const float *fpn0, const float *fpn1, const float *queries, int nq,
             const float *text, const float *bias, int T) {
    const int D = h->hp.d_model, NH = h->hp.heads, HD = D / NH, S = h->hp.feat;
    const int64_t N = static_cast<int64_t>(S) * S, P1 = 4 * N, P2 = 16 * N;
    cudaStream_t s = h->be->stream;
    float *enc = h->enc.as<float>(), *xn = h->xn.as<float>(), *q = h->q.as<float>(), *kv = h->kv.as<float>();
    float *att = h->att.as<float>(), *tmp = h->tmp.as<float>();
    // cross-attention of the encoder tokens to the prompt
    const __half *mask = nullptr;
    if (bias) {
        ew_bias_mask_kernel<<<ew_blocks(N * T), 256, 0, s>>>(bias, N, T, h->mask.as<__half>());
        if (!sok(h, cudaGetLastError(), "seg prompt mask")) return false;
        mask = h->mask.as<__half>();
    }
    ln_rows_kernel<<<ew_blocks(N * 32), 256, 0, s>>>(enc_in, static_cast<int>(N), D, h->canw.as<float>(),
                                                     h->canb.as<float>(), 1e-5f, xn);
    const AttnStrides s1{0, HD, D}, s2{0, HD, 2 * D};
    if (!sok(h, cudaGetLastError(), "seg norm") || !slin(h, h->ca_q, xn, D, N, q, D) ||
        !slin(h, h->ca_kv, text, D, T, kv, 2 * D) ||
        !sok(h, attention_mma(HD, q, s1, static_cast<int>(N), kv, s2, kv + D, s2, T, 1, NH, mask, T,
                               1.0f / sqrtf(static_cast<float>(HD)), att, s1, s),
             "seg prompt attention") ||
        !slin(h, h->ca_o, att, D, N, tmp, D))
        return false;
    ew_add_kernel<<<ew_blocks(N * D), 256, 0, s>>>(enc_in, tmp, N * D, enc);
    if (!sok(h, cudaGetLastError(), "seg residual")) return false;
    // pixel decoder
    float *m0 = h->m0.as<float>(), *m1 = h->m1.as<float>();
    sh_up_add_kernel<<<ew_blocks(P1 * D), 256, 0, s>>>(fpn1, enc, 2 * S, D, m0);
    if (!sok(h, cudaGetLastError(), "seg upsample 0") || !conv_gn(h, 0, m0, 2 * S, m1)) return false;
    sh_up_add_kernel<<<ew_blocks(P2 * D), 256, 0, s>>>(fpn0, m1, 4 * S, D, h->emb.as<float>());
    float *p1 = h->m0.as<float>();  // m0 holds 16N x D values: reused for the 288 x 288 stage
    if (!sok(h, cudaGetLastError(), "seg upsample 1") || !conv_gn(h, 1, h->emb.as<float>(), 4 * S, p1)) return false;
    // instance embedding (1x1) and mask embedding MLP
    float *emb = h->emb.as<float>();
    if (h->inst_f16) {
        sh_round_f16_kernel<<<ew_blocks(P2 * D), 256, 0, s>>>(p1, P2 * D);
        if (!sok(h, cudaGetLastError(), "seg fp16 input")) return false;
    }
    if (!gemm_nt(h, p1, h->instw.as<float>(), P2, D, D, h->instb.as<float>(), emb)) return false;
    float *h1 = h->h1.as<float>(), *h2 = h->h2.as<float>(), *mev = h->mev.as<float>();
    auto relu = [&](float *x, int64_t n) {
        ew_relu_kernel<<<ew_blocks(n), 256, 0, s>>>(x, n);
        return sok(h, cudaGetLastError(), "seg relu");
    };
    if (!slin(h, h->me[0], queries, D, nq, h1, D) || !relu(h1, static_cast<int64_t>(nq) * D) ||
        !slin(h, h->me[1], h1, D, nq, h2, D) || !relu(h2, static_cast<int64_t>(nq) * D) ||
        !slin(h, h->me[2], h2, D, nq, mev, D))
        return false;
    // masks[q][pixel]
    return gemm_nt(h, mev, emb, nq, P2, D, nullptr, h->out.as<float>());
}

bool check_ready(SegHead *h) {
    h->missing.clear();
    auto need = [&](bool ok, const char *n) {
        if (!ok) h->missing.push_back(n);
    };
    need(h->ca_q.set() && h->ca_kv.set() && h->ca_o.set(), "seg.cross_attend_prompt");
    need(h->canw.p && h->canb.p, "seg.cross_attn_norm");
    need(h->convw[0].p && h->convb[0].p && h->gnw[0].p && h->gnb[0].p, "seg.pixel_decoder.*.0");
    need(h->convw[1].p && h->convb[1].p && h->gnw[1].p && h->gnb[1].p, "seg.pixel_decoder.*.1");
    need(h->instw.p && h->instb.p, "seg.instance_seg_head");
    need(h->me[0].set() && h->me[1].set() && h->me[2].set(), "seg.mask_predictor.mask_embed");
    if (!h->missing.empty()) {
        set_error("seg: %zu tensors missing (first: %s)", h->missing.size(), h->missing[0].c_str());
        return false;
    }
    return true;
}

void sfree(SegHead *h, sam3b200_weight *&w) {
    if (w) sam3b200_weight_free(reinterpret_cast<sam3b200_backend *>(h->be), w);
    w = nullptr;
}

bool check_run(SegHead *h, int nq, int T) {
    if (nq <= 0 || nq > h->hp.max_queries || T <= 0 || T > h->hp.max_prompt) {
        set_error("seg_run: %d queries (max %d), %d prompt tokens (max %d)", nq, h->hp.max_queries, T,
                  h->hp.max_prompt);
        return false;
    }
    return check_ready(h);
}

}  // namespace
}  // namespace b200

using namespace b200;

sam3b200_seg *sam3b200_seg_create(sam3b200_backend *hb, const sam3b200_seg_hparams *hp) {
    auto *be = reinterpret_cast<Backend *>(hb);
    if (!be || !hp) return nullptr;
    if (hp->d_model != 256 || hp->heads != 8 || hp->feat <= 0 || hp->feat > 128 || hp->max_queries <= 0 ||
        hp->max_prompt <= 0) {
        set_error("seg_create: unsupported hyperparameters (d_model 256, 8 heads, feat <= 128)");
        return nullptr;
    }
    cudaSetDevice(be->device);
    auto *h = new SegHead();
    h->be = be;
    h->hp = *hp;
    const size_t D = hp->d_model, N = static_cast<size_t>(hp->feat) * hp->feat, T = hp->max_prompt;
    const size_t NQ = hp->max_queries;
    const bool ok = h->enc.alloc(N * D * 4) && h->xn.alloc(N * D * 4) && h->q.alloc(N * D * 4) &&
                    h->kv.alloc(2 * T * D * 4) && h->att.alloc(N * D * 4) && h->tmp.alloc(N * D * 4) &&
                    h->mask.alloc(N * T * 2) && h->m0.alloc(16 * N * D * 4) && h->m1.alloc(4 * N * D * 4) &&
                    h->emb.alloc(16 * N * D * 4) && h->h1.alloc(NQ * D * 4) && h->h2.alloc(NQ * D * 4) &&
                    h->mev.alloc(NQ * D * 4) && h->out.alloc(NQ * 16 * N * 4) &&
                    h->gn_part.alloc(kGroups * GN_BLOCKS * 8) && h->gn_stat.alloc(2 * kGroups * 4) &&
                    h->x16.alloc(16 * N * D * 2) && h->col.alloc(16 * N * 9 * D * 2) &&
                    h->in_enc.alloc(N * D * 4) && h->in_fpn0.alloc(16 * N * D * 4) && h->in_fpn1.alloc(4 * N * D * 4) &&
                    h->in_q.alloc(NQ * D * 4) && h->in_text.alloc(T * D * 4) && h->in_bias.alloc(T * 4);
    if (!ok) {
        delete h;
        return nullptr;
    }
    return reinterpret_cast<sam3b200_seg *>(h);
}

void sam3b200_seg_free(sam3b200_seg *hh) {
    auto *h = reinterpret_cast<SegHead *>(hh);
    if (!h) return;
    cudaSetDevice(h->be->device);
    cudaStreamSynchronize(h->be->stream);
    for (Lin *l : {&h->ca_q, &h->ca_kv, &h->ca_o, &h->me[0], &h->me[1], &h->me[2]}) sfree(h, l->w);
    delete h;
}

int sam3b200_seg_set_tensor(sam3b200_seg *hh, const char *name_c, int type, const void *data, const int64_t *ne) {
    auto *h = reinterpret_cast<SegHead *>(hh);
    if (!h || !name_c || !data || !ne) return SAM3B200_STATUS_FAILED;
    cudaSetDevice(h->be->device);
    auto *hb = reinterpret_cast<sam3b200_backend *>(h->be);
    const std::string name(name_c);
    const int64_t D = h->hp.d_model;
    const int64_t n = ne[0] * (ne[1] > 0 ? ne[1] : 1) * (ne[2] > 0 ? ne[2] : 1) * (ne[3] > 0 ? ne[3] : 1);
    const int OK = SAM3B200_STATUS_SUCCESS, BAD = SAM3B200_STATUS_FAILED;
    std::vector<float> v;
    auto vec_part = [&](DevBuf &b, int64_t want, int64_t off, int64_t len) -> int {
        if (n != want || !to_f32(type, data, n, v)) {
            set_error("%s: %lld elements of type %d, expected %lld F32/F16", name_c, (long long)n, type,
                      (long long)want);
            return BAD;
        }
        return upload(b, v.data() + off, static_cast<size_t>(len) * 4, h->be->stream) ? OK : BAD;
    };
    auto vec = [&](DevBuf &b, int64_t want) { return vec_part(b, want, 0, want); };
    auto shape_ok = [&](int64_t K, int64_t N) {
        if (ne[0] == K && ne[1] == N) return true;
        set_error("%s: shape [%lld, %lld], expected [%lld, %lld]", name_c, (long long)ne[0], (long long)ne[1],
                  (long long)K, (long long)N);
        return false;
    };
    auto rows = [&](Lin &l, int64_t r0, int64_t nr) -> bool {
        sfree(h, l.w);
        l.w = upload_weight_rows(h->be, type, data, D, r0, nr);
        return l.w != nullptr;
    };
    if (name == "seg.cross_attend_prompt.in_proj_weight")
        return shape_ok(D, 3 * D) && rows(h->ca_q, 0, D) && rows(h->ca_kv, D, 2 * D) ? OK : BAD;
    if (name == "seg.cross_attend_prompt.in_proj_bias")
        return vec_part(h->ca_q.b, 3 * D, 0, D) == OK ? vec_part(h->ca_kv.b, 3 * D, D, 2 * D) : BAD;
    if (name == "seg.cross_attend_prompt.out_proj.weight") {
        if (!shape_ok(D, D)) return BAD;
        sfree(h, h->ca_o.w);
        h->ca_o.w = sam3b200_weight_upload(hb, type, data, D, D);
        return h->ca_o.w ? OK : BAD;
    }
    if (name == "seg.cross_attend_prompt.out_proj.bias") return vec(h->ca_o.b, D);
    if (name == "seg.cross_attn_norm.weight") return vec(h->canw, D);
    if (name == "seg.cross_attn_norm.bias") return vec(h->canb, D);
    for (int i = 0; i < 3; ++i) {
        const std::string si = std::to_string(i);
        if (name == "seg.pixel_decoder.conv_layers." + si + ".weight") {  // ggml [3, 3, D, D]
            if (ne[0] != 3 || ne[1] != 3 || ne[2] != D || ne[3] != D) {
                set_error("%s: expected [3, 3, %lld, %lld]", name_c, (long long)D, (long long)D);
                return BAD;
            }
            if (i == 2) return OK;  // registered but unused by the pixel decoder (sam3.cpp:8954-8955)
            if (!to_f32(type, data, n, v)) return BAD;
            std::vector<float> w(static_cast<size_t>(n));  // ggml [kx][ky][c][o] -> [o][(ky*3+kx)*C + c]
            for (int64_t o = 0; o < D; ++o)
                for (int64_t c = 0; c < D; ++c)
                    for (int ky = 0; ky < 3; ++ky)
                        for (int kx = 0; kx < 3; ++kx)
                            w[static_cast<size_t>(o * 9 * D + (ky * 3 + kx) * D + c)] =
                                v[static_cast<size_t>(((o * D + c) * 3 + ky) * 3 + kx)];
            return upload_f16(h->convw[i], w, h->be->stream) ? OK : BAD;
        }
        if (name == "seg.pixel_decoder.conv_layers." + si + ".bias") return i == 2 ? OK : vec(h->convb[i], D);
        if (name == "seg.pixel_decoder.norms." + si + ".weight") return i == 2 ? OK : vec(h->gnw[i], D);
        if (name == "seg.pixel_decoder.norms." + si + ".bias") return i == 2 ? OK : vec(h->gnb[i], D);
        if (name == "seg.mask_predictor.mask_embed.layers." + si + ".weight") {
            if (!shape_ok(D, D)) return BAD;
            sfree(h, h->me[i].w);
            h->me[i].w = sam3b200_weight_upload(hb, type, data, D, D);
            return h->me[i].w ? OK : BAD;
        }
        if (name == "seg.mask_predictor.mask_embed.layers." + si + ".bias") return vec(h->me[i].b, D);
    }
    if (name == "seg.instance_seg_head.weight") {  // ggml [1, 1, D, D], held in f32
        if (n != D * D) {
            set_error("%s: expected [1, 1, %lld, %lld]", name_c, (long long)D, (long long)D);
            return BAD;
        }
        h->inst_f16 = type == SAM3B200_TYPE_F16;
        return vec(h->instw, n);
    }
    if (name == "seg.instance_seg_head.bias") return vec(h->instb, D);
    if (name == "seg.semantic_seg_head.weight" || name == "seg.semantic_seg_head.bias")
        return OK;  // registered, not part of the instance-mask graph
    set_error("seg: unknown tensor %s", name_c);
    return BAD;
}

int sam3b200_seg_missing(sam3b200_seg *hh, char *buf, int cap) {
    auto *h = reinterpret_cast<SegHead *>(hh);
    if (!h) return -1;
    check_ready(h);
    std::string all;
    for (const auto &s : h->missing) all += s + "\n";
    if (buf && cap > 0) snprintf(buf, static_cast<size_t>(cap), "%s", all.c_str());
    return static_cast<int>(h->missing.size());
}

int sam3b200_seg_run_device(sam3b200_seg *hh, const float *enc, const float *fpn0, const float *fpn1,
                            const float *queries, int n_queries, const float *text, const float *text_bias,
                            int n_text) {
    auto *h = reinterpret_cast<SegHead *>(hh);
    if (!h || !enc || !fpn0 || !fpn1 || !queries || !text) {
        set_error("seg_run: null argument");
        return SAM3B200_STATUS_FAILED;
    }
    cudaSetDevice(h->be->device);
    if (!check_run(h, n_queries, n_text)) return SAM3B200_STATUS_FAILED;
    return forward(h, enc, fpn0, fpn1, queries, n_queries, text, text_bias, n_text) ? SAM3B200_STATUS_SUCCESS
                                                                                    : SAM3B200_STATUS_FAILED;
}

int sam3b200_seg_run(sam3b200_seg *hh, const float *enc, const float *fpn0, const float *fpn1, const float *queries,
                     int n_queries, const float *text, const float *text_bias, int n_text) {
    auto *h = reinterpret_cast<SegHead *>(hh);
    if (!h || !enc || !fpn0 || !fpn1 || !queries || !text) {
        set_error("seg_run: null argument");
        return SAM3B200_STATUS_FAILED;
    }
    cudaSetDevice(h->be->device);
    if (!check_run(h, n_queries, n_text)) return SAM3B200_STATUS_FAILED;
    const size_t N = static_cast<size_t>(h->hp.feat) * h->hp.feat, D = h->hp.d_model;
    cudaStream_t s = h->be->stream;
    auto up = [&](DevBuf &d, const void *src, size_t bytes, const char *what) {
        return cuda_ok(cudaMemcpyAsync(d.p, src, bytes, cudaMemcpyHostToDevice, s), what);
    };
    if (!up(h->in_enc, enc, N * D * 4, "seg enc") || !up(h->in_fpn0, fpn0, 16 * N * D * 4, "seg fpn0") ||
        !up(h->in_fpn1, fpn1, 4 * N * D * 4, "seg fpn1") ||
        !up(h->in_q, queries, static_cast<size_t>(n_queries) * D * 4, "seg queries") ||
        !up(h->in_text, text, static_cast<size_t>(n_text) * D * 4, "seg text") ||
        (text_bias && !up(h->in_bias, text_bias, static_cast<size_t>(n_text) * 4, "seg bias")))
        return SAM3B200_STATUS_FAILED;
    return forward(h, h->in_enc.as<float>(), h->in_fpn0.as<float>(), h->in_fpn1.as<float>(), h->in_q.as<float>(),
                   n_queries, h->in_text.as<float>(), text_bias ? h->in_bias.as<float>() : nullptr, n_text)
               ? SAM3B200_STATUS_SUCCESS
               : SAM3B200_STATUS_FAILED;
}

int sam3b200_seg_output(sam3b200_seg *hh, const float **dev) {
    auto *h = reinterpret_cast<SegHead *>(hh);
    if (!h || !dev) return SAM3B200_STATUS_FAILED;
    *dev = h->out.as<float>();
    return SAM3B200_STATUS_SUCCESS;
}
