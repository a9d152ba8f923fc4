// mem_enc.cu -- the memory encoder of the video tracker on the B200 backend:
// sam3_encode_memory (sam3.cpp:11510-11615) from the mask logits to the
// [mem_dim, H, H] memory features it stores:
//
//   mask logits -> bilinear to img -> sigmoid * scale + bias -> bilinear to 16H
//   mask downsampler: 4 x (conv 3x3 s2 p1 + bias, LayerNorm2d, GELU), conv 1x1
//   pix = conv 1x1 (pixel features of the frame)
//   x = pix + downsampled mask
//   fuser: 2 CXBlocks (sam3_cxblock_forward, :9066-9108): depthwise 7x7,
//          LayerNorm2d, pwconv1 -> GELU -> pwconv2, x += gamma * h
//   out = conv 1x1 (d_model -> mem_dim) [+ no_obj_embed_spatial if the object
//         score is <= 0]
//
// Layouts: the downsampler runs channel-major [C][H][W] (ggml's convolution
// layout); the fuser and the output are token-major [H*W][C] (ggml's
// channel-first "internal" layout).  Convolution kernels are held in f32; an
// F16 kernel (F16 weight files) makes ggml round the im2col input to fp16,
// which the direct convolution repeats.  The pointwise MLP of the fuser is
// run_mul_mat (the exact quantised MUL_MAT, or the fp16 GEMM for F16).
#include "../../include/sam3_b200.h"
#include "act.cuh"
#include "model_util.h"
#include "sgemm.cuh"
#include "row_norm.cuh"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

namespace b200 {
namespace {

inline unsigned eblocks(int64_t n) { return static_cast<unsigned>((n + 255) / 256); }

// sam3_bilinear_interpolate (sam3.cpp:9617-9643): half-pixel centres in
// double, clamped, the last row/column pair reused at the edge; the blend is
// evaluated in f32 without contraction.  post == 1 applies the memory
// encoder's sigmoid(v) * scale + bias (sam3.cpp:11521-11524).
__global__ void bilinear_kernel(const float *__restrict__ src, int sw, int sh, float *__restrict__ dst, int dw, int dh,
                                int post, float scale, float bias) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<int64_t>(dw) * dh) return;
    const int x = static_cast<int>(i % dw), y = static_cast<int>(i / dw);
    double fy = (y + 0.5) * (static_cast<double>(sh) / dh) - 0.5;
    fy = fmax(0.0, fmin(fy, static_cast<double>(sh - 1)));
    double fx = (x + 0.5) * (static_cast<double>(sw) / dw) - 0.5;
    fx = fmax(0.0, fmin(fx, static_cast<double>(sw - 1)));
    const int y0 = min(static_cast<int>(fy), sh - 2), x0 = min(static_cast<int>(fx), sw - 2);
    const float wy = static_cast<float>(fy - y0), wx = static_cast<float>(fx - x0);
    const float *r0 = src + static_cast<int64_t>(y0) * sw, *r1 = r0 + sw;
    const float ux = __fsub_rn(1.0f, wx), uy = __fsub_rn(1.0f, wy);
    const float top = __fadd_rn(__fmul_rn(ux, r0[x0]), __fmul_rn(wx, r0[x0 + 1]));
    const float bot = __fadd_rn(__fmul_rn(ux, r1[x0]), __fmul_rn(wx, r1[x0 + 1]));
    float v = __fadd_rn(__fmul_rn(uy, top), __fmul_rn(wy, bot));
    if (post == 1) {
        const float s = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v)));
        v = __fadd_rn(__fmul_rn(s, scale), bias);
    }
    dst[i] = v;
}

// Depthwise KxK convolution, padding K/2, token-major [H][W][C] in and out
// (ggml_conv_2d_dw_direct with an f32 kernel w[c][ky][kx]) plus the bias.
__global__ void depthwise_kernel(const float *__restrict__ x, int H, int W, int C, const float *__restrict__ w,
                                 const float *__restrict__ bias, int K, float *__restrict__ y) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<int64_t>(H) * W * C) return;
    const int c = static_cast<int>(i % C);
    const int px = static_cast<int>((i / C) % W), py = static_cast<int>(i / C / W);
    const float *wc = w + static_cast<int64_t>(c) * K * K;
    const int r = K / 2;
    float acc = 0.0f;
    for (int ky = 0; ky < K; ++ky) {
        const int iy = py + ky - r;
        if (iy < 0 || iy >= H) continue;
        for (int kx = 0; kx < K; ++kx) {
            const int ix = px + kx - r;
            if (ix < 0 || ix >= W) continue;
            acc = fmaf(x[(static_cast<int64_t>(iy) * W + ix) * C + c], wc[ky * K + kx], acc);
        }
    }
    y[i] = __fadd_rn(acc, bias[c]);
}

__global__ void gelu_tanh_kernel(float *x, int64_t n) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) x[i] = gelu_tanh_f16(x[i]);
}

// c = a + b (c may alias a or b)
__global__ void me_add_kernel(const float *a, const float *b, int64_t n, float *c) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) c[i] = __fadd_rn(a[i], b[i]);
}

// x[p][c] += h[p][c] * gamma[c], the product rounded first (ggml_mul, ggml_add)
__global__ void scale_residual_kernel(float *x, const float *__restrict__ h, const float *__restrict__ gamma, int C,
                                      int64_t n) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) x[i] = __fadd_rn(x[i], __fmul_rn(h[i], gamma[i % C]));
}

// x[p][c] += e[c]
__global__ void add_channel_kernel(float *x, const float *__restrict__ e, int C, int64_t n) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) x[i] = __fadd_rn(x[i], e[i % C]);
}

struct ConvW {
    DevBuf w, b;
    int ic = 0, oc = 0, k = 0;
    bool f16 = false;  // the file held an F16 kernel: the input is rounded to fp16
    bool set() const { return w.p && b.p; }
};

struct FuserW {
    DevBuf dww, dwb, nw, nb, gamma, f1b, f2b;
    sam3b200_weight *f1 = nullptr, *f2 = nullptr;
};

constexpr int kDsChannels[5] = {1, 4, 16, 64, 256};
constexpr int kDsConv[4] = {0, 3, 6, 9};
constexpr int kDsNorm[4] = {1, 4, 7, 10};

}  // namespace

struct MemEnc {
    Backend *be = nullptr;
    sam3b200_mem_enc_hparams hp{};
    ConvW ds[5], pix, outp;  // ds[4]: the final 1x1 of the downsampler
    DevBuf dsnw[4], dsnb[4], noobj;
    std::vector<FuserW> fu;
    DevBuf logits, hires, a, b, pixin, x, h, xn, mlp, out;
    DevBuf col;  // im2col rows of the downsampler's convolutions
    std::vector<std::string> missing;
};

namespace {

bool eok(MemEnc *m, cudaError_t e, const char *what) {
    m->be->count(1);
    return cuda_ok(e, what);
}

bool forward(MemEnc *m, const float *logits, int mw, int mh, const float *pixf, float obj_score) {
    const int H = m->hp.feat, I = 16 * H, IMG = m->hp.img, D = m->hp.d_model, MD = m->hp.mem_dim;
    const int F = m->hp.fuser_dim;
    const int64_t P = static_cast<int64_t>(H) * H, PD = P * D;
    cudaStream_t s = m->be->stream;
    float *hires = m->hires.as<float>(), *a = m->a.as<float>(), *b = m->b.as<float>();
    // mask preprocessing: logits -> img x img -> sigmoid * scale + bias -> I x I
    bilinear_kernel<<<eblocks(static_cast<int64_t>(IMG) * IMG), 256, 0, s>>>(logits, mw, mh, hires, IMG, IMG, 1,
                                                                             m->hp.sigmoid_scale, m->hp.sigmoid_bias);
    if (!eok(m, cudaGetLastError(), "mem_enc mask resize")) return false;
    bilinear_kernel<<<eblocks(static_cast<int64_t>(I) * I), 256, 0, s>>>(hires, IMG, IMG, a, I, I, 0, 0.f, 0.f);
    if (!eok(m, cudaGetLastError(), "mem_enc mask interpolate")) return false;
    // downsampler: 4 x (3x3 s2 p1 conv, LayerNorm2d, GELU), channel-major a -> b -> a ...
    int side = I;
    for (int st = 0; st < 4; ++st) {
        const ConvW &c = m->ds[st];
        const int os = (side + 2 - 3) / 2 + 1;
        const int64_t n = static_cast<int64_t>(c.oc) * os * os;
        // 3x3 s2 p1: f32 im2col + f32 GEMM, channel-major out [oc][os * os] (bias per output channel)
        const int64_t pix = static_cast<int64_t>(os) * os, kk = static_cast<int64_t>(c.ic) * 9;
        if (m->col.n < static_cast<size_t>(pix * kk) * 4 && !m->col.alloc(static_cast<size_t>(pix * kk) * 4)) return false;
        if (!eok(m, im2col_chw(a, c.ic, side, side, 3, 2, 1, os, os, m->col.as<float>(), s), "mem_enc im2col") ||
            !eok(m, sgemm_nt(c.w.as<float>(), kk, 1, m->col.as<float>(), kk, 1, c.oc, static_cast<int>(pix),
                             static_cast<int>(kk), c.b.as<float>(), b, pix, false, s, c.f16, true),
                 "mem_enc downsample conv"))
            return false;
        ln_channels_kernel<<<eblocks(static_cast<int64_t>(os) * os), 256, 0, s>>>(
            b, c.oc, static_cast<int64_t>(os) * os, m->dsnw[st].as<float>(), m->dsnb[st].as<float>(), 1e-6f, a);
        if (!eok(m, cudaGetLastError(), "mem_enc downsample norm")) return false;
        gelu_tanh_kernel<<<eblocks(n), 256, 0, s>>>(a, n);
        if (!eok(m, cudaGetLastError(), "mem_enc downsample gelu")) return false;
        side = os;
    }
    // final 1x1 of the downsampler (channel-major a [D][P] -> token-major b [P][D])
    float *x = m->x.as<float>(), *h = m->h.as<float>(), *xn = m->xn.as<float>();
    // (1x1 convolutions as f32 GEMMs: ggml_conv_2d of an F32 kernel is an f32 MUL_MAT)
    if (!eok(m, sgemm_nt(a, 1, P, m->ds[4].w.as<float>(), D, 1, static_cast<int>(P), D, D, m->ds[4].b.as<float>(), b, D,
                         m->ds[4].f16, s),
             "mem_enc downsample 1x1"))
        return false;
    // pixel projection (token-major in and out), then x = pix + mask features
    if (!eok(m, sgemm_nt(pixf, D, 1, m->pix.w.as<float>(), D, 1, static_cast<int>(P), D, D, m->pix.b.as<float>(), x, D,
                         m->pix.f16, s),
             "mem_enc pixel projection"))
        return false;
    me_add_kernel<<<eblocks(PD), 256, 0, s>>>(x, b, PD, x);
    if (!eok(m, cudaGetLastError(), "mem_enc fuse")) return false;
    for (const FuserW &f : m->fu) {
        depthwise_kernel<<<eblocks(PD), 256, 0, s>>>(x, H, H, D, f.dww.as<float>(), f.dwb.as<float>(), 7, h);
        if (!eok(m, cudaGetLastError(), "mem_enc depthwise")) return false;
        ln_rows_kernel<<<eblocks(P * 32), 256, 0, s>>>(h, static_cast<int>(P), D, f.nw.as<float>(), f.nb.as<float>(),
                                                       1e-6f, xn);
        if (!eok(m, cudaGetLastError(), "mem_enc fuser norm") ||
            run_mul_mat(m->be, reinterpret_cast<const Weight *>(f.f1), xn, D, P, f.f1b.as<float>(), m->mlp.as<float>(),
                        F, nullptr) != SAM3B200_STATUS_SUCCESS)
            return false;
        gelu_tanh_kernel<<<eblocks(P * F), 256, 0, s>>>(m->mlp.as<float>(), P * F);
        if (!eok(m, cudaGetLastError(), "mem_enc fuser gelu") ||
            run_mul_mat(m->be, reinterpret_cast<const Weight *>(f.f2), m->mlp.as<float>(), F, P, f.f2b.as<float>(), h,
                        D, nullptr) != SAM3B200_STATUS_SUCCESS)
            return false;
        scale_residual_kernel<<<eblocks(PD), 256, 0, s>>>(x, h, f.gamma.as<float>(), D, PD);
        if (!eok(m, cudaGetLastError(), "mem_enc fuser residual")) return false;
    }
    float *out = m->out.as<float>();
    if (!eok(m, sgemm_nt(x, D, 1, m->outp.w.as<float>(), D, 1, static_cast<int>(P), MD, D, m->outp.b.as<float>(), out,
                         MD, m->outp.f16, s),
             "mem_enc out proj"))
        return false;
    if (obj_score <= 0.0f && m->noobj.p) {  // occluded: + no_obj_embed_spatial (sam3.cpp:11602-11615)
        add_channel_kernel<<<eblocks(P * MD), 256, 0, s>>>(out, m->noobj.as<float>(), MD, P * MD);
        if (!eok(m, cudaGetLastError(), "mem_enc no-object embedding")) return false;
    }
    return true;
}

bool check_ready(MemEnc *m) {
    m->missing.clear();
    for (int st = 0; st < 4; ++st) {
        if (!m->ds[st].set()) m->missing.push_back("mem_enc.ds." + std::to_string(kDsConv[st]));
        if (!m->dsnw[st].p || !m->dsnb[st].p) m->missing.push_back("mem_enc.ds." + std::to_string(kDsNorm[st]));
    }
    if (!m->ds[4].set()) m->missing.push_back("mem_enc.ds.12");
    if (!m->pix.set()) m->missing.push_back("mem_enc.pix_feat_proj");
    if (!m->outp.set()) m->missing.push_back("mem_enc.out_proj");
    for (size_t i = 0; i < m->fu.size(); ++i) {
        const FuserW &f = m->fu[i];
        if (!(f.dww.p && f.dwb.p && f.nw.p && f.nb.p && f.gamma.p && f.f1 && f.f2 && f.f1b.p && f.f2b.p))
            m->missing.push_back("mem_enc.fuser." + std::to_string(i));
    }
    if (!m->missing.empty()) {
        set_error("mem_enc: %zu tensors missing (first: %s)", m->missing.size(), m->missing[0].c_str());
        return false;
    }
    return true;
}

void efree(MemEnc *m, sam3b200_weight *&w) {
    if (w) sam3b200_weight_free(reinterpret_cast<sam3b200_backend *>(m->be), w);
    w = nullptr;
}

bool check_run(MemEnc *m, int mw, int mh) {
    if (mw < 2 || mh < 2 || static_cast<int64_t>(mw) * mh > m->hp.max_mask) {
        set_error("mem_enc_run: mask %dx%d (at least 2x2, at most %d values)", mw, mh, m->hp.max_mask);
        return false;
    }
    return check_ready(m);
}

}  // namespace
}  // namespace b200

using namespace b200;

sam3b200_mem_enc *sam3b200_mem_enc_create(sam3b200_backend *hb, const sam3b200_mem_enc_hparams *hp) {
    auto *be = reinterpret_cast<Backend *>(hb);
    if (!be || !hp) return nullptr;
    if (hp->feat <= 0 || hp->feat > 256 || hp->img < 2 || hp->img > 8192 || hp->d_model != kDsChannels[4] ||
        hp->mem_dim <= 0 || hp->fuser_layers <= 0 || hp->fuser_dim <= 0 || hp->fuser_dim % 32 != 0 ||
        hp->max_mask < 4) {
        set_error("mem_enc_create: unsupported hyperparameters (d_model 256, feat <= 256, fuser_dim %% 32 == 0)");
        return nullptr;
    }
    cudaSetDevice(be->device);
    auto *m = new MemEnc();
    m->be = be;
    m->hp = *hp;
    m->fu.resize(hp->fuser_layers);
    for (int st = 0; st < 4; ++st) {
        m->ds[st].ic = kDsChannels[st];
        m->ds[st].oc = kDsChannels[st + 1];
        m->ds[st].k = 3;
    }
    const int D = hp->d_model;
    m->ds[4].ic = m->ds[4].oc = D;
    m->ds[4].k = 1;
    m->pix.ic = m->pix.oc = D;
    m->pix.k = 1;
    m->outp.ic = D;
    m->outp.oc = hp->mem_dim;
    m->outp.k = 1;
    const size_t I = 16 * static_cast<size_t>(hp->feat), P = static_cast<size_t>(hp->feat) * hp->feat;
    const size_t img = hp->img;
    // every downsampler stage holds I*I values (channels x4 as each side halves); the input mask too
    const bool ok = m->logits.alloc(static_cast<size_t>(hp->max_mask) * 4) && m->hires.alloc(img * img * 4) &&
                    m->a.alloc(I * I * 4) && m->b.alloc(I * I * 4) && m->pixin.alloc(P * D * 4) &&
                    m->x.alloc(P * D * 4) && m->h.alloc(P * D * 4) && m->xn.alloc(P * D * 4) &&
                    m->mlp.alloc(P * hp->fuser_dim * 4) && m->out.alloc(P * hp->mem_dim * 4);
    if (!ok) {
        delete m;
        return nullptr;
    }
    return reinterpret_cast<sam3b200_mem_enc *>(m);
}

void sam3b200_mem_enc_free(sam3b200_mem_enc *hm) {
    auto *m = reinterpret_cast<MemEnc *>(hm);
    if (!m) return;
    cudaSetDevice(m->be->device);
    cudaStreamSynchronize(m->be->stream);
    for (auto &f : m->fu) {
        efree(m, f.f1);
        efree(m, f.f2);
    }
    delete m;
}

int sam3b200_mem_enc_set_tensor(sam3b200_mem_enc *hm, const char *name_c, int type, const void *data,
                                const int64_t *ne) {
    auto *m = reinterpret_cast<MemEnc *>(hm);
    if (!m || !name_c || !data || !ne) return SAM3B200_STATUS_FAILED;
    cudaSetDevice(m->be->device);
    auto *hb = reinterpret_cast<sam3b200_backend *>(m->be);
    const std::string name(name_c);
    const int64_t D = m->hp.d_model, MD = m->hp.mem_dim, F = m->hp.fuser_dim;
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
    auto conv = [&](ConvW &c) -> int {  // ggml [K, K, IC, OC]
        if (ne[0] != c.k || ne[1] != c.k || ne[2] != c.ic || ne[3] != c.oc) {
            set_error("%s: shape [%lld, %lld, %lld, %lld], expected [%d, %d, %d, %d]", name_c, (long long)ne[0],
                      (long long)ne[1], (long long)ne[2], (long long)ne[3], c.k, c.k, c.ic, c.oc);
            return SAM3B200_STATUS_FAILED;
        }
        c.f16 = type == SAM3B200_TYPE_F16;
        return vec(c.w, n);
    };
    auto weight = [&](sam3b200_weight *&w, int64_t K, int64_t N) -> int {
        if (ne[0] != K || ne[1] != N) {
            set_error("%s: shape [%lld, %lld], expected [%lld, %lld]", name_c, (long long)ne[0], (long long)ne[1],
                      (long long)K, (long long)N);
            return SAM3B200_STATUS_FAILED;
        }
        efree(m, w);
        w = sam3b200_weight_upload(hb, type, data, K, N);
        return w ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
    };
    for (int st = 0; st < 4; ++st) {
        const std::string cp = "mem_enc.ds." + std::to_string(kDsConv[st]) + ".";
        const std::string np = "mem_enc.ds." + std::to_string(kDsNorm[st]) + ".";
        if (name == cp + "weight") return conv(m->ds[st]);
        if (name == cp + "bias") return vec(m->ds[st].b, m->ds[st].oc);
        if (name == np + "weight") return vec(m->dsnw[st], m->ds[st].oc);
        if (name == np + "bias") return vec(m->dsnb[st], m->ds[st].oc);
    }
    if (name == "mem_enc.ds.12.weight") return conv(m->ds[4]);
    if (name == "mem_enc.ds.12.bias") return vec(m->ds[4].b, D);
    if (name == "mem_enc.pix_feat_proj.weight") return conv(m->pix);
    if (name == "mem_enc.pix_feat_proj.bias") return vec(m->pix.b, D);
    if (name == "mem_enc.out_proj.weight") return conv(m->outp);
    if (name == "mem_enc.out_proj.bias") return vec(m->outp.b, MD);
    if (name == "no_obj_embed_spatial") return vec(m->noobj, MD);
    if (name == "mem_enc.tpos_enc") return SAM3B200_STATUS_SUCCESS;  // read by the host prompt builder, not here
    int fi = -1;
    char tail[64] = {0};
    if (sscanf(name_c, "mem_enc.fuser.%d.%63s", &fi, tail) == 2 && fi >= 0 && fi < static_cast<int>(m->fu.size())) {
        FuserW &fw = m->fu[fi];
        const std::string t(tail);
        if (t == "dwconv.weight") {  // ggml [7, 7, 1, D]
            if (ne[0] != 7 || ne[1] != 7 || ne[2] != 1 || ne[3] != D) {
                set_error("%s: expected [7, 7, 1, %lld]", name_c, (long long)D);
                return SAM3B200_STATUS_FAILED;
            }
            return vec(fw.dww, n);
        }
        if (t == "dwconv.bias") return vec(fw.dwb, D);
        if (t == "norm.weight") return vec(fw.nw, D);
        if (t == "norm.bias") return vec(fw.nb, D);
        if (t == "gamma") return vec(fw.gamma, D);
        if (t == "pwconv1.weight") return weight(fw.f1, D, F);
        if (t == "pwconv1.bias") return vec(fw.f1b, F);
        if (t == "pwconv2.weight") return weight(fw.f2, F, D);
        if (t == "pwconv2.bias") return vec(fw.f2b, D);
    }
    set_error("mem_enc: unknown tensor %s", name_c);
    return SAM3B200_STATUS_FAILED;
}

int sam3b200_mem_enc_missing(sam3b200_mem_enc *hm, char *buf, int cap) {
    auto *m = reinterpret_cast<MemEnc *>(hm);
    if (!m) return -1;
    check_ready(m);
    std::string all;
    for (const auto &s : m->missing) all += s + "\n";
    if (buf && cap > 0) snprintf(buf, static_cast<size_t>(cap), "%s", all.c_str());
    return static_cast<int>(m->missing.size());
}

int sam3b200_mem_enc_run_device(sam3b200_mem_enc *hm, const float *mask_logits, int mask_w, int mask_h,
                                const float *pix_feat, float obj_score) {
    auto *m = reinterpret_cast<MemEnc *>(hm);
    if (!m || !mask_logits || !pix_feat) {
        set_error("mem_enc_run: null argument");
        return SAM3B200_STATUS_FAILED;
    }
    cudaSetDevice(m->be->device);
    if (!check_run(m, mask_w, mask_h)) return SAM3B200_STATUS_FAILED;
    return forward(m, mask_logits, mask_w, mask_h, pix_feat, obj_score) ? SAM3B200_STATUS_SUCCESS
                                                                        : SAM3B200_STATUS_FAILED;
}

int sam3b200_mem_enc_run(sam3b200_mem_enc *hm, const float *mask_logits, int mask_w, int mask_h,
                         const float *pix_feat, float obj_score) {
    auto *m = reinterpret_cast<MemEnc *>(hm);
    if (!m || !mask_logits || !pix_feat) {
        set_error("mem_enc_run: null argument");
        return SAM3B200_STATUS_FAILED;
    }
    cudaSetDevice(m->be->device);
    if (!check_run(m, mask_w, mask_h)) return SAM3B200_STATUS_FAILED;
    const size_t lb = static_cast<size_t>(mask_w) * mask_h * 4;
    const size_t pb = static_cast<size_t>(m->hp.feat) * m->hp.feat * m->hp.d_model * 4;
    if (!cuda_ok(cudaMemcpyAsync(m->logits.p, mask_logits, lb, cudaMemcpyHostToDevice, m->be->stream), "mask") ||
        !cuda_ok(cudaMemcpyAsync(m->pixin.p, pix_feat, pb, cudaMemcpyHostToDevice, m->be->stream), "pix_feat"))
        return SAM3B200_STATUS_FAILED;
    return forward(m, m->logits.as<float>(), mask_w, mask_h, m->pixin.as<float>(), obj_score)
               ? SAM3B200_STATUS_SUCCESS
               : SAM3B200_STATUS_FAILED;
}

int sam3b200_mem_enc_output(sam3b200_mem_enc *hm, const float **dev) {
    auto *m = reinterpret_cast<MemEnc *>(hm);
    if (!m || !dev) return SAM3B200_STATUS_FAILED;
    *dev = m->out.as<float>();
    return SAM3B200_STATUS_SUCCESS;
}
