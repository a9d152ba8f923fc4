// hiera.cu -- the SAM2 Hiera image encoder on the B200 backend: the graph
// sam2_build_hiera_graph + sam2_build_fpn_neck_graph build (sam3.cpp:4467-4583)
// executed as a fixed sequence of kernels on the backend stream.
//
// Per block (sam2_hiera_block_forward, sam3.cpp:4299-4461), x [H*W][C_in]
// token-major f32 (ggml [C, W, H, 1]):
//   normed  = LN(x) (eps 1e-6)                                   ln_rows_kernel
//   shortcut= dim_proj(normed) (+ 2x2 max pool at a Q-stride block), or x
//   qkv     = MUL_MAT(window-partitioned normed) + bias            win_gather_q8_kernel, mmq_tc
//             (sam2_window_partition: zero padding to a multiple of the window, window index
//              wy + nWh * wx, token lx + ws * ly; global blocks keep the token order)
//   q       = 2x2 max pool of q inside each window at a Q-stride block  qpool_kernel
//   o       = softmax(q k^T / sqrt(hd)) v per (window, head)      attention_simt / fp16 GEMMs
//   x'      = shortcut + crop(unpartition(MUL_MAT(o) + bias))      unpart_add_kernel
//   x'     += fc2(ggml_gelu(fc1(LN(x')))) (tanh GELU through ggml's fp16 table)
// The four MUL_MATs of a block and the dimension projection run on the
// tcgen05 MMQ kernel (exact int32 block dots, mmq.cu); the windowed attention
// is the general SIMT flash loop (attn_simt.cu: any head dimension, query/key
// counts of Q-pooled blocks, padded windows), global attention two fp16
// tensor-core GEMMs around a row softmax.
#include "../../include/sam3_b200.h"
#include "act.cuh"
#include "sgemm.cuh"
#include "attn_simt.cuh"
#include "attn_tcw.cuh"
#include "gemm_f16.cuh"
#include "model_util.h"
#include "row_norm.cuh"
#include "vit_ops.cuh"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

namespace b200 {
namespace {

// Quantise one 32-wide block (ggml-cpu activation rule) and store codes + scale record.
__device__ __forceinline__ void q8_block_store(const float (&v)[32], int8_t *codes, __half *quads, int blk, int64_t r,
                                               int ld, int nblk) {
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
    const float d = __fdiv_rn(amax, 127.f);
    const float id = amax != 0.f ? __fdiv_rn(127.f, amax) : 0.f;
    uint32_t pk[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        uint32_t w = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e)
            w |= (static_cast<uint32_t>(__float2int_rn(__fmul_rn(v[4 * i + e], id))) & 0xFFu) << (8 * e);
        pk[i] = w;
    }
    uint4 *dst = reinterpret_cast<uint4 *>(codes + blk * 32);
    dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
    store_act_scale(quads, blk, static_cast<int>(r), ld, nblk, d);
}

// Window partition (with zero padding) of normed [H][W][C] fused with the Q8
// quantisation of the qkv MUL_MAT input: row r = w * ws^2 + lx + ws * ly of
// window w = wy + nWh * wx.  One warp per row, one lane per 32-wide block.
__global__ void win_gather_q8_kernel(const float *__restrict__ x, int H, int W, int C, int ws, int nWh, int rows,
                                     int8_t *__restrict__ codes, __half *__restrict__ quads, int ld) {
    const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= rows) return;
    const int N = ws * ws, w = r / N, n = r % N;
    const int gx = n % ws + ws * (w / nWh), gy = n / ws + ws * (w % nWh);
    const float *src = (gx < W && gy < H) ? x + (static_cast<int64_t>(gy) * W + gx) * C : nullptr;
    int8_t *cr = codes + static_cast<int64_t>(r) * C;
    for (int blk = lane; blk < C / 32; blk += 32) {
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
            const float4 q = src ? *reinterpret_cast<const float4 *>(src + blk * 32 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            v[i] = q.x;
            v[i + 1] = q.y;
            v[i + 2] = q.z;
            v[i + 3] = q.w;
        }
        q8_block_store(v, cr, quads, blk, r, ld, C / 32);
    }
}

// The same window partition into f32 rows (the input of an F16 / F32 qkv weight).
__global__ void win_gather_f32_kernel(const float *__restrict__ x, int H, int W, int C, int ws, int nWh, int64_t rows,
                                      float *__restrict__ y) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= rows * C) return;
    const int64_t r = i / C;
    const int c = static_cast<int>(i % C);
    const int N = ws * ws, w = static_cast<int>(r / N), n = static_cast<int>(r % N);
    const int gx = n % ws + ws * (w / nWh), gy = n / ws + ws * (w % nWh);
    y[i] = (gx < W && gy < H) ? x[(static_cast<int64_t>(gy) * W + gx) * C + c] : 0.0f;
}

// ggml_gelu (the CPU backend's fp16-table tanh form) in place
__global__ void gelu_tanh_inplace_kernel(float *__restrict__ x, int64_t n) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) x[i] = gelu_tanh_f16(x[i]);
}

__global__ void add_inplace_kernel(float *__restrict__ y, const float *__restrict__ x, int64_t n) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) y[i] = __fadd_rn(y[i], x[i]);
}

// 2x2 max pool of the q part (columns [0, C)) of qkv rows [Bw][wh][ww] (row stride
// ld) -> qp [Bw][wh/2][ww/2][C] (sam2_maxpool_2d on q, sam3.cpp:4371-4381).
__global__ void qpool_kernel(const float *__restrict__ qkv, int64_t ld, int Bw, int ww, int wh, int C,
                             float *__restrict__ qp) {
    const int pw = ww / 2, ph = wh / 2;
    const int64_t total = static_cast<int64_t>(Bw) * pw * ph * C;
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= total) return;
    const int c = static_cast<int>(i % C);
    const int64_t t = i / C;
    const int px = static_cast<int>(t % pw), py = static_cast<int>((t / pw) % ph), w = static_cast<int>(t / (pw * ph));
    const int64_t n0 = static_cast<int64_t>(w) * ww * wh + static_cast<int64_t>(2 * py) * ww + 2 * px;
    const float a = qkv[n0 * ld + c], b = qkv[(n0 + 1) * ld + c];
    const float d = qkv[(n0 + ww) * ld + c], e = qkv[(n0 + ww + 1) * ld + c];
    qp[i] = fmaxf(fmaxf(a, b), fmaxf(d, e));
}

// 2x2 max pool of a token-major map [H][W][C] -> [H/2][W/2][C] (sam2_maxpool_2d)
__global__ void maxpool2_f32_kernel(const float *__restrict__ x, int H, int W, int C, float *__restrict__ y) {
    const int W2 = W / 2, H2 = H / 2;
    const int64_t total = static_cast<int64_t>(H2) * W2 * C;
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= total) return;
    const int c = static_cast<int>(i % C);
    const int64_t t = i / C;
    const int xx = static_cast<int>(t % W2), yy = static_cast<int>(t / W2);
    const int64_t r0 = (static_cast<int64_t>(2 * yy) * W + 2 * xx) * C + c;
    y[i] = fmaxf(fmaxf(x[r0], x[r0 + C]), fmaxf(x[r0 + static_cast<int64_t>(W) * C], x[r0 + static_cast<int64_t>(W) * C + C]));
}

// x_out[t] = shortcut[t] + proj[row(t)] over the H x W output map: the window
// unpartition (with crop) of sam3.cpp:4243-4281 fused with the residual add
// (:4426).  ws == 0: proj is already in token order.
__global__ void unpart_add_kernel(const float *__restrict__ sc, const float *__restrict__ proj, int H, int W, int C,
                                  int ws, int nWh, float *__restrict__ out) {
    const int64_t total = static_cast<int64_t>(H) * W * C;
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= total) return;
    const int c = static_cast<int>(i % C);
    const int64_t t = i / C;
    int64_t r = t;
    if (ws > 0) {
        const int x = static_cast<int>(t % W), y = static_cast<int>(t / W);
        r = static_cast<int64_t>(y / ws + nWh * (x / ws)) * ws * ws + x % ws + ws * (y % ws);
    }
    out[i] = __fadd_rn(sc[i], proj[r * C + c]);
}

// FPN top-down fusion: y[t] = lat[t] + prev[nearest 2x source of t] (sam3.cpp:4568-4573)
__global__ void upsample2_add_kernel(const float *lat, const float *__restrict__ prev, int H, int W, int D,
                                     float *y) {  // y may alias lat
    const int64_t total = static_cast<int64_t>(H) * W * D;
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= total) return;
    const int d = static_cast<int>(i % D);
    const int64_t t = i / D;
    const int x = static_cast<int>(t % W), yy = static_cast<int>(t / W);
    y[i] = __fadd_rn(lat[i], prev[(static_cast<int64_t>(yy / 2) * (W / 2) + x / 2) * D + d]);
}

inline unsigned blocks_for(int64_t n, int per) { return static_cast<unsigned>((n + per - 1) / per); }
inline int round128(int64_t n) { return static_cast<int>((n + 127) / 128 * 128); }

// Bicubic resize of a CHW map (Keys kernel, a = -0.75, half-pixel centres,
// clamped taps): the host-side positional-embedding precompute of
// sam3.cpp:4076-4108, restated.
void bicubic_chw(const std::vector<float> &src, int C, int hi, int wi, std::vector<float> &dst, int ho, int wo) {
    auto cubic = [](float x) -> float {
        x = fabsf(x);
        if (x < 1.0f) return (1.25f * x - 2.25f) * x * x + 1.0f;
        if (x < 2.0f) return ((-0.75f * x + 3.75f) * x - 6.0f) * x + 3.0f;
        return 0.0f;
    };
    dst.assign(static_cast<size_t>(C) * ho * wo, 0.f);
    for (int c = 0; c < C; ++c)
        for (int y = 0; y < ho; ++y) {
            const float fy = (static_cast<float>(y) + 0.5f) * static_cast<float>(hi) / static_cast<float>(ho) - 0.5f;
            const int iy = static_cast<int>(floorf(fy));
            const float dy = fy - static_cast<float>(iy);
            for (int x = 0; x < wo; ++x) {
                const float fx = (static_cast<float>(x) + 0.5f) * static_cast<float>(wi) / static_cast<float>(wo) - 0.5f;
                const int ix = static_cast<int>(floorf(fx));
                const float dx = fx - static_cast<float>(ix);
                float val = 0.0f;
                for (int jj = -1; jj <= 2; ++jj) {
                    const float wy = cubic(dy - static_cast<float>(jj));
                    const int sy = std::min(std::max(iy + jj, 0), hi - 1);
                    for (int ii = -1; ii <= 2; ++ii) {
                        const float wx = cubic(dx - static_cast<float>(ii));
                        const int sx = std::min(std::max(ix + ii, 0), wi - 1);
                        val += wy * wx * src[(static_cast<size_t>(c) * hi + sy) * wi + sx];
                    }
                }
                dst[(static_cast<size_t>(c) * ho + y) * wo + x] = val;
            }
        }
}

// A linear layer of a block: Q8_0 / Q4_0 weights on the int8 tensor-core MUL_MAT, or F16 / F32 ones
// (a file whose row length is no multiple of 32 keeps those tensors F16, as ggml's quantiser does;
// F16 files throughout) on the fp16 tensor-core GEMM with the activations rounded to fp16 -- ggml-cpu's
// vec_dot_f16 arithmetic.
struct HLinear {
    QWeight q;
    sam3b200_weight *dense = nullptr;
    bool set() const { return q.set || dense != nullptr; }
};

struct HBlock {
    int dim_in = 0, dim_out = 0, heads = 0, ws = 0, stage = 0;
    bool q_stride = false;
    DevBuf n1w, n1b, n2w, n2b, qkv_b, proj_b, fc1_b, fc2_b, dproj_b;
    HLinear qkv, proj, fc1, fc2, dproj;
};

struct FpnLevel {
    DevBuf w16, b;  // fp16 [D][C], f32 [D]
    int C = 0;
};

}  // namespace

struct Hiera {
    Backend *be = nullptr;
    sam3b200_hiera_hparams hp{};
    int S = 0;  // patch grid side
    int stage_ends[4] = {0, 0, 0, 0};
    std::vector<HBlock> blk;
    DevBuf patch_w32, patch_b, pe;  // f32 kernel [E][3*7*7]
    std::vector<float> pos_bkg, pos_win;  // host copies until both are set
    FpnLevel fpn[4];
    std::vector<std::string> missing;
    // activations
    DevBuf xa, xb, normed, shortf, shortp, qkv, qp, attn, proj, codes_a, quads_a, codes_b, quads_b;
    DevBuf a16, b16;  // DQ16 arithmetic: codes_a / codes_b dequantised to fp16
    DevBuf stage_out[4], fpn_out[4], x16;
    DevBuf tq, tk, tvt;          // attention operands for the tensor cores (attn_tcw): fp16 q, k, v^T
    DevBuf xwin, hid;            // blocks with F16 / F32 linear layers: f32 windowed rows, MLP hidden rows
    DevBuf col;                  // the patch embedding's f32 im2col rows
    ~Hiera() {
        for (auto &b : blk)
            for (HLinear *l : {&b.qkv, &b.proj, &b.fc1, &b.fc2, &b.dproj})
                if (l->dense) sam3b200_weight_free(reinterpret_cast<sam3b200_backend *>(be), l->dense);
    }
    int stage_side[4] = {0, 0, 0, 0}, stage_dim[4] = {0, 0, 0, 0};
    int n_fpn = 0;
    bool ready = false;
};

namespace {

bool hlaunched(Hiera *h, cudaError_t e, const char *what, int n = 1) {
    h->be->count(n);
    return cuda_ok(e, what);
}

bool h_mmq(Hiera *h, const void *codes, const void *quads, int M, const QWeight &w, int mode, const float *bias,
           float *y, int add, void *oc, void *oq, int gelu) {
    MmqArgs a;
    const int ld = round128(M);
    a.a = QMatrix{codes, quads, M, w.K, ld};
    a.b = QMatrix{w.codes.p, w.quads.p, w.N, w.K, w.ld, w.nib};
    a.bias = bias;
    a.y = y;
    a.ldy = w.N;
    a.dump = nullptr;
    a.err = h->be->err;
    a.add = add;
    a.gelu = gelu;
    a.out_codes = oc;
    a.out_quads = oq;
    a.out_ld = ld;
    if (h->be->mmq_arith == SAM3B200_ARITH_DQ16 && w.w16.p) {
        // DQ16 arithmetic (mmq.cuh): the same Q8_0 codes, dequantised, on the fp16 tensor cores
        void *a16 = codes == h->codes_b.p ? h->b16.p : h->a16.p;
        if (!hlaunched(h, dequant_act_f16(codes, quads, M, w.K, ld, a16, h->be->stream), "hiera dequant")) return false;
        h->be->prof_mark(0);
        const bool ok = hlaunched(h, mmq_dq16(a, a16, w.w16.p, mode, h->be->num_sms, h->be->stream), "hiera mmq dq16");
        h->be->prof_mark(0);
        return ok;
    }
    h->be->prof_mark(0);
    const bool ok = hlaunched(h, mmq_tc(a, mode, h->be->num_sms, h->be->stream, h->be->mmq_cvt, h->be->mmq_bn), "hiera mmq");
    h->be->prof_mark(0);
    return ok;
}

// y = x W^T + bias for an F16 / F32 weight: x f32 rows (ld = K), y rows of N
bool h_dense(Hiera *h, const float *x, int M, const HLinear &w, const float *bias, float *y) {
    const auto *wt = reinterpret_cast<const Weight *>(w.dense);
    return run_mul_mat(h->be, wt, x, wt->K, M, bias, y, wt->N, nullptr) == SAM3B200_STATUS_SUCCESS;
}

// a linear layer on f32 input rows, either kind of weight (f32 out, optionally added to y); a quantised
// weight takes its activation codes in the `wide` (MLP hidden, codes_b / quads_b: To x 4 Co) or the
// narrow (codes_a / quads_a) scratch
bool h_linear(Hiera *h, const float *x, int M, int K, const HLinear &w, const float *bias, float *y, int add,
              float *tmp, bool wide = false) {
    cudaStream_t s = h->be->stream;
    if (w.dense) {
        if (!add) return h_dense(h, x, M, w, bias, y);
        const auto *wt = reinterpret_cast<const Weight *>(w.dense);
        const int64_t n = static_cast<int64_t>(M) * wt->N;
        if (!h_dense(h, x, M, w, bias, tmp)) return false;
        add_inplace_kernel<<<blocks_for(n, 256), 256, 0, s>>>(y, tmp, n);
        return hlaunched(h, cudaGetLastError(), "hiera residual");
    }
    void *codes = wide ? h->codes_b.p : h->codes_a.p, *quads = wide ? h->quads_b.p : h->quads_a.p;
    return hlaunched(h, quantize_rows_q8(x, K, M, K, codes, quads, round128(M), s), "hiera quantize") &&
           h_mmq(h, codes, quads, M, w.q, MMQ_OUT_F32, bias, y, add, nullptr, nullptr, 0);
}

bool ensure_buf(DevBuf &b, size_t bytes) { return b.n >= bytes || b.alloc(bytes); }

// Derive the per-block metadata exactly as sam2_precompute_hiera_metadata (sam3.cpp:1680-1740).
bool hiera_metadata(Hiera *h) {
    const auto &hp = h->hp;
    int total = 0;
    for (int s = 0; s < 4; ++s) {
        if (hp.stages[s] <= 0) return false;
        total += hp.stages[s];
        h->stage_ends[s] = total - 1;
    }
    std::vector<int> qpool;
    for (int s = 0; s < 3 && static_cast<int>(qpool.size()) < hp.q_pool; ++s) qpool.push_back(h->stage_ends[s] + 1);
    h->blk.resize(total);
    int cur = 0, embed = hp.embed, nh = hp.heads;
    for (int i = 0; i < total; ++i) {
        HBlock &b = h->blk[i];
        int ws = hp.window_spec[cur];
        for (int g = 0; g < hp.n_global && g < 8; ++g)
            if (hp.global_idx[g] == i) ws = 0;
        b.ws = ws;
        int dout = embed;
        if (i > 0 && i - 1 == h->stage_ends[cur]) {
            dout = embed * 2;
            nh *= 2;
            ++cur;
        }
        b.stage = cur;
        b.dim_in = embed;
        b.dim_out = dout;
        b.heads = nh;
        b.q_stride = false;
        for (int qb : qpool)
            if (qb == i) b.q_stride = true;
        embed = dout;
        // fp16 GEMM rows need 8 | dim (a Q8_0 / Q4_0 weight further needs 32 | its row length, checked
        // when it is set)
        if (b.dim_in % 8 != 0 || b.dim_out % 8 != 0 || b.dim_out % b.heads != 0) return false;
    }
    return true;
}

struct BlockGeo {
    int H, W, Ho, Wo, ws, nWh, Bw, N, wq_w, wq_h, NQ, ws_o, nWh_o;
};

BlockGeo block_geo(const HBlock &b, int H, int W) {
    BlockGeo g{};
    g.H = H;
    g.W = W;
    g.Ho = b.q_stride ? H / 2 : H;
    g.Wo = b.q_stride ? W / 2 : W;
    g.ws = b.ws;
    if (b.ws > 0) {
        const int Hp = (H + b.ws - 1) / b.ws * b.ws, Wp = (W + b.ws - 1) / b.ws * b.ws;
        g.nWh = Hp / b.ws;
        g.Bw = g.nWh * (Wp / b.ws);
        g.N = b.ws * b.ws;
        g.wq_w = g.wq_h = b.ws;
    } else {
        g.nWh = 1;
        g.Bw = 1;
        g.N = H * W;
        g.wq_w = W;
        g.wq_h = H;
    }
    g.NQ = b.q_stride ? (g.wq_w / 2) * (g.wq_h / 2) : g.N;
    if (b.ws > 0) {
        g.ws_o = b.q_stride ? b.ws / 2 : b.ws;
        const int pad = (g.ws_o - g.Ho % g.ws_o) % g.ws_o;  // sam3.cpp:4409-4414
        g.nWh_o = (g.Ho + pad) / g.ws_o;
    } else {
        g.ws_o = 0;
        g.nWh_o = 1;
    }
    return g;
}

// Windowed and global attention run on the tcgen05 kernel (attn_tcw) for head
// dimensions up to 128 -- every SAM2 Hiera (56 / 72 / 96) -- and on the SIMT
// flash loop otherwise.
bool attn_on_tensor_cores(const HBlock &b) { return b.dim_out / b.heads <= 128; }

bool alloc_hiera(Hiera *h) {
    const auto &hp = h->hp;
    const int S = h->S;
    size_t mx_x = 0, mx_norm = 0, mx_sf = 0, mx_sp = 0, mx_qkv = 0, mx_qp = 0, mx_codes_a = 0, mx_quads_a = 0,
           mx_codes_b = 0, mx_quads_b = 0;
    size_t mx_tq = 0, mx_tkv = 0;
    int H = S, W = S;
    for (size_t i = 0; i < h->blk.size(); ++i) {
        const HBlock &b = h->blk[i];
        const BlockGeo g = block_geo(b, H, W);
        if (attn_on_tensor_cores(b)) {
            const int hd = b.dim_out / b.heads;
            mx_tq = std::max(mx_tq, attn_tcw_q_elems(g.Bw, g.NQ, b.heads, hd));
            mx_tkv = std::max(mx_tkv, attn_tcw_kv_elems(g.Bw, g.N, b.heads, hd));
        }
        const size_t T = static_cast<size_t>(H) * W, To = static_cast<size_t>(g.Ho) * g.Wo;
        const size_t rw = static_cast<size_t>(g.Bw) * g.N, rq = static_cast<size_t>(g.Bw) * g.NQ;
        mx_x = std::max({mx_x, T * b.dim_in, To * b.dim_out});
        mx_norm = std::max(mx_norm, T * b.dim_in);
        mx_sf = std::max(mx_sf, T * b.dim_out);
        mx_sp = std::max(mx_sp, To * b.dim_out);
        mx_qkv = std::max(mx_qkv, rw * 3 * b.dim_out);
        mx_qp = std::max(mx_qp, rq * b.dim_out);
        mx_codes_a = std::max({mx_codes_a, rw * b.dim_in, T * b.dim_in, rq * b.dim_out, To * b.dim_out});
        const size_t ga = static_cast<size_t>((std::max(b.dim_in, b.dim_out) + 255) / 256);
        mx_quads_a = std::max({mx_quads_a, ga * round128(static_cast<int64_t>(std::max({rw, T, rq, To}))) * 16});
        mx_codes_b = std::max(mx_codes_b, To * 4 * b.dim_out);
        mx_quads_b = std::max(mx_quads_b, static_cast<size_t>((4 * b.dim_out + 255) / 256) * round128(To) * 16);
        H = g.Ho;
        W = g.Wo;
        if (static_cast<int>(i) == h->stage_ends[b.stage]) {
            h->stage_side[b.stage] = H;
            h->stage_dim[b.stage] = b.dim_out;
        }
    }
    bool ok = h->xa.alloc(mx_x * 4) &&
              h->xb.alloc(mx_x * 4) && h->normed.alloc(mx_norm * 4) && h->shortf.alloc(mx_sf * 4) &&
              h->shortp.alloc(mx_sp * 4) && h->qkv.alloc(mx_qkv * 4) && h->qp.alloc(mx_qp * 4) &&
              h->attn.alloc(mx_qp * 4) && h->proj.alloc(mx_qp * 4) && h->codes_a.alloc(mx_codes_a) &&
              h->quads_a.alloc(mx_quads_a) && h->codes_b.alloc(mx_codes_b) && h->quads_b.alloc(mx_quads_b) &&
              h->a16.alloc(mx_codes_a * 2) && h->b16.alloc(mx_codes_b * 2);
    size_t mx16 = 0;
    for (int s = 0; s < 4 && ok; ++s) {
        const size_t T = static_cast<size_t>(h->stage_side[s]) * h->stage_side[s];
        ok = h->stage_out[s].alloc(T * h->stage_dim[s] * 4) && h->fpn_out[s].alloc(T * hp.neck_dim * 4);
        mx16 = std::max(mx16, T * h->stage_dim[s] * 2);
    }
    ok = ok && h->x16.alloc(mx16);
    if (ok && mx_tq > 0) ok = h->tq.alloc(mx_tq * 2) && h->tk.alloc(mx_tkv * 2) && h->tvt.alloc(mx_tkv * 2);
    if (!ok) return false;
    return cuda_ok(cudaMemsetAsync(h->quads_a.p, 0, h->quads_a.n, h->be->stream), "memset") &&
           cuda_ok(cudaMemsetAsync(h->quads_b.p, 0, h->quads_b.n, h->be->stream), "memset") &&
           cuda_ok(cudaStreamSynchronize(h->be->stream), "alloc sync");
}

bool make_pe(Hiera *h) {
    const auto &hp = h->hp;
    const int E = hp.embed, S = h->S, ws = hp.window_spec[0];
    std::vector<float> bk;
    bicubic_chw(h->pos_bkg, E, hp.bkg_h, hp.bkg_w, bk, S, S);
    std::vector<float> pe(static_cast<size_t>(E) * S * S);
    for (int e = 0; e < E; ++e)
        for (int y = 0; y < S; ++y)
            for (int x = 0; x < S; ++x)
                pe[static_cast<size_t>(e) + static_cast<size_t>(x) * E + static_cast<size_t>(y) * E * S] =
                    bk[(static_cast<size_t>(e) * S + y) * S + x] +
                    h->pos_win[(static_cast<size_t>(e) * ws + (y % ws)) * ws + (x % ws)];
    return upload(h->pe, pe.data(), pe.size() * 4, h->be->stream);
}

bool run_prefix(Hiera *h, const float *img_chw, float *x) {
    const auto &hp = h->hp;
    const int S = h->S, E = hp.embed;
    cudaStream_t s = h->be->stream;
    // f32 im2col [S*S][3*7*7] and an f32 GEMM with the kernel [E][147] (ggml_conv_2d with an F32
    // kernel), then + bias and + the positional embedding in that order
    const int64_t P = static_cast<int64_t>(S) * S, n = P * E;
    if (!ensure_buf(h->col, static_cast<size_t>(P) * 147 * 4)) return false;
    if (!hlaunched(h, im2col_chw(img_chw, 3, hp.img, hp.img, 7, 4, 3, S, S, h->col.as<float>(), s), "hiera patch im2col") ||
        !hlaunched(h, sgemm_nt(h->col.as<float>(), 147, 1, h->patch_w32.as<float>(), 147, 1, static_cast<int>(P), E, 147,
                               h->patch_b.as<float>(), x, E, false, s),
                   "hiera patch gemm"))
        return false;
    add_inplace_kernel<<<blocks_for(n, 256), 256, 0, s>>>(x, h->pe.as<float>(), n);
    return hlaunched(h, cudaGetLastError(), "hiera patch embedding");
}

bool run_block(Hiera *h, int i, const float *x, int H, int W, float *out) {
    const HBlock &b = h->blk[i];
    const BlockGeo g = block_geo(b, H, W);
    cudaStream_t s = h->be->stream;
    const int Ci = b.dim_in, Co = b.dim_out, T = H * W, To = g.Ho * g.Wo;
    const int rw = g.Bw * g.N, rq = g.Bw * g.NQ;
    if (g.ws_o > 0 && static_cast<int64_t>((g.Wo + g.ws_o - 1) / g.ws_o) * g.nWh_o * g.ws_o * g.ws_o > rq) {
        set_error("hiera block %d: the output windows do not match the partition (%dx%d, window %d)", i, H, W, b.ws);
        return false;
    }
    // 1. LN1
    ln_rows_kernel<<<blocks_for(T, 8), 256, 0, s>>>(x, T, Ci, b.n1w.as<float>(), b.n1b.as<float>(), 1e-6f,
                                                    h->normed.as<float>());
    if (!hlaunched(h, cudaGetLastError(), "hiera ln1")) return false;
    // 2. shortcut
    const float *sc = x;
    if (Ci != Co) {
        if (!h_linear(h, h->normed.as<float>(), T, Ci, b.dproj, b.dproj_b.as<float>(), h->shortf.as<float>(), 0,
                      nullptr))
            return false;
        sc = h->shortf.as<float>();
    }
    if (b.q_stride) {
        maxpool2_f32_kernel<<<blocks_for(static_cast<int64_t>(To) * Co, 256), 256, 0, s>>>(sc, H, W, Co,
                                                                                            h->shortp.as<float>());
        if (!hlaunched(h, cudaGetLastError(), "hiera pool shortcut")) return false;
        sc = h->shortp.as<float>();
    }
    // 3. qkv over the window-partitioned normed input
    if (b.qkv.dense) {
        const float *xin = h->normed.as<float>();
        if (b.ws > 0) {
            if (!ensure_buf(h->xwin, static_cast<size_t>(rw) * Ci * 4)) return false;
            win_gather_f32_kernel<<<blocks_for(static_cast<int64_t>(rw) * Ci, 256), 256, 0, s>>>(
                h->normed.as<float>(), H, W, Ci, b.ws, g.nWh, rw, h->xwin.as<float>());
            if (!hlaunched(h, cudaGetLastError(), "hiera qkv windows")) return false;
            xin = h->xwin.as<float>();
        }
        if (!h_dense(h, xin, rw, b.qkv, b.qkv_b.as<float>(), h->qkv.as<float>())) return false;
    } else {
        cudaError_t e;
        if (b.ws > 0) {
            win_gather_q8_kernel<<<blocks_for(rw, 8), 256, 0, s>>>(h->normed.as<float>(), H, W, Ci, b.ws, g.nWh, rw,
                                                                   h->codes_a.as<int8_t>(), h->quads_a.as<__half>(),
                                                                   round128(rw));
            e = cudaGetLastError();
        } else {
            e = quantize_rows_q8(h->normed.as<float>(), Ci, T, Ci, h->codes_a.p, h->quads_a.p, round128(T), s);
        }
        if (!hlaunched(h, e, "hiera qkv input") ||
            !h_mmq(h, h->codes_a.p, h->quads_a.p, rw, b.qkv.q, MMQ_OUT_F32, b.qkv_b.as<float>(), h->qkv.as<float>(), 0,
                   nullptr, nullptr, 0))
            return false;
    }
    // 4. Q pooling inside the windows
    const float *qptr = h->qkv.as<float>();
    int64_t q_ld = 3 * Co;
    if (b.q_stride) {
        qpool_kernel<<<blocks_for(static_cast<int64_t>(rq) * Co, 256), 256, 0, s>>>(h->qkv.as<float>(), 3 * Co, g.Bw,
                                                                                    g.wq_w, g.wq_h, Co,
                                                                                    h->qp.as<float>());
        if (!hlaunched(h, cudaGetLastError(), "hiera qpool")) return false;
        qptr = h->qp.as<float>();
        q_ld = Co;
    }
    // 5. attention per (window, head)
    const int hd = Co / b.heads;
    const float scale = 1.0f / sqrtf(static_cast<float>(hd));
    if (attn_on_tensor_cores(b)) {
        const float *kv = h->qkv.as<float>();
        if (!hlaunched(h,
                       attn_tcw_stage(qptr, q_ld, kv + Co, kv + 2 * Co, 3 * Co, g.Bw, g.NQ, g.N, b.heads, hd,
                                      h->tq.as<__half>(), h->tk.as<__half>(), h->tvt.as<__half>(), s),
                       "hiera attention staging", 3) ||
            !hlaunched(h,
                       attn_tcw(h->tq.as<__half>(), h->tk.as<__half>(), h->tvt.as<__half>(), g.Bw, g.NQ, g.N,
                                b.heads, hd, scale, h->attn.as<float>(), Co, h->be->err, s),
                       "hiera attention"))
            return false;
    } else {
        const AttnStrides qs{static_cast<int64_t>(g.NQ) * q_ld, hd, q_ld};
        const AttnStrides kvs{static_cast<int64_t>(g.N) * 3 * Co, hd, 3 * Co};
        const AttnStrides os{static_cast<int64_t>(g.NQ) * Co, hd, Co};
        if (!hlaunched(h,
                       attention_simt(hd, qptr, qs, g.NQ, h->qkv.as<float>() + Co, kvs, h->qkv.as<float>() + 2 * Co, kvs,
                                      g.N, g.Bw, b.heads, nullptr, 0, scale, h->attn.as<float>(), os, s),
                       "hiera attention"))
            return false;
    }
    // 6. output projection
    if (!h_linear(h, h->attn.as<float>(), rq, Co, b.proj, b.proj_b.as<float>(), h->proj.as<float>(), 0, nullptr))
        return false;
    // 7. unpartition + crop + residual
    unpart_add_kernel<<<blocks_for(static_cast<int64_t>(To) * Co, 256), 256, 0, s>>>(sc, h->proj.as<float>(), g.Ho, g.Wo,
                                                                                     Co, g.ws_o, g.nWh_o, out);
    if (!hlaunched(h, cudaGetLastError(), "hiera unpartition")) return false;
    // 8. MLP: LN2 -> fc1 + GELU (tanh, fp16 table) -> Q8 -> fc2 + bias, residual
    if (!b.fc1.dense && !b.fc2.dense)
        return hlaunched(h,
                         layernorm_q8(out, To, Co, b.n2w.as<float>(), b.n2b.as<float>(), 1e-6f, g.Wo, 0, h->codes_a.p,
                                      h->quads_a.p, round128(To), s),
                         "hiera ln2") &&
               h_mmq(h, h->codes_a.p, h->quads_a.p, To, b.fc1.q, MMQ_OUT_Q8, b.fc1_b.as<float>(), nullptr, 0,
                     h->codes_b.p, h->quads_b.p, 2) &&
               h_mmq(h, h->codes_b.p, h->quads_b.p, To, b.fc2.q, MMQ_OUT_F32, b.fc2_b.as<float>(), out, 1, nullptr,
                     nullptr, 0);
    // a block with an F16 / F32 MLP weight: the same steps on f32 rows
    const int64_t nh = static_cast<int64_t>(To) * 4 * Co;
    if (!ensure_buf(h->hid, static_cast<size_t>(nh) * 4)) return false;
    ln_rows_kernel<<<blocks_for(To, 8), 256, 0, s>>>(out, To, Co, b.n2w.as<float>(), b.n2b.as<float>(), 1e-6f,
                                                     h->normed.as<float>());
    if (!hlaunched(h, cudaGetLastError(), "hiera ln2") ||
        !h_linear(h, h->normed.as<float>(), To, Co, b.fc1, b.fc1_b.as<float>(), h->hid.as<float>(), 0, nullptr))
        return false;
    gelu_tanh_inplace_kernel<<<blocks_for(nh, 256), 256, 0, s>>>(h->hid.as<float>(), nh);
    return hlaunched(h, cudaGetLastError(), "hiera gelu") &&
           h_linear(h, h->hid.as<float>(), To, 4 * Co, b.fc2, b.fc2_b.as<float>(), out, 1, h->shortf.as<float>(),
                    true);
}

bool run_fpn(Hiera *h) {
    const auto &hp = h->hp;
    cudaStream_t s = h->be->stream;
    const int D = hp.neck_dim;
    // laterals: convs[3 - i] on stage i (1x1 conv = fp16 GEMM + bias), token-major [T][D]
    for (int i = 0; i < 4; ++i) {
        const FpnLevel &L = h->fpn[3 - i];
        const int T = h->stage_side[i] * h->stage_side[i];
        if (!hlaunched(h, f32_to_f16(h->stage_out[i].as<float>(), static_cast<int64_t>(T) * L.C, h->x16.p, s),
                       "fpn f16"))
            return false;
        GemmF16Args g{};
        g.a = h->x16.p;
        g.b = L.w16.p;
        g.M = T;
        g.N = D;
        g.K = L.C;
        g.bias = L.b.as<float>();
        g.out = h->fpn_out[i].p;
        g.ldo = D;
        g.store = GEMM_STORE_ROWMAJOR;
        g.err = h->be->err;
        if (!hlaunched(h, gemm_f16(g, h->be->num_sms, s), "fpn lateral")) return false;
    }
    // top-down: from the coarsest level down; levels listed in fpn_top_down_levels add the
    // 2x nearest upsample of the previous fused level (sam3.cpp:4556-4578)
    int prev = -1;
    for (int ri = 0; ri < 4; ++ri) {
        const int i = 3 - ri;
        bool td = false;
        for (int j = 0; j < hp.fpn_top_down_n && j < 4; ++j)
            if (hp.fpn_top_down_levels[j] == i) td = true;
        if (td && prev >= 0) {
            const int side = h->stage_side[i];
            if (h->stage_side[prev] * 2 != side) {
                set_error("hiera fpn: level %d is not twice level %d", i, prev);
                return false;
            }
            const int64_t n = static_cast<int64_t>(side) * side * D;
            upsample2_add_kernel<<<blocks_for(n, 256), 256, 0, s>>>(h->fpn_out[i].as<float>(),
                                                                     h->fpn_out[prev].as<float>(), side, side, D,
                                                                     h->fpn_out[i].as<float>());
            if (!hlaunched(h, cudaGetLastError(), "fpn top-down")) return false;
            prev = i;
        } else if (td || prev < 0) {
            prev = i;
        }
    }
    return true;
}

bool encode(Hiera *h, const float *img_chw) {
    float *x = h->xa.as<float>(), *y = h->xb.as<float>();
    if (!run_prefix(h, img_chw, x)) return false;
    int H = h->S, W = h->S;
    for (size_t i = 0; i < h->blk.size(); ++i) {
        const HBlock &b = h->blk[i];
        float *dst = b.q_stride ? y : x;  // shape changes need a second buffer
        if (!run_block(h, static_cast<int>(i), x, H, W, dst)) return false;
        if (b.q_stride) std::swap(x, y);
        if (b.q_stride) {
            H /= 2;
            W /= 2;
        }
        if (static_cast<int>(i) == h->stage_ends[b.stage]) {
            const size_t bytes = static_cast<size_t>(H) * W * b.dim_out * 4;
            if (!cuda_ok(cudaMemcpyAsync(h->stage_out[b.stage].p, x, bytes, cudaMemcpyDeviceToDevice, h->be->stream),
                         "stage copy"))
                return false;
        }
    }
    return run_fpn(h);
}

bool check_ready(Hiera *h) {
    if (h->ready) return true;
    h->missing.clear();
    if (!h->patch_w32.p) h->missing.push_back("hiera.patch_embed.weight");
    if (!h->patch_b.p) h->missing.push_back("hiera.patch_embed.bias");
    if (!h->pe.p) h->missing.push_back("hiera.pos_embed / hiera.pos_embed_window");
    for (size_t i = 0; i < h->blk.size(); ++i) {
        const HBlock &b = h->blk[i];
        const std::string p = "hiera.blocks." + std::to_string(i);
        if (!b.n1w.p || !b.n1b.p || !b.n2w.p || !b.n2b.p) h->missing.push_back(p + ".norm1/norm2");
        if (!b.qkv.set() || !b.qkv_b.p) h->missing.push_back(p + ".attn.qkv");
        if (!b.proj.set() || !b.proj_b.p) h->missing.push_back(p + ".attn.proj");
        if (!b.fc1.set() || !b.fc1_b.p || !b.fc2.set() || !b.fc2_b.p) h->missing.push_back(p + ".mlp");
        if (b.dim_in != b.dim_out && (!b.dproj.set() || !b.dproj_b.p)) h->missing.push_back(p + ".proj");
    }
    for (int j = 0; j < 4; ++j)
        if (!h->fpn[j].w16.p || !h->fpn[j].b.p) h->missing.push_back("fpn.convs." + std::to_string(j));
    if (!h->missing.empty()) {
        set_error("hiera: %zu tensors missing (first: %s)", h->missing.size(), h->missing[0].c_str());
        return false;
    }
    h->ready = true;
    return true;
}

}  // namespace
}  // namespace b200

using namespace b200;

sam3b200_hiera *sam3b200_hiera_create(sam3b200_backend *hb, const sam3b200_hiera_hparams *hp) {
    auto *be = reinterpret_cast<Backend *>(hb);
    if (!be || !hp) return nullptr;
    if (hp->img <= 0 || hp->img % 32 != 0 || hp->embed <= 0 || hp->embed % 8 != 0 || hp->heads <= 0 ||
        hp->neck_dim <= 0 || hp->neck_dim % 8 != 0 || hp->window_spec[0] <= 0 || hp->bkg_h <= 0 || hp->bkg_w <= 0 ||
        hp->scalp < 0 || hp->scalp > 3) {
        set_error("hiera_create: unsupported hyperparameters");
        return nullptr;
    }
    cudaSetDevice(be->device);
    auto *h = new Hiera();
    h->be = be;
    h->hp = *hp;
    h->S = (hp->img + 2 * 3 - 7) / 4 + 1;
    if (!hiera_metadata(h)) {
        set_error("hiera_create: block dimensions must be multiples of 8 and divisible by the head count");
        delete h;
        return nullptr;
    }
    h->n_fpn = 4 - hp->scalp;
    if (!alloc_hiera(h)) {
        delete h;
        return nullptr;
    }
    return reinterpret_cast<sam3b200_hiera *>(h);
}

void sam3b200_hiera_free(sam3b200_hiera *hh) {
    auto *h = reinterpret_cast<Hiera *>(hh);
    if (!h) return;
    cudaSetDevice(h->be->device);
    cudaStreamSynchronize(h->be->stream);
    delete h;
}

int sam3b200_hiera_block_info(sam3b200_hiera *hh, int i, int32_t info[5]) {
    auto *h = reinterpret_cast<Hiera *>(hh);
    if (!h || !info || i < 0 || i >= static_cast<int>(h->blk.size())) return SAM3B200_STATUS_FAILED;
    const HBlock &b = h->blk[i];
    info[0] = b.dim_in;
    info[1] = b.dim_out;
    info[2] = b.heads;
    info[3] = b.ws;
    info[4] = b.q_stride ? 1 : 0;
    return SAM3B200_STATUS_SUCCESS;
}

int sam3b200_hiera_set_tensor(sam3b200_hiera *hh, const char *name_c, int type, const void *data, const int64_t *ne) {
    auto *h = reinterpret_cast<Hiera *>(hh);
    if (!h || !name_c || !data || !ne) return SAM3B200_STATUS_FAILED;
    cudaSetDevice(h->be->device);
    const std::string name(name_c);
    const auto &hp = h->hp;
    cudaStream_t s = h->be->stream;
    const int64_t n = ne[0] * (ne[1] > 0 ? ne[1] : 1) * (ne[2] > 0 ? ne[2] : 1) * (ne[3] > 0 ? ne[3] : 1);
    std::vector<float> f;
    auto vec = [&](DevBuf &d, int64_t want) -> int {
        if (n != want) {
            set_error("%s: %lld elements, expected %lld", name_c, (long long)n, (long long)want);
            return SAM3B200_STATUS_FAILED;
        }
        if (!to_f32(type, data, n, f) || !upload(d, f.data(), f.size() * 4, s)) return SAM3B200_STATUS_FAILED;
        return SAM3B200_STATUS_SUCCESS;
    };
    h->ready = false;
    if (name == "hiera.patch_embed.weight") {  // [7, 7, 3, E]: memory [e][(ic, ky, kx)]
        if (ne[0] != 7 || ne[1] != 7 || ne[2] != 3 || ne[3] != hp.embed || !to_f32(type, data, n, f)) {
            set_error("%s: expected [7, 7, 3, %d] F32/F16", name_c, hp.embed);
            return SAM3B200_STATUS_FAILED;
        }
        return upload(h->patch_w32, f.data(), f.size() * 4, s) ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
    }
    if (name == "hiera.patch_embed.bias") return vec(h->patch_b, hp.embed);
    if (name == "hiera.pos_embed" || name == "hiera.pos_embed_window") {
        const bool bkg = name == "hiera.pos_embed";
        const int64_t want = bkg ? static_cast<int64_t>(hp.bkg_h) * hp.bkg_w * hp.embed
                                 : static_cast<int64_t>(hp.window_spec[0]) * hp.window_spec[0] * hp.embed;
        if (n != want || !to_f32(type, data, n, f)) {
            set_error("%s: %lld elements, expected %lld", name_c, (long long)n, (long long)want);
            return SAM3B200_STATUS_FAILED;
        }
        (bkg ? h->pos_bkg : h->pos_win) = f;
        if (!h->pos_bkg.empty() && !h->pos_win.empty() && !make_pe(h)) return SAM3B200_STATUS_FAILED;
        return SAM3B200_STATUS_SUCCESS;
    }
    if (name.rfind("fpn.convs.", 0) == 0) {
        const int j = atoi(name.c_str() + 10);
        if (j < 0 || j > 3) return SAM3B200_STATUS_FAILED;
        FpnLevel &L = h->fpn[j];
        const int C = h->stage_dim[3 - j];
        if (name.size() > 7 && name.compare(name.size() - 7, 7, ".weight") == 0) {
            if (n != static_cast<int64_t>(C) * hp.neck_dim || !to_f32(type, data, n, f)) {
                set_error("%s: expected [1, 1, %d, %d]", name_c, C, hp.neck_dim);
                return SAM3B200_STATUS_FAILED;
            }
            L.C = C;
            return upload_f16(L.w16, f, s) ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
        }
        return vec(L.b, hp.neck_dim);
    }
    if (name.rfind("hiera.blocks.", 0) == 0) {
        const int i = atoi(name.c_str() + 13);
        if (i < 0 || i >= static_cast<int>(h->blk.size())) return SAM3B200_STATUS_FAILED;
        HBlock &b = h->blk[i];
        const std::string p = "hiera.blocks." + std::to_string(i) + ".";
        const std::string r = name.substr(p.size());
        if (r == "norm1.weight") return vec(b.n1w, b.dim_in);
        if (r == "norm1.bias") return vec(b.n1b, b.dim_in);
        if (r == "norm2.weight") return vec(b.n2w, b.dim_out);
        if (r == "norm2.bias") return vec(b.n2b, b.dim_out);
        if (r == "attn.qkv.bias") return vec(b.qkv_b, 3 * b.dim_out);
        if (r == "attn.proj.bias") return vec(b.proj_b, b.dim_out);
        if (r == "mlp.fc1.bias") return vec(b.fc1_b, 4 * b.dim_out);
        if (r == "mlp.fc2.bias") return vec(b.fc2_b, b.dim_out);
        if (r == "proj.bias") return vec(b.dproj_b, b.dim_out);
        HLinear *w = nullptr;
        int64_t K = 0, N = 0;
        if (r == "attn.qkv.weight") w = &b.qkv, K = b.dim_in, N = 3 * b.dim_out;
        else if (r == "attn.proj.weight") w = &b.proj, K = b.dim_out, N = b.dim_out;
        else if (r == "mlp.fc1.weight") w = &b.fc1, K = b.dim_out, N = 4 * b.dim_out;
        else if (r == "mlp.fc2.weight") w = &b.fc2, K = 4 * b.dim_out, N = b.dim_out;
        else if (r == "proj.weight") w = &b.dproj, K = b.dim_in, N = b.dim_out;
        if (w) {
            if (ne[0] != K || ne[1] != N) {
                set_error("%s: shape [%lld, %lld], expected [%lld, %lld]", name_c, (long long)ne[0], (long long)ne[1],
                          (long long)K, (long long)N);
                return SAM3B200_STATUS_FAILED;
            }
            if (type == SAM3B200_TYPE_F16 || type == SAM3B200_TYPE_F32) {
                if (w->dense) sam3b200_weight_free(reinterpret_cast<sam3b200_backend *>(h->be), w->dense);
                w->dense = sam3b200_weight_upload(reinterpret_cast<sam3b200_backend *>(h->be), type, data, K, N);
                w->q.set = false;
                return w->dense ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
            }
            if (w->dense) {
                sam3b200_weight_free(reinterpret_cast<sam3b200_backend *>(h->be), w->dense);
                w->dense = nullptr;
            }
            return upload_qweight(h->be, w->q, type, data, K, N) && make_w16(h->be, w->q) ? SAM3B200_STATUS_SUCCESS
                                                                                          : SAM3B200_STATUS_FAILED;
        }
    }
    set_error("hiera: unknown tensor %s", name_c);
    return SAM3B200_STATUS_FAILED;
}

int sam3b200_hiera_missing(sam3b200_hiera *hh, char *buf, int cap) {
    auto *h = reinterpret_cast<Hiera *>(hh);
    if (!h) return -1;
    check_ready(h);
    std::string all;
    for (const auto &m : h->missing) all += m + "\n";
    if (buf && cap > 0) snprintf(buf, static_cast<size_t>(cap), "%s", all.c_str());
    return static_cast<int>(h->missing.size());
}

int sam3b200_hiera_run_prefix(sam3b200_hiera *hh, const float *img_chw_dev, float *x_dev) {
    auto *h = reinterpret_cast<Hiera *>(hh);
    if (!h || !img_chw_dev || !x_dev || !h->patch_w32.p || !h->patch_b.p || !h->pe.p) return SAM3B200_STATUS_FAILED;
    cudaSetDevice(h->be->device);
    return run_prefix(h, img_chw_dev, x_dev) ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
}

int sam3b200_hiera_run_block(sam3b200_hiera *hh, int i, const float *x_dev, int H, int W, float *out_dev) {
    auto *h = reinterpret_cast<Hiera *>(hh);
    if (!h || !x_dev || !out_dev || i < 0 || i >= static_cast<int>(h->blk.size()) || H <= 0 || W <= 0 ||
        (h->blk[i].q_stride && (H % 2 || W % 2)))
        return SAM3B200_STATUS_FAILED;
    // the activation buffers are sized for the model's own geometry
    int Hs = h->S;
    for (int j = 0; j < i; ++j)
        if (h->blk[j].q_stride) Hs /= 2;
    if (H * W > Hs * Hs) {
        set_error("hiera_run_block: %dx%d exceeds the %dx%d map of block %d", H, W, Hs, Hs, i);
        return SAM3B200_STATUS_FAILED;
    }
    cudaSetDevice(h->be->device);
    return run_block(h, i, x_dev, H, W, out_dev) ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
}

int sam3b200_hiera_encode_device(sam3b200_hiera *hh, const float *img_chw_dev) {
    auto *h = reinterpret_cast<Hiera *>(hh);
    if (!h || !img_chw_dev) return SAM3B200_STATUS_FAILED;
    cudaSetDevice(h->be->device);
    if (!check_ready(h)) return SAM3B200_STATUS_FAILED;
    return encode(h, img_chw_dev) ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
}

int sam3b200_hiera_output(sam3b200_hiera *hh, int i, const float **dev, int64_t *ne) {
    auto *h = reinterpret_cast<Hiera *>(hh);
    if (!h || !dev || !ne || i < 0 || i > 7) return SAM3B200_STATUS_FAILED;
    const int s = i & 3;
    if (i < 4 && s >= h->n_fpn) {
        *dev = nullptr;
        return SAM3B200_STATUS_FAILED;
    }
    *dev = i < 4 ? h->fpn_out[s].as<float>() : h->stage_out[s].as<float>();
    ne[0] = i < 4 ? h->hp.neck_dim : h->stage_dim[s];
    ne[1] = h->stage_side[s];
    ne[2] = h->stage_side[s];
    ne[3] = 1;
    return SAM3B200_STATUS_SUCCESS;
}
