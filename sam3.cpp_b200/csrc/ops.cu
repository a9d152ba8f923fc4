// ops.cu -- op-level entry points of the drop-in boundary besides MUL_MAT:
// the attention, the convolutions and the row gather that sam3.cpp's graphs
// dispatch to the backend.
//
//   GGML_OP_FLASH_ATTN_EXT     contiguous self-attention with head dim 64 and N
//                              a multiple of 8 on the tcgen05 kernel (attn.cu,
//                              bf16 operands); every other form -- head dims 16
//                              to 256, different query/key counts, strided views,
//                              an F16 mask -- on the fp32 loop of attn_simt.cu.
//   GGML_OP_CONV_TRANSPOSE_2D  ggml_conv_transpose_2d_p0 (sam3.cpp:3884,3887,
//                              3898, 10654, 10673): F16 kernel [KW,KH,OC,IC],
//                              F32 input [W,H,IC,1], no padding, any stride.
//   GGML_OP_CONV_2D            ggml_conv_2d / _sk_p0 / _s1_ph (sam3.cpp:3819,
//                              3889-3921, 4474, 11541): im2col + MUL_MAT in
//                              ggml; F16 kernel [KW,KH,IC,OC], F32 input.
//   GGML_OP_GET_ROWS           ggml_get_rows (the text encoder's token
//                              embedding lookup): F32 / F16 / Q4_0 / Q4_1 /
//                              Q8_0 rows -> F32.
//
// Both convolutions run as one fp16 tensor-core GEMM (gemm_f16.cu) between
// fp16 staging kernels.  ggml's CPU path rounds the F32 input to F16 as well
// (its im2col / permute buffers are F16 for an F16 kernel) and accumulates
// the F16 products in F32, so the results differ from it only in summation
// order.
//
//   conv_transpose_2d: cols[(oc, ky, kx)][p] = sum_ic W[ic][oc][ky][kx] * x[ic][p]
//                      (GEMM M = OC*KH*KW, N = IH*IW, K = IC padded to 8), then a
//                      gather: out[oc][oy][ox] = sum over the taps with
//                      oy = s*iy + ky, ox = s*ix + kx of cols.
//   conv_2d:           im2col[p][(ic, ky, kx)] (fp16, K padded to 8), then
//                      out[oc][p] = sum_k W[oc][k] * im2col[p][k] (GEMM M = OC,
//                      N = OH*OW) -- the output is ggml's [OW, OH, OC] layout.
#include "attn.cuh"
#include "attn_simt.cuh"
#include "backend_impl.h"
#include "gemm_f16.cuh"
#include "vit_ops.cuh"
#include "../../include/sam3_b200.h"
#include <cuda_fp16.h>

namespace b200 {
namespace {

constexpr int kOpErrGetRowsIndex = 1 << 20;  // get_rows: an index outside [0, nrows)

__host__ __device__ inline int64_t pad8(int64_t k) { return (k + 7) / 8 * 8; }

// out[r][k] = fp16(in[k][r]) for k < K, 0 for K <= k < Kp.  in: f32 or f16
// (ggml F16 bits) [K][R]; out: fp16 [R][Kp].  32x32 tiles through shared memory.
template <typename T>
__global__ void transpose_pad_f16_kernel(const T *__restrict__ in, int64_t R, int64_t K, int64_t Kp,
                                         __half *__restrict__ out) {
    __shared__ float tile[32][33];
    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * 32, k0 = static_cast<int64_t>(blockIdx.y) * 32;
    const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
    for (int j = ty; j < 32; j += 8) {
        const int64_t k = k0 + j, r = r0 + tx;
        float v = 0.f;
        if (k < K && r < R) {
            if constexpr (sizeof(T) == 4) v = static_cast<float>(in[k * R + r]);
            else v = __half2float(reinterpret_cast<const __half *>(in)[k * R + r]);
        }
        tile[j][tx] = v;
    }
    __syncthreads();
    for (int j = ty; j < 32; j += 8) {
        const int64_t r = r0 + j, k = k0 + tx;
        if (r < R && k < Kp) out[r * Kp + k] = __float2half_rn(tile[tx][j]);
    }
}

template <typename T>
cudaError_t transpose_pad_f16(const T *in, int64_t R, int64_t K, int64_t Kp, __half *out, cudaStream_t s) {
    dim3 grid(static_cast<unsigned>((R + 31) / 32), static_cast<unsigned>((Kp + 31) / 32));
    if (grid.y > 65535) return cudaErrorInvalidValue;
    transpose_pad_f16_kernel<T><<<grid, dim3(32, 8), 0, s>>>(in, R, K, Kp, out);
    return cudaGetLastError();
}

// Row copy with zero padding: out[r][k] = in[r][k] (k < K), 0 (K <= k < Kp); fp16 bits.
__global__ void pad_rows_f16_kernel(const uint16_t *__restrict__ in, int64_t R, int64_t K, int64_t Kp,
                                    uint16_t *__restrict__ out) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= R * Kp) return;
    const int64_t r = i / Kp, k = i % Kp;
    out[i] = k < K ? in[r * K + k] : uint16_t(0);
}

// conv_transpose_2d gather (no padding): out[oc][oy][ox], cols [(oc*KH+ky)*KW+kx][iy*IW+ix]
__global__ void convt_gather_kernel(const float *__restrict__ cols, int IW, int IH, int OC, int KW, int KH, int S,
                                    int OW, int OH, float *__restrict__ out) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t total = static_cast<int64_t>(OC) * OH * OW;
    if (i >= total) return;
    const int ox = static_cast<int>(i % OW);
    const int oy = static_cast<int>((i / OW) % OH);
    const int oc = static_cast<int>(i / (static_cast<int64_t>(OW) * OH));
    const int64_t P = static_cast<int64_t>(IW) * IH;
    float acc = 0.f;
    for (int ky = oy % S; ky < KH; ky += S) {
        const int iy = (oy - ky) / S;
        if (iy < 0) break;
        if (iy >= IH) continue;
        for (int kx = ox % S; kx < KW; kx += S) {
            const int ix = (ox - kx) / S;
            if (ix < 0) break;
            if (ix >= IW) continue;
            acc += cols[(static_cast<int64_t>(oc * KH + ky) * KW + kx) * P + static_cast<int64_t>(iy) * IW + ix];
        }
    }
    out[i] = acc;
}

// im2col in ggml's column order (ic, ky, kx), fp16, K padded to Kp with zeros.
// x f32 [IC][IH][IW]; out fp16 [OH*OW][Kp].
__global__ void im2col_f16_kernel(const float *__restrict__ x, int IW, int IH, int IC, int KW, int KH, int s0, int s1,
                                  int p0, int p1, int d0, int d1, int OW, int OH, int64_t Kp, __half *__restrict__ out) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t total = static_cast<int64_t>(OH) * OW * Kp;
    if (i >= total) return;
    const int64_t k = i % Kp, p = i / Kp;
    float v = 0.f;
    if (k < static_cast<int64_t>(IC) * KH * KW) {
        const int kx = static_cast<int>(k % KW), ky = static_cast<int>((k / KW) % KH), ic = static_cast<int>(k / (KW * KH));
        const int ox = static_cast<int>(p % OW), oy = static_cast<int>(p / OW);
        const int ix = ox * s0 + kx * d0 - p0, iy = oy * s1 + ky * d1 - p1;
        if (ix >= 0 && ix < IW && iy >= 0 && iy < IH) v = x[(static_cast<int64_t>(ic) * IH + iy) * IW + ix];
    }
    out[i] = __float2half_rn(v);
}

// get_rows: dst[i][c] = dequantised src row idx[i]; ggml block formats.
__global__ void get_rows_kernel(int type, const uint8_t *__restrict__ src, int64_t ncols, int64_t nrows,
                                int64_t row_bytes, const int32_t *__restrict__ idx, float *__restrict__ dst, int *err) {
    const int64_t i = blockIdx.x;
    const int32_t r = idx[i];
    float *d = dst + i * ncols;
    if (r < 0 || r >= nrows) {
        if (threadIdx.x == 0) atomicOr(err, kOpErrGetRowsIndex);
        for (int64_t c = threadIdx.x; c < ncols; c += blockDim.x) d[c] = 0.f;
        return;
    }
    const uint8_t *row = src + static_cast<int64_t>(r) * row_bytes;
    for (int64_t c = threadIdx.x; c < ncols; c += blockDim.x) {
        float v;
        if (type == SAM3B200_TYPE_F32) {
            v = reinterpret_cast<const float *>(row)[c];
        } else if (type == SAM3B200_TYPE_F16) {
            v = __half2float(reinterpret_cast<const __half *>(row)[c]);
        } else {
            const int64_t b = c / 32, j = c % 32;
            if (type == SAM3B200_TYPE_Q8_0) {  // {fp16 d; int8 q[32]}: q * d
                const uint8_t *blk = row + b * 34;
                const float dd = __half2float(*reinterpret_cast<const __half *>(blk));
                v = static_cast<float>(static_cast<int8_t>(blk[2 + j])) * dd;
            } else if (type == SAM3B200_TYPE_Q4_0) {  // {fp16 d; u8 q[16]}: (nibble - 8) * d
                const uint8_t *blk = row + b * 18;
                const float dd = __half2float(*reinterpret_cast<const __half *>(blk));
                const int q = j < 16 ? (blk[2 + j] & 0x0F) : (blk[2 + j - 16] >> 4);
                v = static_cast<float>(q - 8) * dd;
            } else {  // Q4_1 {fp16 d, m; u8 q[16]}: nibble * d + m
                const uint8_t *blk = row + b * 20;
                const float dd = __half2float(*reinterpret_cast<const __half *>(blk));
                const float mm = __half2float(*reinterpret_cast<const __half *>(blk + 2));
                const int q = j < 16 ? (blk[4 + j] & 0x0F) : (blk[4 + j - 16] >> 4);
                v = static_cast<float>(q) * dd + mm;
            }
        }
        d[c] = v;
    }
}

int fail(const char *msg) {
    set_error("%s", msg);
    return SAM3B200_STATUS_FAILED;
}

}  // namespace

}  // namespace b200

using namespace b200;

int sam3b200_conv_transpose_2d(sam3b200_backend *hb, const void *w_f16, const float *x, int64_t iw, int64_t ih,
                               int64_t ic, int64_t oc, int64_t kw, int64_t kh, int stride, float *dst) {
    auto *be = reinterpret_cast<Backend *>(hb);
    if (!be || !w_f16 || !x || !dst) return fail("conv_transpose_2d: null argument");
    if (iw <= 0 || ih <= 0 || ic <= 0 || oc <= 0 || kw <= 0 || kh <= 0 || stride <= 0 ||
        iw * ih > (1ll << 30) || oc * kh * kw > (1ll << 30) || ic > (1 << 20))
        return fail("conv_transpose_2d: unsupported shape");
    cudaSetDevice(be->device);
    const int64_t P = iw * ih, J = oc * kh * kw, Kp = pad8(ic);
    const int64_t ow = (iw - 1) * stride + kw, oh = (ih - 1) * stride + kh;
    const size_t wt_bytes = static_cast<size_t>(J * Kp) * 2, xt_bytes = static_cast<size_t>(P * Kp) * 2;
    const size_t col_bytes = static_cast<size_t>(J * P) * 4;
    const size_t off_x = (wt_bytes + 255) / 256 * 256, off_c = off_x + (xt_bytes + 255) / 256 * 256;
    void *buf = nullptr;
    if (!cuda_ok(cudaMallocAsync(&buf, off_c + col_bytes, be->stream), "cudaMallocAsync(conv_transpose_2d)"))
        return SAM3B200_STATUS_ALLOC_FAILED;
    char *base = static_cast<char *>(buf);
    __half *wt = reinterpret_cast<__half *>(base), *xt = reinterpret_cast<__half *>(base + off_x);
    float *cols = reinterpret_cast<float *>(base + off_c);
    // ggml kernel [KW,KH,OC,IC] is [IC][J] in memory: A = its transpose [J][Kp]
    bool ok = cuda_ok(transpose_pad_f16(static_cast<const uint16_t *>(w_f16), J, ic, Kp, wt, be->stream),
                      "conv_transpose_2d weights") &&
              cuda_ok(transpose_pad_f16(x, P, ic, Kp, xt, be->stream), "conv_transpose_2d input");
    if (ok) {
        GemmF16Args g{};
        g.a = wt;
        g.b = xt;
        g.M = static_cast<int>(J);
        g.N = static_cast<int>(P);
        g.K = static_cast<int>(Kp);
        g.out = cols;
        g.ldo = P;
        g.store = GEMM_STORE_ROWMAJOR;
        g.err = be->err;
        ok = cuda_ok(gemm_f16(g, be->num_sms, be->stream), "conv_transpose_2d gemm");
    }
    if (ok) {
        const int64_t total = oc * oh * ow;
        convt_gather_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, be->stream>>>(
            cols, static_cast<int>(iw), static_cast<int>(ih), static_cast<int>(oc), static_cast<int>(kw),
            static_cast<int>(kh), stride, static_cast<int>(ow), static_cast<int>(oh), dst);
        ok = cuda_ok(cudaGetLastError(), "conv_transpose_2d gather");
    }
    be->count(4);
    cudaFreeAsync(buf, be->stream);
    return ok ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
}

int sam3b200_conv_2d(sam3b200_backend *hb, const void *w_f16, const float *x, int64_t iw, int64_t ih, int64_t ic,
                     int64_t oc, int64_t kw, int64_t kh, int s0, int s1, int p0, int p1, int d0, int d1, float *dst) {
    auto *be = reinterpret_cast<Backend *>(hb);
    if (!be || !w_f16 || !x || !dst) return fail("conv_2d: null argument");
    if (iw <= 0 || ih <= 0 || ic <= 0 || oc <= 0 || kw <= 0 || kh <= 0 || s0 <= 0 || s1 <= 0 || p0 < 0 || p1 < 0 ||
        d0 <= 0 || d1 <= 0 || iw > (1 << 20) || ih > (1 << 20) || ic * kh * kw > (1 << 24) || oc > (1 << 24))
        return fail("conv_2d: unsupported shape");
    // a negative span (dilated kernel overhanging the padded input) must not truncate to one output column
    const int64_t span_w = iw + 2 * p0 - d0 * (kw - 1) - 1, span_h = ih + 2 * p1 - d1 * (kh - 1) - 1;
    if (span_w < 0 || span_h < 0) return fail("conv_2d: kernel larger than the padded input");
    const int64_t ow = span_w / s0 + 1;
    const int64_t oh = span_h / s1 + 1;
    if (ow <= 0 || oh <= 0 || ow * oh > (1ll << 30)) return fail("conv_2d: empty or oversized output");
    cudaSetDevice(be->device);
    const int64_t K = ic * kh * kw, Kp = pad8(K), P = ow * oh;
    const size_t col_bytes = static_cast<size_t>(P * Kp) * 2;
    const size_t w_bytes = Kp == K ? 0 : static_cast<size_t>(oc * Kp) * 2;
    const size_t off_w = (col_bytes + 255) / 256 * 256;
    void *buf = nullptr;
    if (!cuda_ok(cudaMallocAsync(&buf, off_w + w_bytes + 256, be->stream), "cudaMallocAsync(conv_2d)"))
        return SAM3B200_STATUS_ALLOC_FAILED;
    char *base = static_cast<char *>(buf);
    __half *cols = reinterpret_cast<__half *>(base);
    const void *a = w_f16;
    bool ok = true;
    int launches = 2;
    if (Kp != K) {  // ggml kernel rows are [OC][(ic, ky, kx)]: pad each to Kp
        uint16_t *wp = reinterpret_cast<uint16_t *>(base + off_w);
        const int64_t n = oc * Kp;
        pad_rows_f16_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, be->stream>>>(
            static_cast<const uint16_t *>(w_f16), oc, K, Kp, wp);
        ok = cuda_ok(cudaGetLastError(), "conv_2d weights");
        a = wp;
        ++launches;
    }
    if (ok) {
        const int64_t n = P * Kp;
        im2col_f16_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, be->stream>>>(
            x, static_cast<int>(iw), static_cast<int>(ih), static_cast<int>(ic), static_cast<int>(kw),
            static_cast<int>(kh), s0, s1, p0, p1, d0, d1, static_cast<int>(ow), static_cast<int>(oh), Kp, cols);
        ok = cuda_ok(cudaGetLastError(), "conv_2d im2col");
    }
    if (ok) {
        GemmF16Args g{};
        g.a = a;
        g.b = cols;
        g.M = static_cast<int>(oc);
        g.N = static_cast<int>(P);
        g.K = static_cast<int>(Kp);
        g.out = dst;
        g.ldo = P;
        g.store = GEMM_STORE_ROWMAJOR;
        g.err = be->err;
        ok = cuda_ok(gemm_f16(g, be->num_sms, be->stream), "conv_2d gemm");
    }
    be->count(launches);
    cudaFreeAsync(buf, be->stream);
    return ok ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
}

int sam3b200_get_rows(sam3b200_backend *hb, int type, const void *src, int64_t ncols, int64_t nrows,
                      const int32_t *idx, int64_t n, float *dst) {
    auto *be = reinterpret_cast<Backend *>(hb);
    if (!be || !src || !idx || !dst) return fail("get_rows: null argument");
    int64_t row_bytes;
    switch (type) {
        case SAM3B200_TYPE_F32: row_bytes = ncols * 4; break;
        case SAM3B200_TYPE_F16: row_bytes = ncols * 2; break;
        case SAM3B200_TYPE_Q8_0: row_bytes = ncols / 32 * 34; break;
        case SAM3B200_TYPE_Q4_0: row_bytes = ncols / 32 * 18; break;
        case SAM3B200_TYPE_Q4_1: row_bytes = ncols / 32 * 20; break;
        default: return fail("get_rows: unsupported source type (F32, F16, Q4_0, Q4_1, Q8_0)");
    }
    const bool blocked = type != SAM3B200_TYPE_F32 && type != SAM3B200_TYPE_F16;
    if (ncols <= 0 || nrows <= 0 || n < 0 || n > 0x7fffffff || (blocked && ncols % 32 != 0))
        return fail("get_rows: unsupported shape");
    if (n == 0) return SAM3B200_STATUS_SUCCESS;
    cudaSetDevice(be->device);
    get_rows_kernel<<<static_cast<unsigned>(n), 256, 0, be->stream>>>(type, static_cast<const uint8_t *>(src), ncols,
                                                                       nrows, row_bytes, idx, dst, be->err);
    be->count(1);
    return cuda_ok(cudaGetLastError(), "get_rows") ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
}

int sam3b200_flash_attn_ext(sam3b200_backend *hb, const float *q, const float *k, const float *v, int64_t D,
                            int64_t N, int64_t heads, int64_t batch, float scale, float *dst) {
    const int64_t nb[3] = {D, N * D, heads * N * D};
    return sam3b200_flash_attn_ext_view(hb, q, k, v, nullptr, 0, D, N, N, heads, batch, nb, nb, nb, scale, dst);
}

int sam3b200_flash_attn_ext_view(sam3b200_backend *hb, const float *q, const float *k, const float *v,
                                 const void *mask_f16, int64_t mask_nb1, int64_t D, int64_t NQ, int64_t NKV,
                                 int64_t heads, int64_t batch, const int64_t q_nb[3], const int64_t k_nb[3],
                                 const int64_t v_nb[3], float scale, float *dst) {
    auto *be = reinterpret_cast<Backend *>(hb);
    if (!be || !q || !k || !v || !dst || !q_nb || !k_nb || !v_nb) return fail("flash_attn_ext: null argument");
    const bool dims_ok = (D == 16 || D == 32 || D == 48 || D == 56 || D == 64 || D == 72 || D == 96 || D == 112 ||
                          D == 128 || D == 256);
    if (!dims_ok || NQ <= 0 || NKV <= 0 || heads <= 0 || batch <= 0 || NQ > (1 << 24) || NKV > (1 << 24) ||
        heads * batch > 65535 || (mask_f16 && mask_nb1 < NKV)) {
        set_error("flash_attn_ext: unsupported shape D=%lld NQ=%lld NKV=%lld heads=%lld batch=%lld (D in {16, 32, 48, "
                  "56, 64, 72, 96, 112, 128, 256})",
                  (long long)D, (long long)NQ, (long long)NKV, (long long)heads, (long long)batch);
        return SAM3B200_STATUS_FAILED;
    }
    cudaSetDevice(be->device);
    auto contiguous = [&](const int64_t *nb, int64_t n) { return nb[0] == D && nb[1] == n * D && nb[2] == heads * n * D; };
    const AttnStrides os{NQ * heads * D, D, heads * D};  // dst [D, heads, NQ, batch]
    // the tensor-core path stages q, k, v with 8-byte loads and stores dst 16 bytes at a time; views at
    // other offsets take the fp32 path, which reads and writes single floats
    auto aligned = [](const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; };
    if (D == 64 && !mask_f16 && NQ == NKV && NQ % 8 == 0 && contiguous(q_nb, NQ) && contiguous(k_nb, NKV) &&
        contiguous(v_nb, NKV) && aligned(q, 8) && aligned(k, 8) && aligned(v, 8) && aligned(dst, 16)) {
        // tensor cores: bf16 q, k and v^T staged from the f32 tensors
        const int BH = static_cast<int>(heads * batch), Ni = static_cast<int>(NQ);
        const size_t bytes = static_cast<size_t>(BH) * Ni * 64 * 2;
        void *buf = nullptr;
        if (!cuda_ok(cudaMallocAsync(&buf, 3 * bytes, be->stream), "cudaMallocAsync(attention inputs)"))
            return SAM3B200_STATUS_ALLOC_FAILED;
        char *qb = static_cast<char *>(buf);
        AttnOut o;
        o.f32 = dst;
        be->count(2);
        const bool ok = cuda_ok(attn_inputs_from_f32(q, k, v, BH, Ni, qb, qb + bytes, qb + 2 * bytes, be->stream),
                                "attention inputs") &&
                        cuda_ok(flash_attention(qb, qb + bytes, qb + 2 * bytes, static_cast<int>(batch), Ni,
                                                static_cast<int>(heads), scale, o, be->err, be->stream),
                                "flash_attn_ext");
        cudaFreeAsync(buf, be->stream);
        return ok ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
    }
    be->count(1);
    const AttnStrides qs{q_nb[2], q_nb[1], q_nb[0]}, ks{k_nb[2], k_nb[1], k_nb[0]}, vs{v_nb[2], v_nb[1], v_nb[0]};
    return cuda_ok(attention_simt(static_cast<int>(D), q, qs, static_cast<int>(NQ), k, ks, v, vs,
                                  static_cast<int>(NKV), static_cast<int>(batch), static_cast<int>(heads),
                                  static_cast<const __half *>(mask_f16), mask_nb1, scale, dst, os, be->stream),
                   "flash_attn_ext")
               ? SAM3B200_STATUS_SUCCESS
               : SAM3B200_STATUS_FAILED;
}
