// vit_ops.cu -- see vit_ops.cuh.  All float arithmetic that the CPU oracle
// performs in a fixed order is written with explicit round-to-nearest
// intrinsics so nvcc cannot contract it into FMAs; LayerNorm sums in double
// like ggml_norm does.
#include "vit_ops.cuh"
#include "mmq.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace b200 {

static inline unsigned grid_for(int64_t n, int threads) { return static_cast<unsigned>((n + threads - 1) / threads); }

// ---- preprocessing -----------------------------------------------------------
// (p / 255 - mean[c]) / std[c] per channel, every step rounded as the
// reference's float expression is
struct ChannelNorm {
    float mean[3], std[3];
};

__global__ void preprocess_kernel(const uint8_t *__restrict__ rgb, int img, const ChannelNorm nrm,
                                  float *__restrict__ out) {
    const int64_t p = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t plane = static_cast<int64_t>(img) * img;
    if (p >= plane) return;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        const float v = __fdiv_rn(static_cast<float>(rgb[p * 3 + c]), 255.0f);
        out[c * plane + p] = __fdiv_rn(__fsub_rn(v, nrm.mean[c]), nrm.std[c]);
    }
}

static cudaError_t preprocess_norm(const uint8_t *rgb, int img, const ChannelNorm &nrm, float *out, cudaStream_t s) {
    if (img <= 0) return cudaErrorInvalidValue;
    preprocess_kernel<<<grid_for(static_cast<int64_t>(img) * img, 256), 256, 0, s>>>(rgb, img, nrm, out);
    return cudaGetLastError();
}

cudaError_t preprocess_sam3(const uint8_t *rgb, int img, float *out, cudaStream_t s) {
    return preprocess_norm(rgb, img, ChannelNorm{{0.5f, 0.5f, 0.5f}, {0.5f, 0.5f, 0.5f}}, out, s);
}

cudaError_t preprocess_sam2(const uint8_t *rgb, int img, float *out, cudaStream_t s) {
    return preprocess_norm(rgb, img, ChannelNorm{{0.485f, 0.456f, 0.406f}, {0.229f, 0.224f, 0.225f}}, out, s);
}

__global__ void resize_kernel(const uint8_t *__restrict__ src, int sw, int sh, uint8_t *__restrict__ dst, int dw,
                              int dh) {
    const int64_t p = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (p >= static_cast<int64_t>(dw) * dh) return;
    const int x = static_cast<int>(p % dw), y = static_cast<int>(p / dw);
    const double sx = __ddiv_rn(sw, dw), sy = __ddiv_rn(sh, dh);
    double fy = __dsub_rn(__dmul_rn(__dadd_rn(y, 0.5), sy), 0.5);
    if (fy < 0.0) fy = 0.0;
    const int y0 = static_cast<int>(fy), y1 = (y0 < sh - 1) ? y0 + 1 : y0;
    const double wy = __dsub_rn(fy, y0), wy0 = __dsub_rn(1.0, wy);
    double fx = __dsub_rn(__dmul_rn(__dadd_rn(x, 0.5), sx), 0.5);
    if (fx < 0.0) fx = 0.0;
    const int x0 = static_cast<int>(fx), x1 = (x0 < sw - 1) ? x0 + 1 : x0;
    const double wx = __dsub_rn(fx, x0), wx0 = __dsub_rn(1.0, wx);
    for (int c = 0; c < 3; ++c) {
        const double p00 = src[(y0 * sw + x0) * 3 + c], p01 = src[(y0 * sw + x1) * 3 + c];
        const double p10 = src[(y1 * sw + x0) * 3 + c], p11 = src[(y1 * sw + x1) * 3 + c];
        const double top = __dadd_rn(__dmul_rn(wx0, p00), __dmul_rn(wx, p01));
        const double bot = __dadd_rn(__dmul_rn(wx0, p10), __dmul_rn(wx, p11));
        const double v = __dadd_rn(__dmul_rn(wy0, top), __dmul_rn(wy, bot));
        int iv = static_cast<int>(__dadd_rn(v, 0.5));
        iv = iv < 0 ? 0 : (iv > 255 ? 255 : iv);
        dst[(static_cast<int64_t>(y) * dw + x) * 3 + c] = static_cast<uint8_t>(iv);
    }
}

cudaError_t resize_bilinear_u8(const uint8_t *src, int sw, int sh, uint8_t *dst, int dw, int dh, cudaStream_t s) {
    if (sw <= 0 || sh <= 0 || dw <= 0 || dh <= 0) return cudaErrorInvalidValue;
    resize_kernel<<<grid_for(static_cast<int64_t>(dw) * dh, 256), 256, 0, s>>>(src, sw, sh, dst, dw, dh);
    return cudaGetLastError();
}

// ---- patch embedding im2col --------------------------------------------------
__global__ void im2col_patch_kernel(const float *__restrict__ img, int S, int p, int G, int kp, __half *__restrict__ a) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<int64_t>(G) * G * kp) return;
    const int t = static_cast<int>(i / kp), k = static_cast<int>(i % kp);
    float v = 0.f;
    if (k < 3 * p * p) {
        const int c = k / (p * p), ky = (k / p) % p, kx = k % p;
        const int px = t % G, py = t / G;
        v = img[static_cast<int64_t>(c) * S * S + static_cast<int64_t>(py * p + ky) * S + px * p + kx];
    }
    a[i] = __float2half_rn(v);
}

cudaError_t im2col_patch(const float *img, int S, int p, int kp, void *a, cudaStream_t s) {
    const int G = S / p;
    if (G <= 0 || kp < 3 * p * p) return cudaErrorInvalidValue;
    im2col_patch_kernel<<<grid_for(static_cast<int64_t>(G) * G * kp, 256), 256, 0, s>>>(img, S, p, G, kp,
                                                                                       static_cast<__half *>(a));
    return cudaGetLastError();
}

// ---- LayerNorm helpers (ggml_norm semantics, warp per row) -------------------
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// mean and 1/sqrt(var + eps) of a row, as ggml_norm computes them
__device__ __forceinline__ void row_stats(const float *__restrict__ r, int n, float eps, int lane, float &mean,
                                          float &scale) {
    double sum = 0.0;
    for (int i = lane; i < n; i += 32) sum += r[i];
    sum = warp_sum_d(sum);
    mean = static_cast<float>(sum / n);
    double sum2 = 0.0;
    for (int i = lane; i < n; i += 32) {
        const float v = __fsub_rn(r[i], mean);
        sum2 += static_cast<double>(__fmul_rn(v, v));
    }
    sum2 = warp_sum_d(sum2);
    const float variance = static_cast<float>(sum2 / n);
    scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(variance, eps)));
}

__device__ __forceinline__ float ln_apply(float x, float mean, float scale, float w, float b) {
    return __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x, mean), scale), w), b);
}

__global__ void add_pos_ln_kernel(const float *__restrict__ conv, const float *__restrict__ pos, int g, int G, int E,
                                  const float *__restrict__ w, const float *__restrict__ b, float eps,
                                  float *__restrict__ x) {
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= G * G) return;
    const int gw = (row % G) % g, gh = (row / G) % g;
    const float *cr = conv + static_cast<int64_t>(row) * E;
    const float *pr = pos + static_cast<int64_t>(gw + g * gh) * E;
    float *xr = x + static_cast<int64_t>(row) * E;
    for (int i = lane; i < E; i += 32) xr[i] = __fadd_rn(cr[i], pr[i]);
    __syncwarp();
    float mean, scale;
    row_stats(xr, E, eps, lane, mean, scale);
    for (int i = lane; i < E; i += 32) xr[i] = ln_apply(xr[i], mean, scale, w[i], b[i]);
}

cudaError_t add_pos_layernorm(const float *conv, const float *pos, int g, int G, int E, const float *w,
                              const float *b, float eps, float *x, cudaStream_t s) {
    if (E % 32 != 0 || G <= 0 || g <= 0) return cudaErrorInvalidValue;
    add_pos_ln_kernel<<<grid_for(static_cast<int64_t>(G) * G, 8), 256, 0, s>>>(conv, pos, g, G, E, w, b, eps, x);
    return cudaGetLastError();
}

__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
    return (static_cast<uint32_t>(a) & 0xFFu) | ((static_cast<uint32_t>(b) & 0xFFu) << 8) |
           ((static_cast<uint32_t>(c) & 0xFFu) << 16) | ((static_cast<uint32_t>(d) & 0xFFu) << 24);
}

// One warp per token row, one pass over HBM: lane l keeps the 32-wide
// blocks l and l + 32 (E <= 2048) in registers, the row statistics are
// formed from registers (double sums, as ggml_norm), then each lane
// normalises and quantises its own blocks.
__global__ void ln_q8_kernel(const float *__restrict__ x, int rows, int E, const float *__restrict__ w,
                             const float *__restrict__ b, float eps, int G, int win, int8_t *__restrict__ codes,
                             __half *__restrict__ quads, int ld) {
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (t >= rows) return;
    const float *xr = x + static_cast<int64_t>(t) * E;
    const int nblk = E >> 5;
    float v[2][32];
    double sum = 0.0;
#pragma unroll
    for (int s = 0; s < 2; ++s) {
        const int blk = lane + 32 * s;
        if (blk < nblk) {
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
                const float4 q = *reinterpret_cast<const float4 *>(xr + blk * 32 + i);
                v[s][i] = q.x;
                v[s][i + 1] = q.y;
                v[s][i + 2] = q.z;
                v[s][i + 3] = q.w;
            }
#pragma unroll
            for (int i = 0; i < 32; ++i) sum += v[s][i];
        }
    }
    sum = warp_sum_d(sum);
    const float mean = static_cast<float>(sum / E);
    double sum2 = 0.0;
#pragma unroll
    for (int s = 0; s < 2; ++s) {
        if (lane + 32 * s < nblk) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const float d = __fsub_rn(v[s][i], mean);
                sum2 += static_cast<double>(__fmul_rn(d, d));
            }
        }
    }
    sum2 = warp_sum_d(sum2);
    const float variance = static_cast<float>(sum2 / E);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(variance, eps)));
    int r = t;
    if (win > 0) {  // ggml_win_part position (image-major: rows of image i are [i G^2, (i + 1) G^2))
        const int img = t / (G * G), tl = t - img * (G * G);
        const int tx = tl % G, ty = tl / G, nw = G / win;
        r = img * (G * G) + ((ty / win) * nw + tx / win) * win * win + (tx % win) + win * (ty % win);
    }
#pragma unroll
    for (int s = 0; s < 2; ++s) {
        const int blk = lane + 32 * s;
        if (blk >= nblk) continue;
        float y[32];
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
            const float4 ww = *reinterpret_cast<const float4 *>(w + blk * 32 + i);
            const float4 bb = *reinterpret_cast<const float4 *>(b + blk * 32 + i);
            y[i] = ln_apply(v[s][i], mean, scale, ww.x, bb.x);
            y[i + 1] = ln_apply(v[s][i + 1], mean, scale, ww.y, bb.y);
            y[i + 2] = ln_apply(v[s][i + 2], mean, scale, ww.z, bb.z);
            y[i + 3] = ln_apply(v[s][i + 3], mean, scale, ww.w, bb.w);
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(y[i]));
        const float d = __fdiv_rn(amax, 127.f);
        const float id = amax != 0.f ? __fdiv_rn(127.f, amax) : 0.f;
        uint32_t pk[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
            pk[i] = pack4(__float2int_rn(__fmul_rn(y[4 * i], id)), __float2int_rn(__fmul_rn(y[4 * i + 1], id)),
                          __float2int_rn(__fmul_rn(y[4 * i + 2], id)), __float2int_rn(__fmul_rn(y[4 * i + 3], id)));
        uint4 *dst = reinterpret_cast<uint4 *>(codes + static_cast<int64_t>(r) * E + blk * 32);
        dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        store_act_scale(quads, blk, r, ld, nblk, d);
    }
}

// Coalesced variant for E a multiple of 128 (NJ = E / 128): lane l holds
// x[128 j + 4 l .. + 3], so every load is one 512-byte warp transaction.  The
// 32-element quantisation block 4 j + l / 8 then spans lanes 8 (l / 8) ..
// + 7 and its amax is a three-step shuffle.  The double-precision sums are
// those of ggml_norm (exact for these magnitudes, so the lane order does not
// change them).
// 128-thread CTAs; for E = 1024 at most 56 registers: 9 CTAs (36 warps) per
// SM, so the 5184 rows of a 72 x 72 map run as one wave (64 registers gave 32
// warps per SM: 1.09 waves, the last 4% of rows a second round of DRAM
// latency).  Other widths keep a budget they fit without spilling.
template <int NJ>
struct LnMinBlocks {
    static constexpr int value = NJ <= 4 || NJ == 8 ? 9 : NJ <= 6 ? 8 : 4;
};

// DQ: write the row's Q8_0 blocks dequantised, fp16(q * fp16(d)), into o16
// [rows][E] (the A operand of mmq_dq16) instead of codes + scale records.
template <int NJ, bool DQ = false>
__global__ void __launch_bounds__(128, LnMinBlocks<NJ>::value)
    ln_q8_coal_kernel(const float *__restrict__ x, int rows, const float *__restrict__ w,
                                  const float *__restrict__ b, float eps, int G, int win, int8_t *__restrict__ codes,
                                  __half *__restrict__ quads, int ld, __half *__restrict__ o16 = nullptr) {
    constexpr int E = NJ * 128;
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (t >= rows) return;
    const float *xr = x + static_cast<int64_t>(t) * E + 4 * lane;
    float4 v[NJ];
#pragma unroll
    for (int j = 0; j < NJ; ++j) v[j] = *reinterpret_cast<const float4 *>(xr + 128 * j);
    double s0 = 0.0, s1 = 0.0;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
        s0 += static_cast<double>(v[j].x) + static_cast<double>(v[j].y);
        s1 += static_cast<double>(v[j].z) + static_cast<double>(v[j].w);
    }
    const double sum = warp_sum_d(s0 + s1);
    const float mean = static_cast<float>(sum / E);
    double q0 = 0.0, q1 = 0.0;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
        const float d0 = __fsub_rn(v[j].x, mean), d1 = __fsub_rn(v[j].y, mean);
        const float d2 = __fsub_rn(v[j].z, mean), d3 = __fsub_rn(v[j].w, mean);
        q0 += static_cast<double>(__fmul_rn(d0, d0)) + static_cast<double>(__fmul_rn(d1, d1));
        q1 += static_cast<double>(__fmul_rn(d2, d2)) + static_cast<double>(__fmul_rn(d3, d3));
    }
    const double sum2 = warp_sum_d(q0 + q1);
    const float variance = static_cast<float>(sum2 / E);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(variance, eps)));
    int r = t;
    if (win > 0) {  // ggml_win_part position (image-major: rows of image i are [i G^2, (i + 1) G^2))
        const int img = t / (G * G), tl = t - img * (G * G);
        const int tx = tl % G, ty = tl / G, nw = G / win;
        r = img * (G * G) + ((ty / win) * nw + tx / win) * win * win + (tx % win) + win * (ty % win);
    }
    int8_t *cr = codes + static_cast<int64_t>(r) * E + 4 * lane;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
        const int e = 128 * j + 4 * lane;
        const float4 ww = *reinterpret_cast<const float4 *>(w + e);
        const float4 bb = *reinterpret_cast<const float4 *>(b + e);
        const float y0 = ln_apply(v[j].x, mean, scale, ww.x, bb.x), y1 = ln_apply(v[j].y, mean, scale, ww.y, bb.y);
        const float y2 = ln_apply(v[j].z, mean, scale, ww.z, bb.z), y3 = ln_apply(v[j].w, mean, scale, ww.w, bb.w);
        float amax = fmaxf(fmaxf(fabsf(y0), fabsf(y1)), fmaxf(fabsf(y2), fabsf(y3)));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
        const float d = __fdiv_rn(amax, 127.f);
        const float id = amax != 0.f ? __fdiv_rn(127.f, amax) : 0.f;
        if constexpr (DQ) {
            const float dh = __half2float(__float2half_rn(d));
            const __half2 h01 = __floats2half2_rn(__fmul_rn(q8_code_f(__fmul_rn(y0, id)), dh),
                                                  __fmul_rn(q8_code_f(__fmul_rn(y1, id)), dh));
            const __half2 h23 = __floats2half2_rn(__fmul_rn(q8_code_f(__fmul_rn(y2, id)), dh),
                                                  __fmul_rn(q8_code_f(__fmul_rn(y3, id)), dh));
            *reinterpret_cast<uint2 *>(o16 + static_cast<int64_t>(r) * E + 128 * j + 4 * lane) =
                make_uint2(*reinterpret_cast<const uint32_t *>(&h01), *reinterpret_cast<const uint32_t *>(&h23));
        } else {
            *reinterpret_cast<uint32_t *>(cr + 128 * j) =
                pack4(__float2int_rn(__fmul_rn(y0, id)), __float2int_rn(__fmul_rn(y1, id)),
                      __float2int_rn(__fmul_rn(y2, id)), __float2int_rn(__fmul_rn(y3, id)));
            if ((lane & 7) == 0) {
                const int blk = 4 * j + (lane >> 3);
                store_act_scale(quads, blk, r, ld, E >> 5, d);
            }
        }
    }
}

template <int NJ>
static void launch_ln_dq16(const float *x, int rows, const float *w, const float *b, float eps, int G, int win,
                           void *out16, cudaStream_t s) {
    ln_q8_coal_kernel<NJ, true><<<grid_for(rows, 4), 128, 0, s>>>(x, rows, w, b, eps, G, win, nullptr, nullptr, 0,
                                                                   static_cast<__half *>(out16));
}

cudaError_t layernorm_dq16(const float *x, int rows, int E, const float *w, const float *b, float eps, int G, int win,
                           void *out16, cudaStream_t s) {
    if (rows <= 0 || (reinterpret_cast<uintptr_t>(out16) & 15) || (win > 0 && (G % win != 0 || rows % (G * G) != 0)))
        return cudaErrorInvalidValue;
    switch (E) {
    case 256: launch_ln_dq16<2>(x, rows, w, b, eps, G, win, out16, s); break;
    case 512: launch_ln_dq16<4>(x, rows, w, b, eps, G, win, out16, s); break;
    case 768: launch_ln_dq16<6>(x, rows, w, b, eps, G, win, out16, s); break;
    case 1024: launch_ln_dq16<8>(x, rows, w, b, eps, G, win, out16, s); break;
    case 1280: launch_ln_dq16<10>(x, rows, w, b, eps, G, win, out16, s); break;
    case 1536: launch_ln_dq16<12>(x, rows, w, b, eps, G, win, out16, s); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

template <int NJ>
static void launch_ln_coal(const float *x, int rows, const float *w, const float *b, float eps, int G, int win,
                           void *codes, void *quads, int ld, cudaStream_t s) {
    ln_q8_coal_kernel<NJ><<<grid_for(rows, 4), 128, 0, s>>>(x, rows, w, b, eps, G, win, static_cast<int8_t *>(codes),
                                                             static_cast<__half *>(quads), ld);
}

cudaError_t layernorm_q8(const float *x, int rows, int E, const float *w, const float *b, float eps, int G, int win,
                         void *codes, void *quads, int ld, cudaStream_t s) {
    if (E % 32 != 0 || E > 2048 || rows <= 0 || ld < rows || (win > 0 && (G % win != 0 || rows % (G * G) != 0)))
        return cudaErrorInvalidValue;
    switch (E) {
    case 128: launch_ln_coal<1>(x, rows, w, b, eps, G, win, codes, quads, ld, s); break;
    case 256: launch_ln_coal<2>(x, rows, w, b, eps, G, win, codes, quads, ld, s); break;
    case 512: launch_ln_coal<4>(x, rows, w, b, eps, G, win, codes, quads, ld, s); break;
    case 768: launch_ln_coal<6>(x, rows, w, b, eps, G, win, codes, quads, ld, s); break;
    case 1024: launch_ln_coal<8>(x, rows, w, b, eps, G, win, codes, quads, ld, s); break;
    case 1280: launch_ln_coal<10>(x, rows, w, b, eps, G, win, codes, quads, ld, s); break;
    case 1536: launch_ln_coal<12>(x, rows, w, b, eps, G, win, codes, quads, ld, s); break;
    case 2048: launch_ln_coal<16>(x, rows, w, b, eps, G, win, codes, quads, ld, s); break;
    default:
        ln_q8_kernel<<<grid_for(rows, 8), 256, 0, s>>>(x, rows, E, w, b, eps, G, win, static_cast<int8_t *>(codes),
                                                       static_cast<__half *>(quads), ld);
    }
    return cudaGetLastError();
}

// ---- attention inputs from ggml f32 tensors ----------------------------------
// Q, K, V f32 [BH][N][64] (ggml [64, N, H, B]) -> bf16 Q, K in the same layout
// and bf16 V^T [BH][64][N]; one CTA per (64-token tile, bh), V through a
// shared-memory transpose.
__global__ void __launch_bounds__(256) attn_inputs_kernel(const float *__restrict__ q, const float *__restrict__ k,
                                                          const float *__restrict__ v, int N,
                                                          __nv_bfloat16 *__restrict__ qb, __nv_bfloat16 *__restrict__ kb,
                                                          __nv_bfloat16 *__restrict__ vt) {
    __shared__ __nv_bfloat16 vs[64][64 + 8];  // [dim][token]
    const int64_t bh = blockIdx.y;
    const int t0 = blockIdx.x * 64;
#pragma unroll
    for (int it = 0; it < 8; ++it) {
        const int item = it * 256 + threadIdx.x;  // (token, dim pair)
        const int tl = item >> 5, pr = item & 31, n = t0 + tl;
        if (n < N) {
            const int64_t o = (bh * N + n) * 64 + 2 * pr;
            const float2 qq = *reinterpret_cast<const float2 *>(q + o);
            const float2 kk = *reinterpret_cast<const float2 *>(k + o);
            const float2 vv = *reinterpret_cast<const float2 *>(v + o);
            *reinterpret_cast<__nv_bfloat162 *>(qb + o) = __floats2bfloat162_rn(qq.x, qq.y);
            *reinterpret_cast<__nv_bfloat162 *>(kb + o) = __floats2bfloat162_rn(kk.x, kk.y);
            vs[2 * pr][tl] = __float2bfloat16_rn(vv.x);
            vs[2 * pr + 1][tl] = __float2bfloat16_rn(vv.y);
        }
    }
    __syncthreads();
#pragma unroll
    for (int it = 0; it < 2; ++it) {
        const int item = it * 256 + threadIdx.x;  // (dim, 8-token chunk); N % 8 == 0 keeps 16-byte stores aligned
        const int d = item >> 3, ch = item & 7, n = t0 + ch * 8;
        if (n < N) {
            uint4 w;
            uint32_t *wp = reinterpret_cast<uint32_t *>(&w);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                __nv_bfloat162 pair;
                pair.x = vs[d][ch * 8 + 2 * e];
                pair.y = vs[d][ch * 8 + 2 * e + 1];
                wp[e] = *reinterpret_cast<uint32_t *>(&pair);
            }
            *reinterpret_cast<uint4 *>(vt + (bh * 64 + d) * N + n) = w;
        }
    }
}

cudaError_t attn_inputs_from_f32(const float *q, const float *k, const float *v, int BH, int N, void *qb, void *kb,
                                 void *vt, cudaStream_t s) {
    if (BH <= 0 || N <= 0 || N % 8 != 0) return cudaErrorInvalidValue;
    dim3 grid((N + 63) / 64, BH);
    attn_inputs_kernel<<<grid, 256, 0, s>>>(q, k, v, N, static_cast<__nv_bfloat16 *>(qb),
                                            static_cast<__nv_bfloat16 *>(kb), static_cast<__nv_bfloat16 *>(vt));
    return cudaGetLastError();
}

__global__ void rowmap_kernel(int G, int win, int nimg, int *__restrict__ rowmap) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= nimg * G * G) return;
    const int img = t / (G * G), tl = t - img * (G * G);
    const int tx = tl % G, ty = tl / G, nw = G / win;
    const int r = ((ty / win) * nw + tx / win) * win * win + (tx % win) + win * (ty % win);
    rowmap[img * (G * G) + r] = t;
}

cudaError_t window_rowmap(int G, int win, int *rowmap, cudaStream_t s, int nimg) {
    if (win <= 0 || G % win != 0 || nimg <= 0) return cudaErrorInvalidValue;
    rowmap_kernel<<<grid_for(static_cast<int64_t>(nimg) * G * G, 256), 256, 0, s>>>(G, win, nimg, rowmap);
    return cudaGetLastError();
}

// ---- neck helpers ----------------------------------------------------------------
__global__ void f32_to_f16_kernel(const float4 *__restrict__ x, int64_t n4, uint2 *__restrict__ y) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n4) return;
    const float4 v = x[i];
    __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
    y[i] = make_uint2(*reinterpret_cast<uint32_t *>(&a), *reinterpret_cast<uint32_t *>(&b));
}

__global__ void f32_rows_to_f16_kernel(const float *__restrict__ x, int64_t ldx, int M, int K,
                                       __half *__restrict__ y) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<int64_t>(M) * K) return;
    const int64_t m = i / K, k = i % K;
    y[i] = __float2half_rn(x[m * ldx + k]);
}

cudaError_t f32_rows_to_f16(const float *x, int64_t ldx, int M, int K, void *y, cudaStream_t s) {
    if (M <= 0 || K <= 0 || ldx < K) return cudaErrorInvalidValue;
    f32_rows_to_f16_kernel<<<grid_for(static_cast<int64_t>(M) * K, 256), 256, 0, s>>>(x, ldx, M, K,
                                                                                      static_cast<__half *>(y));
    return cudaGetLastError();
}

cudaError_t f32_to_f16(const float *x, int64_t n, void *y, cudaStream_t s) {
    if (n % 4 != 0) return cudaErrorInvalidValue;
    f32_to_f16_kernel<<<grid_for(n / 4, 256), 256, 0, s>>>(reinterpret_cast<const float4 *>(x), n / 4,
                                                           static_cast<uint2 *>(y));
    return cudaGetLastError();
}

__global__ void maxpool_kernel(const float *__restrict__ x, int G, int C, __half *__restrict__ y) {
    const int g = G / 2;
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<int64_t>(g) * g * C) return;
    const int c = static_cast<int>(i % C);
    const int p = static_cast<int>(i / C), ox = p % g, oy = p / g;
    const float *b0 = x + (static_cast<int64_t>(2 * oy) * G + 2 * ox) * C + c;
    float m = b0[0];
    const float v1 = b0[C], v2 = b0[static_cast<int64_t>(G) * C], v3 = b0[static_cast<int64_t>(G) * C + C];
    if (v1 > m) m = v1;
    if (v2 > m) m = v2;
    if (v3 > m) m = v3;
    y[i] = __float2half_rn(m);
}

cudaError_t maxpool2x2_f16(const float *x, int G, int C, void *y, cudaStream_t s) {
    if (G % 2 != 0) return cudaErrorInvalidValue;
    maxpool_kernel<<<grid_for(static_cast<int64_t>(G / 2) * (G / 2) * C, 256), 256, 0, s>>>(x, G, C,
                                                                                            static_cast<__half *>(y));
    return cudaGetLastError();
}

// one thread per (pixel, tap, 8 channels)
__global__ void im2col3x3_kernel(const uint4 *__restrict__ x, int W, int H, int C8, uint4 *__restrict__ a) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<int64_t>(W) * H * 9 * C8) return;
    const int c8 = static_cast<int>(i % C8);
    const int tap = static_cast<int>((i / C8) % 9);
    const int64_t p = i / (9 * C8);
    const int px = static_cast<int>(p % W), py = static_cast<int>(p / W);
    const int sx = px + tap % 3 - 1, sy = py + tap / 3 - 1;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (sx >= 0 && sy >= 0 && sx < W && sy < H) v = x[(static_cast<int64_t>(sy) * W + sx) * C8 + c8];
    a[i] = v;
}

cudaError_t im2col3x3_f16(const void *x, int W, int H, int C, void *a, cudaStream_t s) {
    if (C % 8 != 0) return cudaErrorInvalidValue;
    im2col3x3_kernel<<<grid_for(static_cast<int64_t>(W) * H * 9 * (C / 8), 256), 256, 0, s>>>(
        static_cast<const uint4 *>(x), W, H, C / 8, static_cast<uint4 *>(a));
    return cudaGetLastError();
}

}  // namespace b200
