// graph.cu -- the backend's supports_op and graph_compute over flattened ggml
// graph nodes (sam3b200_tensor, include/sam3_b200.h).
//
// sam3.cpp reaches every kernel through ggml_backend_graph_compute
// (sam3.cpp:1019-1030), which hands the backend the nodes of one graph in
// execution order.  This file is that executor: MUL_MAT (with the bias ADD
// that follows every linear layer fused into it when nothing else reads the
// product, sam3.cpp:3742-3743), FLASH_ATTN_EXT (:3778), CONV_TRANSPOSE_2D
// (:3884), CONV_2D (:3819) and GET_ROWS (the text encoder's token rows) run
// through the same entry points a direct caller uses, so their results are
// those of the op-level entries; the elementwise ops of the graphs (ADD, MUL,
// SCALE, the activations, ggml_norm, SOFT_MAX_EXT, WIN_PART / WIN_UNPART,
// CONT) run on the general-stride kernels below.  Views run nothing (their
// data already aliases their source).  The whole graph is checked before
// anything is launched, so a rejected graph leaves the device untouched.
#include "../../include/sam3_b200.h"
#include "act.cuh"
#include "backend_impl.h"
#include "gemm_f16.cuh"

#include <cuda_fp16.h>

#include <cfloat>
#include <cstdarg>
#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

static_assert(sizeof(sam3b200_tensor) == 192, "sam3b200_tensor layout is part of the C ABI");
static_assert(offsetof(sam3b200_tensor, src) == 144, "sam3b200_tensor layout is part of the C ABI");

namespace b200 {
namespace {

using T = sam3b200_tensor;

// Bytes of one ggml block and elements per block (ggml's type traits for the
// types this backend reads).
bool type_traits(int type, size_t *block_bytes, int64_t *block_elems) {
    switch (type) {
        case SAM3B200_TYPE_F32: *block_bytes = 4; *block_elems = 1; return true;
        case SAM3B200_TYPE_F16: *block_bytes = 2; *block_elems = 1; return true;
        case SAM3B200_TYPE_I32: *block_bytes = 4; *block_elems = 1; return true;
        case SAM3B200_TYPE_Q4_0: *block_bytes = 18; *block_elems = 32; return true;
        case SAM3B200_TYPE_Q4_1: *block_bytes = 20; *block_elems = 32; return true;
        case SAM3B200_TYPE_Q8_0: *block_bytes = 34; *block_elems = 32; return true;
        default: return false;
    }
}

bool shape_ok(const T *t) {
    for (int d = 0; d < 4; ++d)
        if (t->ne[d] < 1 || t->ne[d] > (1ll << 31)) return false;
    return true;
}

bool is_empty(const T *t) {
    for (int d = 0; d < 4; ++d)
        if (t->ne[d] == 0) return true;
    return false;
}

// ggml_is_contiguous: strides are the packed ones of the type.
bool contiguous(const T *t) {
    size_t bb;
    int64_t be;
    if (!type_traits(t->type, &bb, &be) || t->ne[0] % be != 0) return false;
    size_t expect = bb;
    if (t->nb[0] != expect) return false;
    expect = bb * static_cast<size_t>(t->ne[0] / be);
    for (int d = 1; d < 4; ++d) {
        if (t->ne[d] > 1 && t->nb[d] != expect) return false;
        expect *= static_cast<size_t>(t->ne[d]);
    }
    return true;
}

// Byte stride between consecutive rows of an F32 / F16 tensor whose dims 1..3 are
// read as one run of ne1*ne2*ne3 rows (ggml_mul_mat broadcasting a 2-D weight
// over them); 0 if those dims do not flatten to one evenly strided run or the
// elements of a row are not packed.
size_t flat_row_stride(const T *t) {
    const size_t elt = t->type == SAM3B200_TYPE_F32 ? 4 : t->type == SAM3B200_TYPE_F16 ? 2 : 0;
    if (!elt || t->nb[0] != elt) return 0;
    size_t stride = 0, next = 0;
    for (int d = 1; d < 4; ++d) {
        if (t->ne[d] == 1) continue;
        if (stride == 0) stride = t->nb[d];
        else if (t->nb[d] != next) return 0;
        next = t->nb[d] * static_cast<size_t>(t->ne[d]);
    }
    if (stride == 0) stride = static_cast<size_t>(t->ne[0]) * elt;  // one row
    if (stride % elt != 0 || stride < static_cast<size_t>(t->ne[0]) * elt) return 0;
    return stride;
}

int64_t rows_of(const T *t) { return t->ne[1] * t->ne[2] * t->ne[3]; }

float param_f32(const T *t, int i) {
    float f;
    std::memcpy(&f, &t->op_params[i], sizeof f);
    return f;
}

bool attn_dim_ok(int64_t D) {
    return D == 16 || D == 32 || D == 48 || D == 56 || D == 64 || D == 72 || D == 96 || D == 112 || D == 128 ||
           D == 256;
}

__attribute__((format(printf, 3, 4))) bool reject(char *why, size_t cap, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(why, cap, fmt, ap);
    va_end(ap);
    return false;
}

// Elementwise ops over ggml strides: one thread per result element (grid-stride), the result's
// coordinates read back into each source's strides (src1 broadcast by coordinate modulo its ne,
// ggml_can_repeat).  CONT pairs element i of the source with element i of the result, each in its own
// ggml order (ggml_cpy / ggml_cont_Nd may reshape).  Memory-bound scalar code; the model-level runners
// fuse these ops into their neighbours instead.
struct Shape4 {
    int64_t ne[4];
    int64_t nb[4];  // bytes
};

Shape4 shape_of(const T *t) {
    Shape4 s;
    for (int d = 0; d < 4; ++d) {
        s.ne[d] = t->ne[d];
        s.nb[d] = static_cast<int64_t>(t->nb[d]);
    }
    return s;
}

__device__ __forceinline__ int64_t offset_of(int64_t i, const Shape4 &s) {
    int64_t off = 0;
#pragma unroll
    for (int d = 0; d < 4; ++d) {
        off += (i % s.ne[d]) * s.nb[d];
        i /= s.ne[d];
    }
    return off;
}

__global__ void eltwise_kernel(int op, int unary, float scale, int cvt, const char *__restrict__ a, Shape4 sa,
                               const char *__restrict__ b, Shape4 sb, char *__restrict__ d, Shape4 sd,
                               int64_t total) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t c[4], t = i, od = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            c[k] = t % sd.ne[k];
            t /= sd.ne[k];
            od += c[k] * sd.nb[k];
        }
        if (op == SAM3B200_OP_CONT) {
            // cvt: bit 0 = source F16, bit 1 = result F16 (ggml_cast converts, round to nearest even)
            const int64_t oa = offset_of(i, sa);
            const float v = (cvt & 1) ? __half2float(*reinterpret_cast<const __half *>(a + oa))
                                      : *reinterpret_cast<const float *>(a + oa);
            if ((cvt & 3) == 3) *reinterpret_cast<__half *>(d + od) = *reinterpret_cast<const __half *>(a + oa);
            else if (cvt & 2) *reinterpret_cast<__half *>(d + od) = __float2half_rn(v);
            else *reinterpret_cast<float *>(d + od) = v;
            continue;
        }
        if (op == SAM3B200_OP_REPEAT) {
            int64_t oa = 0;
#pragma unroll
            for (int k = 0; k < 4; ++k) oa += (c[k] % sa.ne[k]) * sa.nb[k];
            *reinterpret_cast<float *>(d + od) = *reinterpret_cast<const float *>(a + oa);
            continue;
        }
        const float x = *reinterpret_cast<const float *>(a + c[0] * sa.nb[0] + c[1] * sa.nb[1] + c[2] * sa.nb[2] +
                                                         c[3] * sa.nb[3]);
        float y = x;
        if (op == SAM3B200_OP_ADD || op == SAM3B200_OP_MUL || op == SAM3B200_OP_SUB) {
            int64_t ob = 0;
#pragma unroll
            for (int k = 0; k < 4; ++k) ob += (c[k] % sb.ne[k]) * sb.nb[k];
            const float v = *reinterpret_cast<const float *>(b + ob);
            y = op == SAM3B200_OP_ADD ? __fadd_rn(x, v) : op == SAM3B200_OP_SUB ? __fsub_rn(x, v) : __fmul_rn(x, v);
        } else if (op == SAM3B200_OP_SCALE) {
            y = __fmul_rn(x, scale);
        } else if (op == SAM3B200_OP_UNARY) {
            switch (unary) {
                case SAM3B200_UNARY_RELU: y = x > 0.0f ? x : 0.0f; break;
                case SAM3B200_UNARY_SIGMOID: y = 1.0f / (1.0f + expf(-x)); break;
                case SAM3B200_UNARY_GELU_ERF: y = gelu_erf_f(x); break;
                default: y = gelu_tanh_f16(x); break;
            }
        }
        *reinterpret_cast<float *>(d + od) = y;
    }
}

// ggml_norm: per row of ne0 floats, mean and variance as double sums, y = (x - mean) / sqrt(var + eps).
// One warp per row.
__global__ void norm_rows_kernel(const char *__restrict__ a, Shape4 sa, char *__restrict__ d, Shape4 sd,
                                 int64_t rows, float eps) {
    const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const int64_t r1 = row % sa.ne[1], r2 = (row / sa.ne[1]) % sa.ne[2], r3 = row / (sa.ne[1] * sa.ne[2]);
    const char *ar = a + r1 * sa.nb[1] + r2 * sa.nb[2] + r3 * sa.nb[3];
    char *dr = d + r1 * sd.nb[1] + r2 * sd.nb[2] + r3 * sd.nb[3];
    const int64_t n = sa.ne[0];
    auto x = [&](int64_t i) { return *reinterpret_cast<const float *>(ar + i * sa.nb[0]); };
    double s = 0.0;
    for (int64_t i = lane; i < n; i += 32) s += static_cast<double>(x(i));
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = static_cast<float>(s / static_cast<double>(n));
    double s2 = 0.0;
    for (int64_t i = lane; i < n; i += 32) {
        const float v = __fsub_rn(x(i), mean);
        s2 += static_cast<double>(__fmul_rn(v, v));
    }
    for (int o = 16; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    const float var = static_cast<float>(s2 / static_cast<double>(n));
    const float sc = 1.0f / sqrtf(__fadd_rn(var, eps));
    for (int64_t i = lane; i < n; i += 32)
        *reinterpret_cast<float *>(dr + i * sd.nb[0]) = __fmul_rn(__fsub_rn(x(i), mean), sc);
}

// ggml_soft_max_ext with max_bias 0: per row of ne0, v = x * scale (+ mask row, F16 or F32, broadcast
// over dims 2 and 3), y = exp(v - max v) / sum (the sum in double, one reciprocal).  One warp per row.
__global__ void soft_max_rows_kernel(const char *__restrict__ a, Shape4 sa, const char *__restrict__ m, Shape4 sm,
                                     int m_f16, char *__restrict__ d, Shape4 sd, int64_t rows, float scale) {
    const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const int64_t r1 = row % sa.ne[1], r2 = (row / sa.ne[1]) % sa.ne[2], r3 = row / (sa.ne[1] * sa.ne[2]);
    const char *ar = a + r1 * sa.nb[1] + r2 * sa.nb[2] + r3 * sa.nb[3];
    char *dr = d + r1 * sd.nb[1] + r2 * sd.nb[2] + r3 * sd.nb[3];
    const char *mr = m ? m + r1 * sm.nb[1] + (r2 % sm.ne[2]) * sm.nb[2] + (r3 % sm.ne[3]) * sm.nb[3] : nullptr;
    const int64_t n = sa.ne[0];
    auto v = [&](int64_t i) {
        float t = __fmul_rn(*reinterpret_cast<const float *>(ar + i * sa.nb[0]), scale);
        if (mr) {
            const char *p = mr + i * sm.nb[0];
            t = __fadd_rn(t, m_f16 ? __half2float(*reinterpret_cast<const __half *>(p))
                                   : *reinterpret_cast<const float *>(p));
        }
        return t;
    };
    float mx = -INFINITY;
    for (int64_t i = lane; i < n; i += 32) mx = fmaxf(mx, v(i));
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    double s = 0.0;
    for (int64_t i = lane; i < n; i += 32) s += static_cast<double>(expf(__fsub_rn(v(i), mx)));
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float inv = static_cast<float>(1.0 / s);
    for (int64_t i = lane; i < n; i += 32)
        *reinterpret_cast<float *>(dr + i * sd.nb[0]) = __fmul_rn(expf(__fsub_rn(v(i), mx)), inv);
}

// ggml_win_part / ggml_win_unpart on contiguous f32 maps: windows of w x w tokens, window k = py * npx + px,
// zero padding right and bottom to whole windows.  part: dst [C, w, w, npx * npy] from src [C, W, H];
// unpart: dst [C, W, H] from src [C, w, w, nw].  One thread per result element.
__global__ void win_kernel(int unpart, const float *__restrict__ src, float *__restrict__ dst, int64_t C, int64_t W,
                           int64_t H, int64_t w, int64_t npx, int64_t total) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t c = i % C;
        if (!unpart) {
            const int64_t i1 = (i / C) % w, i2 = (i / (C * w)) % w, k = i / (C * w * w);
            const int64_t x = (k % npx) * w + i1, y = (k / npx) * w + i2;
            dst[i] = (x < W && y < H) ? src[(y * W + x) * C + c] : 0.0f;
        } else {
            const int64_t x = (i / C) % W, y = i / (C * W);
            const int64_t k = (y / w) * npx + x / w;
            dst[i] = src[((k * w + y % w) * w + x % w) * C + c];
        }
    }
}

// ggml_concat(a, b, dim): result coordinate c reads a at c when c[dim] < a.ne[dim], else b at c with
// c[dim] - a.ne[dim].  General strides, f32.
__global__ void concat_kernel(const char *__restrict__ a, Shape4 sa, const char *__restrict__ b, Shape4 sb,
                              char *__restrict__ d, Shape4 sd, int dim, int64_t total) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t c[4], t = i, od = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            c[k] = t % sd.ne[k];
            t /= sd.ne[k];
            od += c[k] * sd.nb[k];
        }
        const bool from_a = c[dim] < sa.ne[dim];
        if (!from_a) c[dim] -= sa.ne[dim];
        const Shape4 &ss = from_a ? sa : sb;
        const char *src = from_a ? a : b;
        *reinterpret_cast<float *>(d + od) = *reinterpret_cast<const float *>(
            src + c[0] * ss.nb[0] + c[1] * ss.nb[1] + c[2] * ss.nb[2] + c[3] * ss.nb[3]);
    }
}

// ggml_im2col (2-D) of x [IW, IH, IC, N] for a KW x KH kernel: result [IC*KH*KW, OW, OH, N], element
// iic*KH*KW + iky*KW + ikx of column (ow, oh, n) = x[ow*s0 + ikx*d0 - p0, oh*s1 + iky*d1 - p1, iic, n], zero
// outside the input.  F32 or F16 result, general input strides.
__global__ void im2col_kernel(const char *__restrict__ x, Shape4 sx, int x_f16, char *__restrict__ d, Shape4 sd,
                              int d_f16, int KW, int KH, int s0, int s1, int p0, int p1, int d0, int d1,
                              int64_t total) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t k = i % sd.ne[0], ow = (i / sd.ne[0]) % sd.ne[1], oh = (i / (sd.ne[0] * sd.ne[1])) % sd.ne[2],
                      n = i / (sd.ne[0] * sd.ne[1] * sd.ne[2]);
        const int64_t ikx = k % KW, iky = (k / KW) % KH, iic = k / (KW * KH);
        const int64_t ix = ow * s0 + ikx * d0 - p0, iy = oh * s1 + iky * d1 - p1;
        float v = 0.0f;
        if (ix >= 0 && ix < sx.ne[0] && iy >= 0 && iy < sx.ne[1]) {
            const char *p = x + ix * sx.nb[0] + iy * sx.nb[1] + iic * sx.nb[2] + n * sx.nb[3];
            v = x_f16 ? __half2float(*reinterpret_cast<const __half *>(p)) : *reinterpret_cast<const float *>(p);
        }
        char *q = d + k * sd.nb[0] + ow * sd.nb[1] + oh * sd.nb[2] + n * sd.nb[3];
        if (d_f16) *reinterpret_cast<__half *>(q) = __float2half_rn(v);
        else *reinterpret_cast<float *>(q) = v;
    }
}

// ggml_pool_2d over ne0, ne1 of x [IW, IH, C, N]: result [OW, OH, C, N]; window (k0 x k1) at
// (ox*s0 - p0, oy*s1 - p1); max over the in-bounds elements (from -FLT_MAX), or their sum over k0*k1.
__global__ void pool2d_kernel(const char *__restrict__ x, Shape4 sx, int x_f16, char *__restrict__ d, Shape4 sd,
                              int avg, int k0, int k1, int s0, int s1, int p0, int p1, int64_t total) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t ox = i % sd.ne[0], oy = (i / sd.ne[0]) % sd.ne[1], c2 = (i / (sd.ne[0] * sd.ne[1])) % sd.ne[2],
                      c3 = i / (sd.ne[0] * sd.ne[1] * sd.ne[2]);
        const char *base = x + c2 * sx.nb[2] + c3 * sx.nb[3];
        float acc = avg ? 0.0f : -FLT_MAX;
        for (int ky = 0; ky < k1; ++ky) {
            const int64_t iy = oy * s1 - p1 + ky;
            if (iy < 0 || iy >= sx.ne[1]) continue;
            for (int kx = 0; kx < k0; ++kx) {
                const int64_t ix = ox * s0 - p0 + kx;
                if (ix < 0 || ix >= sx.ne[0]) continue;
                const char *p = base + ix * sx.nb[0] + iy * sx.nb[1];
                const float v = x_f16 ? __half2float(*reinterpret_cast<const __half *>(p))
                                      : *reinterpret_cast<const float *>(p);
                acc = avg ? __fadd_rn(acc, v) : fmaxf(acc, v);
            }
        }
        if (avg) acc = __fdiv_rn(acc, static_cast<float>(k0 * k1));
        *reinterpret_cast<float *>(d + ox * sd.nb[0] + oy * sd.nb[1] + c2 * sd.nb[2] + c3 * sd.nb[3]) = acc;
    }
}

// ggml_pad_ext: result coordinate c reads x at c - lp when that lies inside x, else 0.
struct Pad4 {
    int64_t lp[4];
};
__global__ void pad_kernel(const char *__restrict__ x, Shape4 sx, char *__restrict__ d, Shape4 sd, Pad4 pad,
                           int64_t total) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t t = i, od = 0, ox = 0;
        bool in = true;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int64_t c = t % sd.ne[k];
            t /= sd.ne[k];
            od += c * sd.nb[k];
            const int64_t cs = c - pad.lp[k];
            in = in && cs >= 0 && cs < sx.ne[k];
            ox += cs * sx.nb[k];
        }
        *reinterpret_cast<float *>(d + od) = in ? *reinterpret_cast<const float *>(x + ox) : 0.0f;
    }
}

// ggml_upscale, nearest: result coordinate c reads x at c * x.ne / d.ne per dimension (integer factors).
__global__ void upscale_kernel(const char *__restrict__ x, Shape4 sx, char *__restrict__ d, Shape4 sd,
                               int64_t total) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t t = i, od = 0, ox = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int64_t c = t % sd.ne[k];
            t /= sd.ne[k];
            od += c * sd.nb[k];
            ox += (c * sx.ne[k] / sd.ne[k]) * sx.nb[k];
        }
        *reinterpret_cast<float *>(d + od) = *reinterpret_cast<const float *>(x + ox);
    }
}

// ggml_conv_2d_dw_direct: kernel [KW, KH, 1, C] (f32), x [W, H, C, N] -> result [OW, OH, C, N]; each
// channel convolved with its own kernel, products summed in fp32 row by row of the kernel.
__global__ void conv2d_dw_kernel(const char *__restrict__ kern, Shape4 sk, const char *__restrict__ x, Shape4 sx,
                                 char *__restrict__ d, Shape4 sd, int s0, int s1, int p0, int p1, int d0, int d1,
                                 int64_t total) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t ox = i % sd.ne[0], oy = (i / sd.ne[0]) % sd.ne[1], c = (i / (sd.ne[0] * sd.ne[1])) % sd.ne[2],
                      n = i / (sd.ne[0] * sd.ne[1] * sd.ne[2]);
        const char *kc = kern + c * sk.nb[3];
        const char *xc = x + c * sx.nb[2] + n * sx.nb[3];
        float acc = 0.0f;
        for (int64_t ky = 0; ky < sk.ne[1]; ++ky) {
            const int64_t iy = oy * s1 + ky * d1 - p1;
            if (iy < 0 || iy >= sx.ne[1]) continue;
            for (int64_t kx = 0; kx < sk.ne[0]; ++kx) {
                const int64_t ix = ox * s0 + kx * d0 - p0;
                if (ix < 0 || ix >= sx.ne[0]) continue;
                acc = fmaf(*reinterpret_cast<const float *>(kc + kx * sk.nb[0] + ky * sk.nb[1]),
                           *reinterpret_cast<const float *>(xc + ix * sx.nb[0] + iy * sx.nb[1]), acc);
            }
        }
        *reinterpret_cast<float *>(d + ox * sd.nb[0] + oy * sd.nb[1] + c * sd.nb[2] + n * sd.nb[3]) = acc;
    }
}

// ggml_group_norm: x [W, H, C, N], groups of ceil(C / G) channels; per (group, n) the mean and variance
// of its W*H*channels values as double sums, y = (x - mean) * (1 / sqrt(var + eps)).  One CTA per
// (group, n).
__global__ void __launch_bounds__(256) group_norm_kernel(const char *__restrict__ x, Shape4 sx, char *__restrict__ d,
                                                         Shape4 sd, int groups, float eps) {
    const int g = blockIdx.x % groups, n = blockIdx.x / groups;
    const int64_t cpg = (sx.ne[2] + groups - 1) / groups;
    const int64_t c0 = g * cpg, c1 = (c0 + cpg < sx.ne[2]) ? c0 + cpg : sx.ne[2];
    if (c0 >= c1) return;
    const int64_t plane = sx.ne[0] * sx.ne[1], count = plane * (c1 - c0);
    auto xat = [&](int64_t j) {
        const int64_t i0 = j % sx.ne[0], i1 = (j / sx.ne[0]) % sx.ne[1], c = c0 + j / plane;
        return *reinterpret_cast<const float *>(x + i0 * sx.nb[0] + i1 * sx.nb[1] + c * sx.nb[2] + n * sx.nb[3]);
    };
    __shared__ double red[8];
    __shared__ float stat[2];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    double s = 0.0;
    for (int64_t j = threadIdx.x; j < count; j += blockDim.x) s += static_cast<double>(xat(j));
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
        stat[0] = static_cast<float>(t / static_cast<double>(count));
    }
    __syncthreads();
    const float mean = stat[0];
    double s2 = 0.0;
    for (int64_t j = threadIdx.x; j < count; j += blockDim.x) {
        const float v = __fsub_rn(xat(j), mean);
        s2 += static_cast<double>(__fmul_rn(v, v));
    }
    for (int o = 16; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    __syncthreads();
    if (lane == 0) red[warp] = s2;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
        const float var = static_cast<float>(t / static_cast<double>(count));
        stat[1] = __fdiv_rn(1.0f, sqrtf(__fadd_rn(var, eps)));
    }
    __syncthreads();
    const float sc = stat[1];
    for (int64_t j = threadIdx.x; j < count; j += blockDim.x) {
        const int64_t i0 = j % sx.ne[0], i1 = (j / sx.ne[0]) % sx.ne[1], c = c0 + j / plane;
        *reinterpret_cast<float *>(d + i0 * sd.nb[0] + i1 * sd.nb[1] + c * sd.nb[2] + n * sd.nb[3]) =
            __fmul_rn(__fsub_rn(xat(j), mean), sc);
    }
}

// Rows of an F32 / F16 matrix (row stride ld elements) to fp16 [rows, Kp], zero beyond K: the operands of
// the fp16 tensor-core GEMM behind a MUL_MAT whose src0 is a tensor of the graph.
__global__ void rows_to_f16_padded_kernel(const char *__restrict__ x, int64_t ld_bytes, int f16, int64_t rows,
                                          int64_t K, int64_t Kp, __half *__restrict__ y) {
    const int64_t total = rows * Kp;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / Kp, k = i % Kp;
        float v = 0.0f;
        if (k < K) {
            const char *p = x + r * ld_bytes;
            v = f16 ? __half2float(reinterpret_cast<const __half *>(p)[k]) : reinterpret_cast<const float *>(p)[k];
        }
        y[i] = __float2half_rn(v);
    }
}

// MUL_MAT of two tensors of the graph (ggml_mul_mat whose src0 is not a weight: attention scores and
// their product with V, sam3.cpp:8584-8588, 10218-10240; mask logits, sam3.cpp:9055, 10717):
//   result[n, m, i2, i3] = sum_k src0[k, n, i2 / r2, i3 / r3] * src1[k, m, i2, i3],
// r2 = ne12 / ne02, r3 = ne13 / ne03 (ggml's batch broadcast).  64 x 64 result tiles per CTA, K staged
// through shared memory 16 at a time, 4 x 4 results per thread, fp32 FMAs in k order.  With an F16
// src0 the src1 values are rounded to fp16 first (ggml-cpu's vec_dot_type for F16 rows).
constexpr int RT_TILE = 64, RT_K = 16;

__device__ __forceinline__ float load_elt(const char *p, int f16) {
    return f16 ? __half2float(*reinterpret_cast<const __half *>(p)) : *reinterpret_cast<const float *>(p);
}

__global__ void __launch_bounds__(256) mul_mat_rt_kernel(const char *__restrict__ s0, Shape4 a0, int f16_0,
                                                         const char *__restrict__ s1, Shape4 a1, int f16_1,
                                                         char *__restrict__ d, Shape4 sd, int64_t K) {
    __shared__ float xs[RT_K][RT_TILE + 4];  // src1 rows (result columns m)
    __shared__ float ws[RT_K][RT_TILE + 4];  // src0 rows (result rows n)
    const int64_t N = sd.ne[0], M = sd.ne[1];
    const int64_t n0 = static_cast<int64_t>(blockIdx.x) * RT_TILE, m0 = static_cast<int64_t>(blockIdx.y) * RT_TILE;
    const int64_t i2 = blockIdx.z % sd.ne[2], i3 = blockIdx.z / sd.ne[2];
    const int64_t r2 = sd.ne[2] / a0.ne[2], r3 = sd.ne[3] / a0.ne[3];
    const char *w = s0 + (i2 / r2) * a0.nb[2] + (i3 / r3) * a0.nb[3];
    const char *x = s1 + i2 * a1.nb[2] + i3 * a1.nb[3];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
    for (int64_t k0 = 0; k0 < K; k0 += RT_K) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int idx = threadIdx.x + 256 * j, kk = idx % RT_K, r = idx / RT_K;
            const int64_t k = k0 + kk;
            float xv = 0.0f, wv = 0.0f;
            if (k < K && m0 + r < M) {
                xv = load_elt(x + k * a1.nb[0] + (m0 + r) * a1.nb[1], f16_1);
                if (f16_0) xv = __half2float(__float2half_rn(xv));
            }
            if (k < K && n0 + r < N) wv = load_elt(w + k * a0.nb[0] + (n0 + r) * a0.nb[1], f16_0);
            xs[kk][r] = xv;
            ws[kk][r] = wv;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < RT_K; ++kk) {
            float xv[4], wv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                xv[i] = xs[kk][ty + 16 * i];
                wv[i] = ws[kk][tx + 16 * i];
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(xv[i], wv[j], acc[i][j]);
        }
        __syncthreads();
    }
    char *o = d + i2 * sd.nb[2] + i3 * sd.nb[3];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t m = m0 + ty + 16 * i;
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int64_t n = n0 + tx + 16 * j;
            if (n < N) *reinterpret_cast<float *>(o + n * sd.nb[0] + m * sd.nb[1]) = acc[i][j];
        }
    }
}

bool strides_ok(const T *t, size_t elt) {
    for (int d = 0; d < 4; ++d)
        if (t->nb[d] % elt != 0 || t->nb[d] == 0) return false;
    return true;
}

int64_t nelements(const T *t) { return t->ne[0] * t->ne[1] * t->ne[2] * t->ne[3]; }

size_t elt_size(int type) { return type == SAM3B200_TYPE_F16 ? 2 : 4; }

bool f32_or_f16(const T *t) { return t->type == SAM3B200_TYPE_F32 || t->type == SAM3B200_TYPE_F16; }

// MUL_MAT whose src0 is an F32 / F16 tensor of the graph rather than an uploaded weight.
bool runtime_src0(const T *n) {
    const T *a = n->src[0];
    return n->op == SAM3B200_OP_MUL_MAT && a && f32_or_f16(a) && !a->extra;
}

// ggml_calc_conv_output_size: (in + 2p - d (k - 1) - 1) / s + 1, or 0 when the kernel overhangs.
int64_t conv_out(int64_t in, int64_t k, int s, int p, int d) {
    const int64_t span = in + 2 * static_cast<int64_t>(p) - static_cast<int64_t>(d) * (k - 1) - 1;
    return span < 0 ? 0 : span / s + 1;
}

bool check_mul_mat_rt(const T *n, char *why, size_t cap) {
    const T *a = n->src[0], *b = n->src[1];
    if (!f32_or_f16(b) || !shape_ok(a) || !shape_ok(b) || b->ne[0] != a->ne[0])
        return reject(why, cap, "MUL_MAT of two graph tensors: src1 F32 / F16 with ne0 == K=%lld", (long long)a->ne[0]);
    if (b->ne[2] % a->ne[2] != 0 || b->ne[3] % a->ne[3] != 0)
        return reject(why, cap, "MUL_MAT: src0 batches [%lld, %lld] do not broadcast over src1's [%lld, %lld]",
                      (long long)a->ne[2], (long long)a->ne[3], (long long)b->ne[2], (long long)b->ne[3]);
    if (n->type != SAM3B200_TYPE_F32 || n->ne[0] != a->ne[1] || n->ne[1] != b->ne[1] || n->ne[2] != b->ne[2] ||
        n->ne[3] != b->ne[3])
        return reject(why, cap, "MUL_MAT result must be f32 [src0 ne1, src1 ne1, src1 ne2, src1 ne3]");
    if (!strides_ok(a, elt_size(a->type)) || !strides_ok(b, elt_size(b->type)) || !strides_ok(n, 4))
        return reject(why, cap, "MUL_MAT: strides must be whole elements");
    if ((n->ne[1] + RT_TILE - 1) / RT_TILE > 65535 || n->ne[2] * n->ne[3] > 65535)
        return reject(why, cap, "MUL_MAT of two graph tensors: more than 4194240 rows or 65535 batches");
    return true;
}

// The node-local rules of each op; on failure `why` says which.
bool check_node(const T *n, char *why, size_t cap) {
    if (!n) return reject(why, cap, "null node");
    const T *a = n->src[0], *b = n->src[1];
    switch (n->op) {
        case SAM3B200_OP_NONE: return true;
        case SAM3B200_OP_VIEW: return a ? true : reject(why, cap, "VIEW without a source");
        case SAM3B200_OP_MUL_MAT: {
            if (!a || !b) return reject(why, cap, "MUL_MAT needs src0 (weight) and src1 (x)");
            if (runtime_src0(n)) return check_mul_mat_rt(n, why, cap);
            if (a->type != SAM3B200_TYPE_Q8_0 && a->type != SAM3B200_TYPE_Q4_0 && a->type != SAM3B200_TYPE_Q4_1 &&
                a->type != SAM3B200_TYPE_F16 && a->type != SAM3B200_TYPE_F32)
                return reject(why, cap, "MUL_MAT weight type %d (F32, F16, Q4_0, Q4_1, Q8_0)", a->type);
            if (!shape_ok(a) || a->ne[2] != 1 || a->ne[3] != 1 || !contiguous(a))
                return reject(why, cap, "MUL_MAT weight must be a contiguous 2-D tensor");
            const bool quant = a->type != SAM3B200_TYPE_F16 && a->type != SAM3B200_TYPE_F32;
            if (a->ne[0] % (quant ? 32 : 8) != 0)
                return reject(why, cap, "MUL_MAT K=%lld is not a multiple of %d", (long long)a->ne[0], quant ? 32 : 8);
            if (b->type != SAM3B200_TYPE_F32 || !shape_ok(b) || b->ne[0] != a->ne[0])
                return reject(why, cap, "MUL_MAT x must be f32 with ne0 == K=%lld", (long long)a->ne[0]);
            if (!flat_row_stride(b)) return reject(why, cap, "MUL_MAT x rows do not flatten to one strided run");
            if (n->type != SAM3B200_TYPE_F32 || n->ne[0] != a->ne[1] || n->ne[1] != b->ne[1] ||
                n->ne[2] != b->ne[2] || n->ne[3] != b->ne[3])
                return reject(why, cap, "MUL_MAT result must be f32 [N, ne1, ne2, ne3] of x");
            if (!flat_row_stride(n)) return reject(why, cap, "MUL_MAT result rows do not flatten to one strided run");
            if (rows_of(b) > (1 << 24)) return reject(why, cap, "MUL_MAT with more than 2^24 rows");
            return true;
        }
        case SAM3B200_OP_ADD:
        case SAM3B200_OP_SUB:
        case SAM3B200_OP_MUL: {
            const char *name = n->op == SAM3B200_OP_ADD ? "ADD" : n->op == SAM3B200_OP_SUB ? "SUB" : "MUL";
            if (!a || !b) return reject(why, cap, "%s needs two sources", name);
            if (a->type != SAM3B200_TYPE_F32 || b->type != SAM3B200_TYPE_F32 || n->type != SAM3B200_TYPE_F32 ||
                !shape_ok(a) || !shape_ok(b) || std::memcmp(n->ne, a->ne, sizeof n->ne) != 0)
                return reject(why, cap, "%s: f32 operands, result of src0's shape", name);
            for (int d = 0; d < 4; ++d)
                if (a->ne[d] % b->ne[d] != 0) return reject(why, cap, "%s: src1 does not repeat into src0", name);
            if (!strides_ok(a, 4) || !strides_ok(b, 4) || !strides_ok(n, 4))
                return reject(why, cap, "%s: strides must be whole floats", name);
            return true;
        }
        case SAM3B200_OP_SCALE:
        case SAM3B200_OP_UNARY:
        case SAM3B200_OP_NORM: {
            if (!a || a->type != SAM3B200_TYPE_F32 || n->type != SAM3B200_TYPE_F32 || !shape_ok(a) ||
                std::memcmp(n->ne, a->ne, sizeof n->ne) != 0 || !strides_ok(a, 4) || !strides_ok(n, 4))
                return reject(why, cap, "SCALE / UNARY / NORM: f32 source and result of the same shape");
            if (n->op == SAM3B200_OP_UNARY && (n->op_params[0] < SAM3B200_UNARY_RELU ||
                                               n->op_params[0] > SAM3B200_UNARY_GELU))
                return reject(why, cap, "UNARY kind %d (RELU 1, SIGMOID 2, GELU_ERF 3, GELU 4)", n->op_params[0]);
            if (n->op == SAM3B200_OP_NORM && !(param_f32(n, 0) >= 0.0f))
                return reject(why, cap, "NORM eps must be >= 0");
            return true;
        }
        case SAM3B200_OP_SOFT_MAX: {
            if (!a || a->type != SAM3B200_TYPE_F32 || n->type != SAM3B200_TYPE_F32 || !shape_ok(a) ||
                std::memcmp(n->ne, a->ne, sizeof n->ne) != 0 || !strides_ok(a, 4) || !strides_ok(n, 4))
                return reject(why, cap, "SOFT_MAX: f32 source and result of the same shape");
            if (param_f32(n, 1) != 0.0f) return reject(why, cap, "SOFT_MAX with max_bias (ALiBi) is not run here");
            if (b) {
                const size_t elt = b->type == SAM3B200_TYPE_F16 ? 2 : 4;
                if ((b->type != SAM3B200_TYPE_F16 && b->type != SAM3B200_TYPE_F32) || !shape_ok(b) ||
                    b->ne[0] != a->ne[0] || b->ne[1] < a->ne[1] || a->ne[2] % b->ne[2] != 0 ||
                    a->ne[3] % b->ne[3] != 0 || !strides_ok(b, elt))
                    return reject(why, cap, "SOFT_MAX mask: F16 / F32 [ne0, >= ne1] repeating over dims 2, 3");
            }
            return true;
        }
        case SAM3B200_OP_WIN_PART:
        case SAM3B200_OP_WIN_UNPART: {
            const bool part = n->op == SAM3B200_OP_WIN_PART;
            if (!a || a->type != SAM3B200_TYPE_F32 || n->type != SAM3B200_TYPE_F32 || !shape_ok(a) || !shape_ok(n) ||
                !contiguous(a) || !contiguous(n))
                return reject(why, cap, "WIN_PART / WIN_UNPART: contiguous f32 source and result");
            const T *map = part ? a : n, *win = part ? n : a;
            const int64_t w = part ? n->op_params[2] : n->op_params[0];
            if (w <= 0 || map->ne[3] != 1 || win->ne[0] != map->ne[0] || win->ne[1] != w || win->ne[2] != w)
                return reject(why, cap, "WIN_PART / WIN_UNPART: windows [C, w, w, n] of a map [C, W, H, 1]");
            const int64_t npx = (map->ne[1] + w - 1) / w, npy = (map->ne[2] + w - 1) / w;
            if (win->ne[3] != npx * npy || (part && (n->op_params[0] != npx || n->op_params[1] != npy)))
                return reject(why, cap, "WIN_PART / WIN_UNPART: %lld x %lld windows expected", (long long)npx,
                              (long long)npy);
            return true;
        }
        case SAM3B200_OP_CONT: {
            if (!a || !shape_ok(a) || !shape_ok(n) || !f32_or_f16(a) || !f32_or_f16(n) ||
                nelements(a) != nelements(n))
                return reject(why, cap, "CONT: F32 or F16 source and result of one element count");
            if (!strides_ok(a, elt_size(a->type)) || !strides_ok(n, elt_size(n->type)))
                return reject(why, cap, "CONT: strides must be whole elements");
            return true;
        }
        case SAM3B200_OP_REPEAT: {
            if (!a || a->type != SAM3B200_TYPE_F32 || n->type != SAM3B200_TYPE_F32 || !shape_ok(a) || !shape_ok(n) ||
                !strides_ok(a, 4) || !strides_ok(n, 4))
                return reject(why, cap, "REPEAT: f32 source and result");
            for (int d = 0; d < 4; ++d)
                if (n->ne[d] % a->ne[d] != 0) return reject(why, cap, "REPEAT: source does not repeat into the result");
            return true;
        }
        case SAM3B200_OP_CONCAT: {
            const int dim = n->op_params[0];
            if (!a || !b || a->type != SAM3B200_TYPE_F32 || b->type != SAM3B200_TYPE_F32 ||
                n->type != SAM3B200_TYPE_F32 || !shape_ok(a) || !shape_ok(b) || !shape_ok(n) || !strides_ok(a, 4) ||
                !strides_ok(b, 4) || !strides_ok(n, 4))
                return reject(why, cap, "CONCAT: f32 sources and result");
            if (dim < 0 || dim > 3) return reject(why, cap, "CONCAT dim %d", dim);
            for (int d = 0; d < 4; ++d)
                if ((d == dim && n->ne[d] != a->ne[d] + b->ne[d]) ||
                    (d != dim && (a->ne[d] != n->ne[d] || b->ne[d] != n->ne[d])))
                    return reject(why, cap, "CONCAT: shapes do not join along dim %d", dim);
            return true;
        }
        case SAM3B200_OP_IM2COL: {
            const int32_t *p = n->op_params;  // s0, s1, p0, p1, d0, d1, is_2D
            if (!a || !b || !shape_ok(a) || !shape_ok(b) || !shape_ok(n) || !f32_or_f16(b) || !f32_or_f16(n))
                return reject(why, cap, "IM2COL needs a kernel shape (src0), an F32 / F16 input and an F32 / F16 result");
            if (p[6] != 1) return reject(why, cap, "IM2COL: only the 2-D form is run here");
            if (p[0] <= 0 || p[1] <= 0 || p[2] < 0 || p[3] < 0 || p[4] <= 0 || p[5] <= 0)
                return reject(why, cap, "IM2COL stride/padding/dilation (%d %d %d %d %d %d)", p[0], p[1], p[2], p[3],
                              p[4], p[5]);
            if (b->ne[2] != a->ne[2]) return reject(why, cap, "IM2COL: input channels != kernel channels");
            const int64_t ow = conv_out(b->ne[0], a->ne[0], p[0], p[2], p[4]);
            const int64_t oh = conv_out(b->ne[1], a->ne[1], p[1], p[3], p[5]);
            if (n->ne[0] != a->ne[0] * a->ne[1] * a->ne[2] || n->ne[1] != ow || n->ne[2] != oh || n->ne[3] != b->ne[3])
                return reject(why, cap, "IM2COL result must be [IC*KH*KW, %lld, %lld, N]", (long long)ow, (long long)oh);
            if (!strides_ok(b, elt_size(b->type)) || !strides_ok(n, elt_size(n->type)))
                return reject(why, cap, "IM2COL: strides must be whole elements");
            return true;
        }
        case SAM3B200_OP_POOL_2D: {
            const int32_t *p = n->op_params;  // op, k0, k1, s0, s1, p0, p1
            if (!a || !f32_or_f16(a) || n->type != SAM3B200_TYPE_F32 || !shape_ok(a) || !shape_ok(n) ||
                !strides_ok(a, elt_size(a->type)) || !strides_ok(n, 4))
                return reject(why, cap, "POOL_2D: F32 / F16 source, f32 result");
            if ((p[0] != 0 && p[0] != 1) || p[1] <= 0 || p[2] <= 0 || p[3] <= 0 || p[4] <= 0 || p[5] < 0 || p[6] < 0)
                return reject(why, cap, "POOL_2D op/kernel/stride/padding (%d %d %d %d %d %d %d)", p[0], p[1], p[2],
                              p[3], p[4], p[5], p[6]);
            const int64_t ow = conv_out(a->ne[0], p[1], p[3], p[5], 1), oh = conv_out(a->ne[1], p[2], p[4], p[6], 1);
            if (n->ne[0] != ow || n->ne[1] != oh || n->ne[2] != a->ne[2] || n->ne[3] != a->ne[3] || ow < 1 || oh < 1)
                return reject(why, cap, "POOL_2D result must be [%lld, %lld, ne2, ne3]", (long long)ow, (long long)oh);
            return true;
        }
        case SAM3B200_OP_PAD: {
            const int32_t *p = n->op_params;  // lp0, rp0, lp1, rp1, lp2, rp2, lp3, rp3, mode
            if (!a || a->type != SAM3B200_TYPE_F32 || n->type != SAM3B200_TYPE_F32 || !shape_ok(a) || !shape_ok(n) ||
                !strides_ok(a, 4) || !strides_ok(n, 4))
                return reject(why, cap, "PAD: f32 source and result");
            if (p[8] != 0) return reject(why, cap, "PAD: only zero padding is run here");
            for (int d = 0; d < 4; ++d)
                if (p[2 * d] < 0 || p[2 * d + 1] < 0 || n->ne[d] != a->ne[d] + p[2 * d] + p[2 * d + 1])
                    return reject(why, cap, "PAD: result ne%d must be the source's plus its two pads", d);
            return true;
        }
        case SAM3B200_OP_UPSCALE: {
            if (!a || a->type != SAM3B200_TYPE_F32 || n->type != SAM3B200_TYPE_F32 || !shape_ok(a) || !shape_ok(n) ||
                !strides_ok(a, 4) || !strides_ok(n, 4))
                return reject(why, cap, "UPSCALE: f32 source and result");
            if (n->op_params[0] != 0) return reject(why, cap, "UPSCALE mode %d: only nearest (0) is run here", n->op_params[0]);
            for (int d = 0; d < 4; ++d)
                if (n->ne[d] % a->ne[d] != 0 || n->ne[d] >= (1 << 24))
                    return reject(why, cap, "UPSCALE: whole scale factors only (ne%d)", d);
            return true;
        }
        case SAM3B200_OP_CONV_2D_DW: {
            const int32_t *p = n->op_params;  // s0, s1, p0, p1, d0, d1
            if (!a || !b || a->type != SAM3B200_TYPE_F32 || b->type != SAM3B200_TYPE_F32 ||
                n->type != SAM3B200_TYPE_F32 || !shape_ok(a) || !shape_ok(b) || !shape_ok(n) || !strides_ok(a, 4) ||
                !strides_ok(b, 4) || !strides_ok(n, 4))
                return reject(why, cap, "CONV_2D_DW: f32 kernel, input and result");
            if (a->ne[2] != 1 || a->ne[3] != b->ne[2])
                return reject(why, cap, "CONV_2D_DW kernel must be [KW, KH, 1, C] with C = input channels");
            if (p[0] <= 0 || p[1] <= 0 || p[2] < 0 || p[3] < 0 || p[4] <= 0 || p[5] <= 0)
                return reject(why, cap, "CONV_2D_DW stride/padding/dilation (%d %d %d %d %d %d)", p[0], p[1], p[2],
                              p[3], p[4], p[5]);
            const int64_t ow = conv_out(b->ne[0], a->ne[0], p[0], p[2], p[4]);
            const int64_t oh = conv_out(b->ne[1], a->ne[1], p[1], p[3], p[5]);
            if (ow < 1 || oh < 1 || n->ne[0] != ow || n->ne[1] != oh || n->ne[2] != b->ne[2] || n->ne[3] != b->ne[3])
                return reject(why, cap, "CONV_2D_DW result must be [%lld, %lld, C, N]", (long long)ow, (long long)oh);
            return true;
        }
        case SAM3B200_OP_GROUP_NORM: {
            if (!a || a->type != SAM3B200_TYPE_F32 || n->type != SAM3B200_TYPE_F32 || !shape_ok(a) ||
                std::memcmp(n->ne, a->ne, sizeof n->ne) != 0 || !strides_ok(a, 4) || !strides_ok(n, 4))
                return reject(why, cap, "GROUP_NORM: f32 source and result of the same shape");
            if (n->op_params[0] < 1 || !(param_f32(n, 1) >= 0.0f) || n->op_params[0] * a->ne[3] > (1ll << 31) - 1)
                return reject(why, cap, "GROUP_NORM groups %d / eps", n->op_params[0]);
            return true;
        }
        case SAM3B200_OP_FLASH_ATTN_EXT: {
            const T *v = n->src[2], *m = n->src[3];
            if (!a || !b || !v) return reject(why, cap, "FLASH_ATTN_EXT needs q, k and v");
            const int64_t D = a->ne[0], NQ = a->ne[1], NKV = b->ne[1], H = a->ne[2], B = a->ne[3];
            for (const T *t : {a, b, v})
                if (t->type != SAM3B200_TYPE_F32 || !shape_ok(t) || t->nb[0] != 4 || t->nb[1] % 4 || t->nb[2] % 4 ||
                    t->nb[3] % 4)
                    return reject(why, cap, "FLASH_ATTN_EXT q, k, v must be f32 with packed rows");
            if (b->ne[0] != D || v->ne[0] != D || v->ne[1] != NKV || b->ne[2] != H || v->ne[2] != H ||
                b->ne[3] != B || v->ne[3] != B)
                return reject(why, cap, "FLASH_ATTN_EXT k, v must be [D, NKV, heads, batch] of q's D, heads and batch");
            if (!attn_dim_ok(D))
                return reject(why, cap, "FLASH_ATTN_EXT head dim %lld (16, 32, 48, 56, 64, 72, 96, 112, 128, 256)",
                              (long long)D);
            if (NQ > (1 << 24) || NKV > (1 << 24) || H * B > 65535) return reject(why, cap, "FLASH_ATTN_EXT too large");
            if (param_f32(n, 1) != 0.f || param_f32(n, 2) != 0.f)
                return reject(why, cap, "FLASH_ATTN_EXT with max_bias or logit softcap (sam3.cpp uses neither)");
            if (m && (m->type != SAM3B200_TYPE_F16 || !shape_ok(m) || m->ne[0] != NKV || m->ne[1] < NQ ||
                      m->ne[2] != 1 || m->ne[3] != 1 || m->nb[0] != 2 || m->nb[1] % 2))
                return reject(why, cap, "FLASH_ATTN_EXT mask must be F16 [NKV, >= NQ] shared by every head");
            if (n->type != SAM3B200_TYPE_F32 || n->ne[0] != D || n->ne[1] != H || n->ne[2] != NQ || n->ne[3] != B ||
                !contiguous(n))
                return reject(why, cap, "FLASH_ATTN_EXT result must be contiguous f32 [D, heads, NQ, batch]");
            return true;
        }
        case SAM3B200_OP_CONV_TRANSPOSE_2D: {
            if (!a || !b) return reject(why, cap, "CONV_TRANSPOSE_2D needs the kernel and the input");
            const int s = n->op_params[0];
            if (a->type != SAM3B200_TYPE_F16 || !shape_ok(a) || !contiguous(a))
                return reject(why, cap, "CONV_TRANSPOSE_2D kernel must be contiguous F16 [KW, KH, OC, IC]");
            if (b->type != SAM3B200_TYPE_F32 || !shape_ok(b) || !contiguous(b) || b->ne[2] != a->ne[3] ||
                b->ne[3] != 1)
                return reject(why, cap, "CONV_TRANSPOSE_2D input must be contiguous f32 [IW, IH, IC, 1]");
            if (s <= 0) return reject(why, cap, "CONV_TRANSPOSE_2D stride %d", s);
            const int64_t ow = (b->ne[0] - 1) * s + a->ne[0], oh = (b->ne[1] - 1) * s + a->ne[1];
            if (n->type != SAM3B200_TYPE_F32 || n->ne[0] != ow || n->ne[1] != oh || n->ne[2] != a->ne[2] ||
                n->ne[3] != 1 || !contiguous(n))
                return reject(why, cap, "CONV_TRANSPOSE_2D result must be contiguous f32 [%lld, %lld, OC, 1]",
                              (long long)ow, (long long)oh);
            return true;
        }
        case SAM3B200_OP_CONV_2D: {
            if (!a || !b) return reject(why, cap, "CONV_2D needs the kernel and the input");
            const int32_t *p = n->op_params;  // s0, s1, p0, p1, d0, d1
            if (a->type != SAM3B200_TYPE_F16 || !shape_ok(a) || !contiguous(a))
                return reject(why, cap, "CONV_2D kernel must be contiguous F16 [KW, KH, IC, OC]");
            if (b->type != SAM3B200_TYPE_F32 || !shape_ok(b) || !contiguous(b) || b->ne[2] != a->ne[2] ||
                b->ne[3] != 1)
                return reject(why, cap, "CONV_2D input must be contiguous f32 [IW, IH, IC, 1]");
            if (p[0] <= 0 || p[1] <= 0 || p[2] < 0 || p[3] < 0 || p[4] <= 0 || p[5] <= 0)
                return reject(why, cap, "CONV_2D stride/padding/dilation (%d %d %d %d %d %d)", p[0], p[1], p[2],
                              p[3], p[4], p[5]);
            // span of the last kernel start; negative = the dilated kernel overhangs the padded input
            const int64_t span_w = b->ne[0] + 2 * p[2] - p[4] * (a->ne[0] - 1) - 1;
            const int64_t span_h = b->ne[1] + 2 * p[3] - p[5] * (a->ne[1] - 1) - 1;
            if (span_w < 0 || span_h < 0) return reject(why, cap, "CONV_2D kernel larger than the padded input");
            const int64_t ow = span_w / p[0] + 1, oh = span_h / p[1] + 1;
            if (n->type != SAM3B200_TYPE_F32 || n->ne[0] != ow || n->ne[1] != oh || n->ne[2] != a->ne[3] ||
                n->ne[3] != 1 || !contiguous(n))
                return reject(why, cap, "CONV_2D result must be contiguous f32 [%lld, %lld, OC, 1]", (long long)ow,
                              (long long)oh);
            return true;
        }
        case SAM3B200_OP_GET_ROWS: {
            if (!a || !b) return reject(why, cap, "GET_ROWS needs the rows and the indices");
            size_t bb;
            int64_t be;
            if (a->type == SAM3B200_TYPE_I32 || !type_traits(a->type, &bb, &be))
                return reject(why, cap, "GET_ROWS source type %d (F32, F16, Q4_0, Q4_1, Q8_0)", a->type);
            if (!shape_ok(a) || a->ne[2] != 1 || a->ne[3] != 1 || !contiguous(a))
                return reject(why, cap, "GET_ROWS source must be a contiguous 2-D tensor");
            if (b->type != SAM3B200_TYPE_I32 || !shape_ok(b) || b->ne[1] != 1 || b->ne[2] != 1 || b->ne[3] != 1 ||
                !contiguous(b))
                return reject(why, cap, "GET_ROWS indices must be a contiguous I32 vector");
            if (n->type != SAM3B200_TYPE_F32 || n->ne[0] != a->ne[0] || n->ne[1] != b->ne[0] || n->ne[2] != 1 ||
                n->ne[3] != 1 || !contiguous(n))
                return reject(why, cap, "GET_ROWS result must be contiguous f32 [ncols, n]");
            return true;
        }
        default: return reject(why, cap, "op %d is not executed by this backend", n->op);
    }
}

bool computes(const T *n) { return n->op != SAM3B200_OP_NONE && n->op != SAM3B200_OP_VIEW && !is_empty(n); }


}  // namespace
}  // namespace b200

using namespace b200;

extern "C" int sam3b200_supports_op(const sam3b200_tensor *node) {
    char why[256];
    if (node && is_empty(node)) return 1;  // empty nodes run nothing
    return check_node(node, why, sizeof why) ? 1 : 0;
}

namespace b200 {
namespace {

// The ADD at nodes[i] is the bias of the MUL_MAT right before it and runs inside it: it reads that
// MUL_MAT, nothing else reads the MUL_MAT, which is not an output, and the bias is a packed [N] vector.
bool fuses_into_mul_mat(sam3b200_tensor *const *nodes, int i, std::unordered_map<const T *, int> &uses) {
    const T *n = nodes[i];
    if (n->op != SAM3B200_OP_ADD || i == 0) return false;
    const T *mm = n->src[0], *bias = n->src[1];
    return nodes[i - 1] == mm && mm->op == SAM3B200_OP_MUL_MAT && !runtime_src0(mm) &&
           !(mm->flags & SAM3B200_TENSOR_FLAG_OUTPUT) &&
           uses[mm] == 1 && bias->ne[0] == mm->ne[0] && bias->ne[1] == 1 && bias->ne[2] == 1 && bias->ne[3] == 1 &&
           bias->nb[0] == 4 && flat_row_stride(n) != 0;
}

// Alignment the op's kernels need of every data pointer: the tensor-core paths stage through 16-byte
// loads and stores; the element-by-element kernels (return 1) need each tensor aligned to its element.
uintptr_t data_align(const T *n) {
    switch (n->op) {
        case SAM3B200_OP_ADD: case SAM3B200_OP_SUB: case SAM3B200_OP_MUL: case SAM3B200_OP_SCALE:
        case SAM3B200_OP_UNARY: case SAM3B200_OP_NORM: case SAM3B200_OP_SOFT_MAX: case SAM3B200_OP_WIN_PART:
        case SAM3B200_OP_WIN_UNPART: case SAM3B200_OP_CONT: case SAM3B200_OP_REPEAT: case SAM3B200_OP_CONCAT:
        case SAM3B200_OP_IM2COL: case SAM3B200_OP_POOL_2D: case SAM3B200_OP_PAD: case SAM3B200_OP_UPSCALE:
        case SAM3B200_OP_CONV_2D_DW: case SAM3B200_OP_GROUP_NORM: return 1;
        case SAM3B200_OP_MUL_MAT: return runtime_src0(n) ? 1 : 16;
        default: return 16;
    }
}

uintptr_t need_align(const T *n, const T *t) {
    const uintptr_t al = data_align(n), e = elt_size(t->type);
    return al > e ? al : e;
}

bool aligned_to(const void *p, uintptr_t a) { return p && (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

cudaError_t launch_eltwise(b200::Backend *bk, const T *n) {
    const T *a = n->src[0], *b = n->src[1];
    const int64_t total = nelements(n);
    const int threads = 256;
    const int64_t want = (total + threads - 1) / threads, cap_blocks = static_cast<int64_t>(bk->num_sms) * 16;
    const unsigned blocks = static_cast<unsigned>(want < cap_blocks ? want : cap_blocks);
    const Shape4 sb = b ? shape_of(b) : shape_of(a);
    eltwise_kernel<<<blocks, threads, 0, bk->stream>>>(
        n->op, n->op_params[0], param_f32(n, 0),
        (a->type == SAM3B200_TYPE_F16 ? 1 : 0) | (n->type == SAM3B200_TYPE_F16 ? 2 : 0),
        static_cast<const char *>(a->data), shape_of(a), b ? static_cast<const char *>(b->data) : nullptr, sb,
        static_cast<char *>(n->data), shape_of(n), total);
    bk->count(1);
    return cudaGetLastError();
}

cudaError_t launch_soft_max(b200::Backend *bk, const T *n) {
    const T *a = n->src[0], *m = n->src[1];
    const int64_t rows = a->ne[1] * a->ne[2] * a->ne[3];
    const unsigned blocks = static_cast<unsigned>((rows + 7) / 8);
    soft_max_rows_kernel<<<blocks, 256, 0, bk->stream>>>(
        static_cast<const char *>(a->data), shape_of(a), m ? static_cast<const char *>(m->data) : nullptr,
        m ? shape_of(m) : shape_of(a), m && m->type == SAM3B200_TYPE_F16 ? 1 : 0, static_cast<char *>(n->data),
        shape_of(n), rows, param_f32(n, 0));
    bk->count(1);
    return cudaGetLastError();
}

cudaError_t launch_win(b200::Backend *bk, const T *n) {
    const bool part = n->op == SAM3B200_OP_WIN_PART;
    const T *a = n->src[0], *map = part ? a : n;
    const int64_t w = part ? n->op_params[2] : n->op_params[0];
    const int64_t total = nelements(n);
    const int64_t want = (total + 255) / 256, cap_blocks = static_cast<int64_t>(bk->num_sms) * 16;
    win_kernel<<<static_cast<unsigned>(want < cap_blocks ? want : cap_blocks), 256, 0, bk->stream>>>(
        part ? 0 : 1, static_cast<const float *>(a->data), static_cast<float *>(n->data), map->ne[0], map->ne[1],
        map->ne[2], w, (map->ne[1] + w - 1) / w, total);
    bk->count(1);
    return cudaGetLastError();
}

cudaError_t launch_norm(b200::Backend *bk, const T *n) {
    const T *a = n->src[0];
    const int64_t rows = a->ne[1] * a->ne[2] * a->ne[3];
    const unsigned blocks = static_cast<unsigned>((rows + 7) / 8);  // 8 warps, one row each
    norm_rows_kernel<<<blocks, 256, 0, bk->stream>>>(static_cast<const char *>(a->data), shape_of(a),
                                                     static_cast<char *>(n->data), shape_of(n), rows,
                                                     param_f32(n, 0));
    bk->count(1);
    return cudaGetLastError();
}

unsigned grid_for(const b200::Backend *bk, int64_t total) {
    const int64_t want = (total + 255) / 256, cap_blocks = static_cast<int64_t>(bk->num_sms) * 16;
    return static_cast<unsigned>(want < cap_blocks ? want : cap_blocks);
}

const char *cdata(const T *t) { return static_cast<const char *>(t->data); }
char *mdata(const T *t) { return static_cast<char *>(t->data); }

// The shape-moving and convolution ops of the graph, one element-parallel kernel each.
cudaError_t launch_layout(b200::Backend *bk, const T *n) {
    const T *a = n->src[0], *b = n->src[1];
    const int64_t total = nelements(n);
    const unsigned g = grid_for(bk, total);
    const int32_t *p = n->op_params;
    cudaStream_t s = bk->stream;
    switch (n->op) {
        case SAM3B200_OP_CONCAT:
            concat_kernel<<<g, 256, 0, s>>>(cdata(a), shape_of(a), cdata(b), shape_of(b), mdata(n), shape_of(n), p[0],
                                            total);
            break;
        case SAM3B200_OP_IM2COL:
            im2col_kernel<<<g, 256, 0, s>>>(cdata(b), shape_of(b), b->type == SAM3B200_TYPE_F16, mdata(n), shape_of(n),
                                            n->type == SAM3B200_TYPE_F16, static_cast<int>(a->ne[0]),
                                            static_cast<int>(a->ne[1]), p[0], p[1], p[2], p[3], p[4], p[5], total);
            break;
        case SAM3B200_OP_POOL_2D:
            pool2d_kernel<<<g, 256, 0, s>>>(cdata(a), shape_of(a), a->type == SAM3B200_TYPE_F16, mdata(n), shape_of(n),
                                            p[0], p[1], p[2], p[3], p[4], p[5], p[6], total);
            break;
        case SAM3B200_OP_PAD: {
            Pad4 pad;
            for (int d = 0; d < 4; ++d) pad.lp[d] = p[2 * d];
            pad_kernel<<<g, 256, 0, s>>>(cdata(a), shape_of(a), mdata(n), shape_of(n), pad, total);
            break;
        }
        case SAM3B200_OP_UPSCALE:
            upscale_kernel<<<g, 256, 0, s>>>(cdata(a), shape_of(a), mdata(n), shape_of(n), total);
            break;
        case SAM3B200_OP_CONV_2D_DW:
            conv2d_dw_kernel<<<g, 256, 0, s>>>(cdata(a), shape_of(a), cdata(b), shape_of(b), mdata(n), shape_of(n),
                                               p[0], p[1], p[2], p[3], p[4], p[5], total);
            break;
        case SAM3B200_OP_GROUP_NORM:
            group_norm_kernel<<<static_cast<unsigned>(p[0] * a->ne[3]), 256, 0, s>>>(cdata(a), shape_of(a), mdata(n),
                                                                                   shape_of(n), p[0], param_f32(n, 1));
            break;
        default: return cudaErrorInvalidValue;
    }
    bk->count(1);
    return cudaGetLastError();
}

// MUL_MAT of two graph tensors.  A 2-D F16 src0 (an IM2COL result: ggml_conv_2d's contraction, and the
// patch embedding of sam3.cpp:6726-6742) with rows that flatten runs on the fp16 tensor-core GEMM: both
// operands rounded to fp16 (K zero-padded to a multiple of 8) in the backend's scratch, fp32 accumulation
// -- ggml-cpu's arithmetic for F16 rows.  Everything else runs mul_mat_rt_kernel.
int run_mul_mat_rt(b200::Backend *bk, const T *n) {
    const T *a = n->src[0], *b = n->src[1];
    const int64_t K = a->ne[0], N = a->ne[1], M = rows_of(b);
    const size_t lda = flat_row_stride(a), ldb = flat_row_stride(b), ldd = flat_row_stride(n);
    const bool tc = a->type == SAM3B200_TYPE_F16 && a->ne[2] == 1 && a->ne[3] == 1 && lda && ldb && ldd &&
                    M >= 128 && N >= 64 && K >= 32 && M <= (1 << 24) && N <= (1 << 24) && K <= (1 << 20);
    if (tc) {
        const int64_t Kp = (K + 7) / 8 * 8;
        const size_t bytes_x = static_cast<size_t>(M * Kp) * 2, bytes_w = static_cast<size_t>(N * Kp) * 2;
        if (!bk->ensure_scratch(bytes_x + bytes_w, 16)) return SAM3B200_STATUS_ALLOC_FAILED;
        __half *xs = static_cast<__half *>(bk->act_codes);
        __half *ws = reinterpret_cast<__half *>(static_cast<char *>(bk->act_codes) + bytes_x);
        rows_to_f16_padded_kernel<<<grid_for(bk, M * Kp), 256, 0, bk->stream>>>(
            cdata(b), static_cast<int64_t>(ldb), b->type == SAM3B200_TYPE_F16, M, K, Kp, xs);
        rows_to_f16_padded_kernel<<<grid_for(bk, N * Kp), 256, 0, bk->stream>>>(cdata(a), static_cast<int64_t>(lda), 1,
                                                                               N, K, Kp, ws);
        GemmF16Args g;
        g.a = xs;
        g.b = ws;
        g.M = static_cast<int>(M);
        g.N = static_cast<int>(N);
        g.K = static_cast<int>(Kp);
        g.bias = nullptr;
        g.gelu = 0;
        g.out_f16 = 0;
        g.out = n->data;
        g.ldo = static_cast<int64_t>(ldd / 4);
        g.store = GEMM_STORE_ROWMAJOR;
        g.win = 0;
        g.cout = 0;
        g.err = bk->err;
        bk->count(3);
        if (!cuda_ok(cudaGetLastError(), "graph mul_mat operands to f16") ||
            !cuda_ok(gemm_f16(g, bk->num_sms, bk->stream), "graph mul_mat f16 gemm"))
            return SAM3B200_STATUS_FAILED;
        return SAM3B200_STATUS_SUCCESS;
    }
    const dim3 grid(static_cast<unsigned>((N + RT_TILE - 1) / RT_TILE),
                    static_cast<unsigned>((b->ne[1] + RT_TILE - 1) / RT_TILE),
                    static_cast<unsigned>(n->ne[2] * n->ne[3]));
    mul_mat_rt_kernel<<<grid, 256, 0, bk->stream>>>(cdata(a), shape_of(a), a->type == SAM3B200_TYPE_F16, cdata(b),
                                                    shape_of(b), b->type == SAM3B200_TYPE_F16, mdata(n), shape_of(n), K);
    bk->count(1);
    return cuda_ok(cudaGetLastError(), "graph mul_mat") ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
}

}  // namespace
}  // namespace b200

extern "C" int sam3b200_graph_compute(sam3b200_backend *h, sam3b200_tensor *const *nodes, int n_nodes) {
    if (n_nodes < 0 || (n_nodes > 0 && !nodes)) {
        set_error("graph_compute: null node list");
        return SAM3B200_STATUS_FAILED;
    }
    char why[256];
    // pass 1: every node on its own
    std::unordered_map<const T *, int> uses;
    for (int i = 0; i < n_nodes; ++i) {
        const T *n = nodes[i];
        if (!n) {
            set_error("graph_compute: node %d is null", i);
            return SAM3B200_STATUS_FAILED;
        }
        for (const T *s : n->src)
            if (s) ++uses[s];
    }
    for (int i = 0; i < n_nodes; ++i) {
        const T *n = nodes[i];
        if (is_empty(n)) continue;
        if (!check_node(n, why, sizeof why)) {
            set_error("graph_compute: node %d rejected: %s", i, why);
            return SAM3B200_STATUS_FAILED;
        }
    }
    std::vector<char> fused(n_nodes + 1, 0);  // fused[i]: node i is an ADD running inside node i - 1
    for (int i = 0; i < n_nodes; ++i)
        if (!is_empty(nodes[i]) && fuses_into_mul_mat(nodes, i, uses)) fused[i] = 1;
    // pass 2: device data of every node that computes, and the uploaded weights
    for (int i = 0; i < n_nodes; ++i) {
        const T *n = nodes[i];
        if (!computes(n)) continue;
        const bool writes_own = !(n->op == SAM3B200_OP_MUL_MAT && fused[i + 1]);
        if (writes_own && !aligned_to(n->data, need_align(n, n))) {
            set_error("graph_compute: node %d rejected: result data is null or not %d-byte aligned", i,
                      static_cast<int>(need_align(n, n)));
            return SAM3B200_STATUS_FAILED;
        }
        for (int s = 0; s < 4; ++s) {
            const T *src = n->src[s];
            // a weight is read through its handle; IM2COL reads only its kernel's shape
            if (!src || (n->op == SAM3B200_OP_MUL_MAT && s == 0 && !runtime_src0(n)) ||
                (n->op == SAM3B200_OP_IM2COL && s == 0) || (fused[i] && s == 0))
                continue;
            const uintptr_t al = fused[i] ? 16 : need_align(n, src);
            if (!aligned_to(src->data, al)) {
                set_error("graph_compute: node %d rejected: src%d data is null or not %d-byte aligned", i, s,
                          static_cast<int>(al));
                return SAM3B200_STATUS_FAILED;
            }
        }
        if (n->op == SAM3B200_OP_MUL_MAT && !runtime_src0(n)) {
            const T *wt = n->src[0];
            const auto *w = static_cast<const Weight *>(wt->extra);
            if (!w) {
                set_error("graph_compute: node %d rejected: MUL_MAT weight has no handle from sam3b200_weight_upload "
                          "in extra",
                          i);
                return SAM3B200_STATUS_FAILED;
            }
            if (w->type != wt->type || w->K != wt->ne[0] || w->N != wt->ne[1]) {
                set_error("graph_compute: node %d rejected: MUL_MAT weight handle is type %d [%d, %d], the node says "
                          "type %d [%lld, %lld]",
                          i, w->type, w->K, w->N, wt->type, (long long)wt->ne[0], (long long)wt->ne[1]);
                return SAM3B200_STATUS_FAILED;
            }
        }
    }
    auto *be = reinterpret_cast<sam3b200_backend *>(h);
    if (!be) {
        set_error("graph_compute: null backend");
        return SAM3B200_STATUS_FAILED;
    }
    auto *bk = reinterpret_cast<Backend *>(h);
    cudaSetDevice(bk->device);
    // run the nodes in order
    for (int i = 0; i < n_nodes; ++i) {
        const T *n = nodes[i];
        if (!computes(n) || fused[i]) continue;
        const T *a = n->src[0], *b = n->src[1];
        int st = SAM3B200_STATUS_SUCCESS;
        switch (n->op) {
            case SAM3B200_OP_MUL_MAT: {
                if (runtime_src0(n)) {
                    st = run_mul_mat_rt(bk, n);
                    break;
                }
                // a bias add right after it runs inside it, writing the ADD's result
                const T *add = fused[i + 1] ? nodes[i + 1] : nullptr;
                const T *out = add ? add : n;
                st = sam3b200_mul_mat(be, static_cast<const sam3b200_weight *>(a->extra),
                                      static_cast<const float *>(b->data), static_cast<int64_t>(flat_row_stride(b) / 4),
                                      rows_of(b), add ? static_cast<const float *>(add->src[1]->data) : nullptr,
                                      static_cast<float *>(out->data), static_cast<int64_t>(flat_row_stride(out) / 4));
                break;
            }
            case SAM3B200_OP_ADD:
            case SAM3B200_OP_SUB:
            case SAM3B200_OP_MUL:
            case SAM3B200_OP_SCALE:
            case SAM3B200_OP_UNARY:
            case SAM3B200_OP_CONT:
            case SAM3B200_OP_REPEAT:
                if (!cuda_ok(launch_eltwise(bk, n), "graph elementwise")) st = SAM3B200_STATUS_FAILED;
                break;
            case SAM3B200_OP_CONCAT:
            case SAM3B200_OP_IM2COL:
            case SAM3B200_OP_POOL_2D:
            case SAM3B200_OP_PAD:
            case SAM3B200_OP_UPSCALE:
            case SAM3B200_OP_CONV_2D_DW:
            case SAM3B200_OP_GROUP_NORM:
                if (!cuda_ok(launch_layout(bk, n), "graph layout / convolution op")) st = SAM3B200_STATUS_FAILED;
                break;
            case SAM3B200_OP_NORM:
                if (!cuda_ok(launch_norm(bk, n), "graph norm")) st = SAM3B200_STATUS_FAILED;
                break;
            case SAM3B200_OP_SOFT_MAX:
                if (!cuda_ok(launch_soft_max(bk, n), "graph soft_max")) st = SAM3B200_STATUS_FAILED;
                break;
            case SAM3B200_OP_WIN_PART:
            case SAM3B200_OP_WIN_UNPART:
                if (!cuda_ok(launch_win(bk, n), "graph win_part")) st = SAM3B200_STATUS_FAILED;
                break;
            case SAM3B200_OP_FLASH_ATTN_EXT: {
                const T *v = n->src[2], *m = n->src[3];
                const int64_t qn[3] = {static_cast<int64_t>(a->nb[1] / 4), static_cast<int64_t>(a->nb[2] / 4),
                                       static_cast<int64_t>(a->nb[3] / 4)};
                const int64_t kn[3] = {static_cast<int64_t>(b->nb[1] / 4), static_cast<int64_t>(b->nb[2] / 4),
                                       static_cast<int64_t>(b->nb[3] / 4)};
                const int64_t vn[3] = {static_cast<int64_t>(v->nb[1] / 4), static_cast<int64_t>(v->nb[2] / 4),
                                       static_cast<int64_t>(v->nb[3] / 4)};
                st = sam3b200_flash_attn_ext_view(be, static_cast<const float *>(a->data),
                                                  static_cast<const float *>(b->data),
                                                  static_cast<const float *>(v->data), m ? m->data : nullptr,
                                                  m ? static_cast<int64_t>(m->nb[1] / 2) : 0, a->ne[0], a->ne[1],
                                                  b->ne[1], a->ne[2], a->ne[3], qn, kn, vn, param_f32(n, 0),
                                                  static_cast<float *>(n->data));
                break;
            }
            case SAM3B200_OP_CONV_TRANSPOSE_2D:
                st = sam3b200_conv_transpose_2d(be, a->data, static_cast<const float *>(b->data), b->ne[0], b->ne[1],
                                                b->ne[2], a->ne[2], a->ne[0], a->ne[1], n->op_params[0],
                                                static_cast<float *>(n->data));
                break;
            case SAM3B200_OP_CONV_2D: {
                const int32_t *p = n->op_params;
                st = sam3b200_conv_2d(be, a->data, static_cast<const float *>(b->data), b->ne[0], b->ne[1], b->ne[2],
                                      a->ne[3], a->ne[0], a->ne[1], p[0], p[1], p[2], p[3], p[4], p[5],
                                      static_cast<float *>(n->data));
                break;
            }
            case SAM3B200_OP_GET_ROWS:
                st = sam3b200_get_rows(be, a->type, a->data, a->ne[0], a->ne[1], static_cast<const int32_t *>(b->data),
                                       b->ne[0], static_cast<float *>(n->data));
                break;
            default: break;
        }
        if (st != SAM3B200_STATUS_SUCCESS) {
            const std::string msg = sam3b200_last_error();
            sam3b200_backend_synchronize(be);  // let the nodes already queued finish before returning
            set_error("graph_compute: node %d failed: %s", i, msg.c_str());
            return st;
        }
    }
    return sam3b200_backend_synchronize(be);
}
