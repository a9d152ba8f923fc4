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

#include <cuda_fp16.h>

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

// Byte stride between consecutive rows of an f32 tensor whose dims 1..3 are
// read as one run of ne1*ne2*ne3 rows (ggml_mul_mat broadcasting a 2-D weight
// over them); 0 if those dims do not flatten to one evenly strided run or the
// elements of a row are not packed.
size_t flat_row_stride(const T *t) {
    if (t->type != SAM3B200_TYPE_F32 || t->nb[0] != 4) return 0;
    size_t stride = 0, next = 0;
    for (int d = 1; d < 4; ++d) {
        if (t->ne[d] == 1) continue;
        if (stride == 0) stride = t->nb[d];
        else if (t->nb[d] != next) return 0;
        next = t->nb[d] * static_cast<size_t>(t->ne[d]);
    }
    if (stride == 0) stride = static_cast<size_t>(t->ne[0]) * 4;  // one row
    if (stride % 4 != 0 || stride < static_cast<size_t>(t->ne[0]) * 4) return 0;
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

__global__ void eltwise_kernel(int op, int unary, float scale, int f16, const char *__restrict__ a, Shape4 sa,
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
            const int64_t oa = offset_of(i, sa);
            if (f16) *reinterpret_cast<__half *>(d + od) = *reinterpret_cast<const __half *>(a + oa);
            else *reinterpret_cast<float *>(d + od) = *reinterpret_cast<const float *>(a + oa);
            continue;
        }
        const float x = *reinterpret_cast<const float *>(a + c[0] * sa.nb[0] + c[1] * sa.nb[1] + c[2] * sa.nb[2] +
                                                         c[3] * sa.nb[3]);
        float y = x;
        if (op == SAM3B200_OP_ADD || op == SAM3B200_OP_MUL) {
            int64_t ob = 0;
#pragma unroll
            for (int k = 0; k < 4; ++k) ob += (c[k] % sb.ne[k]) * sb.nb[k];
            const float v = *reinterpret_cast<const float *>(b + ob);
            y = op == SAM3B200_OP_ADD ? __fadd_rn(x, v) : __fmul_rn(x, v);
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

bool strides_ok(const T *t, size_t elt) {
    for (int d = 0; d < 4; ++d)
        if (t->nb[d] % elt != 0 || t->nb[d] == 0) return false;
    return true;
}

int64_t nelements(const T *t) { return t->ne[0] * t->ne[1] * t->ne[2] * t->ne[3]; }

// The node-local rules of each op; on failure `why` says which.
bool check_node(const T *n, char *why, size_t cap) {
    if (!n) return reject(why, cap, "null node");
    const T *a = n->src[0], *b = n->src[1];
    switch (n->op) {
        case SAM3B200_OP_NONE: return true;
        case SAM3B200_OP_VIEW: return a ? true : reject(why, cap, "VIEW without a source");
        case SAM3B200_OP_MUL_MAT: {
            if (!a || !b) return reject(why, cap, "MUL_MAT needs src0 (weight) and src1 (x)");
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
        case SAM3B200_OP_MUL: {
            const char *name = n->op == SAM3B200_OP_ADD ? "ADD" : "MUL";
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
            if (!a || !shape_ok(a) || !shape_ok(n) || a->type != n->type ||
                (a->type != SAM3B200_TYPE_F32 && a->type != SAM3B200_TYPE_F16) || nelements(a) != nelements(n))
                return reject(why, cap, "CONT: F32 or F16 source and result of one type and element count");
            const size_t elt = a->type == SAM3B200_TYPE_F32 ? 4 : 2;
            if (!strides_ok(a, elt) || !strides_ok(n, elt)) return reject(why, cap, "CONT: strides must be whole elements");
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
    return nodes[i - 1] == mm && mm->op == SAM3B200_OP_MUL_MAT && !(mm->flags & SAM3B200_TENSOR_FLAG_OUTPUT) &&
           uses[mm] == 1 && bias->ne[0] == mm->ne[0] && bias->ne[1] == 1 && bias->ne[2] == 1 && bias->ne[3] == 1 &&
           bias->nb[0] == 4 && flat_row_stride(n) != 0;
}

// Alignment the op's kernels need of every data pointer: the tensor-core paths stage through 16-byte
// loads and stores, the elementwise ops read and write single elements.
uintptr_t data_align(const T *n) {
    switch (n->op) {
        case SAM3B200_OP_ADD: case SAM3B200_OP_MUL: case SAM3B200_OP_SCALE: case SAM3B200_OP_UNARY:
        case SAM3B200_OP_NORM: case SAM3B200_OP_SOFT_MAX: case SAM3B200_OP_WIN_PART:
        case SAM3B200_OP_WIN_UNPART: return 4;
        case SAM3B200_OP_CONT: return n->type == SAM3B200_TYPE_F16 ? 2 : 4;
        default: return 16;
    }
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
        n->op, n->op_params[0], param_f32(n, 0), n->type == SAM3B200_TYPE_F16 ? 1 : 0,
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
        const uintptr_t al = data_align(n);
        const bool writes_own = !(n->op == SAM3B200_OP_MUL_MAT && fused[i + 1]);
        if (writes_own && !aligned_to(n->data, al)) {
            set_error("graph_compute: node %d rejected: result data is null or not %d-byte aligned", i,
                      static_cast<int>(al));
            return SAM3B200_STATUS_FAILED;
        }
        for (int s = 0; s < 4; ++s) {
            const T *src = n->src[s];
            if (!src || (n->op == SAM3B200_OP_MUL_MAT && s == 0) || (fused[i] && s == 0)) continue;
            if (!aligned_to(src->data, fused[i] ? 16 : al)) {
                set_error("graph_compute: node %d rejected: src%d data is null or not %d-byte aligned", i, s,
                          static_cast<int>(fused[i] ? 16 : al));
                return SAM3B200_STATUS_FAILED;
            }
        }
        if (n->op == SAM3B200_OP_MUL_MAT) {
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
            case SAM3B200_OP_MUL:
            case SAM3B200_OP_SCALE:
            case SAM3B200_OP_UNARY:
            case SAM3B200_OP_CONT:
                if (!cuda_ok(launch_eltwise(bk, n), "graph elementwise")) st = SAM3B200_STATUS_FAILED;
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
