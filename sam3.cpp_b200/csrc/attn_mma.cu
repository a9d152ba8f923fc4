// attn_mma.cu -- attention on the tensor cores for the runners whose shapes
// the tcgen05 flash kernel (attn.cu: head dim 64, self-attention, no mask)
// does not take: head dims 32 / 64 / 128 / 256, any query and key counts,
// strided operands, an optional additive mask (fp16 shared by the heads, or
// f32 per head).
//
// Flash-attention loop with warp-level mma.sync m16n8k16 (fp16 operands, fp32
// accumulation): a CTA holds 64 query rows (4 warps x 16) and walks the keys
// in tiles of 64 staged in shared memory as fp16 (K row-major, V transposed);
// S = Q K^T and O += P V run on the tensor cores, the online softmax (base 2,
// fp32) in registers.  Q, K and V are rounded to fp16 and P to fp16 for the
// second product, the scores and the output accumulate in fp32.
#include "attn_mma.cuh"

#include <cmath>
#include <cuda_fp16.h>

namespace b200 {
namespace {

constexpr int BQ = 64, BK = 64, NTHREADS = 128;

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t ld32(const __half *p) { return *reinterpret_cast<const uint32_t *>(p); }

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&h);
}

__device__ __forceinline__ float mask_f(__half m) { return __half2float(m); }
__device__ __forceinline__ float mask_f(float m) { return m; }

__device__ __forceinline__ __half to_half(float x) { return __float2half_rn(x); }
__device__ __forceinline__ __half to_half(__half x) { return x; }

// KVT: f32 or fp16 keys / values.  Split-KV (gridDim.z > 1): split z takes
// keys [z * chunk, (z + 1) * chunk) and writes its unnormalised accumulator
// and (max, sum) per row to part_o / part_ml instead of o; attn_combine_kernel
// merges the splits.
template <int D, typename KVT, typename MT>
__global__ void __launch_bounds__(NTHREADS) attn_mma_kernel(const float *__restrict__ q, AttnStrides qs, int NQ,
                                                            const KVT *__restrict__ k, AttnStrides ks,
                                                            const KVT *__restrict__ v, AttnStrides vs, int NKV,
                                                            int heads, const MT *__restrict__ mask, int64_t mask_ld,
                                                            int64_t mask_hs, float scale_log2, float *__restrict__ o,
                                                            AttnStrides os, int chunk, float *__restrict__ part_o,
                                                            float2 *__restrict__ part_ml) {
    constexpr int DP = D + 8;   // shared row pitch (halves) of Q and K: fragment loads hit distinct banks
    constexpr int KP = BK + 8;  // shared row pitch of V^T
    constexpr int DT = D / 8;   // 8-wide output column tiles per warp
    constexpr float LOG2E = 1.4426950408889634f;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __half *qsm = reinterpret_cast<__half *>(smem_raw);  // [BQ][DP]
    __half *ksm = qsm + BQ * DP;                          // [BK][DP]
    __half *vts = ksm + BK * DP;                          // [D][KP]
    const int b = blockIdx.y / heads, h = blockIdx.y % heads;
    const int q0 = blockIdx.x * BQ;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t4 = lane & 3;
    const float *qb = q + b * qs.b + h * qs.h;
    const KVT *kb = k + b * ks.b + h * ks.h;
    const KVT *vb = v + b * vs.b + h * vs.h;
    const int kv_lo = blockIdx.z * chunk, kv_hi = min(NKV, kv_lo + chunk);

    for (int e = threadIdx.x; e < BQ * D; e += NTHREADS) {
        const int r = e / D, d = e % D, row = q0 + r;
        qsm[r * DP + d] = __float2half_rn(row < NQ ? qb[static_cast<int64_t>(row) * qs.n + d] : 0.f);
    }
    const int rw = warp * 16 + g;  // this thread's tile rows rw and rw + 8
    const int row_a = q0 + rw, row_b = row_a + 8;
    const MT *mh = mask ? mask + h * mask_hs : nullptr;  // the head's mask (mask_hs 0: shared by the heads)
    const MT *mrow_a = mh && row_a < NQ ? mh + static_cast<int64_t>(row_a) * mask_ld : nullptr;
    const MT *mrow_b = mh && row_b < NQ ? mh + static_cast<int64_t>(row_b) * mask_ld : nullptr;

    float oacc[DT][4];
#pragma unroll
    for (int i = 0; i < DT; ++i) oacc[i][0] = oacc[i][1] = oacc[i][2] = oacc[i][3] = 0.f;
    float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;

    for (int j0 = kv_lo; j0 < kv_hi; j0 += BK) {
        __syncthreads();
        for (int e = threadIdx.x; e < BK * D; e += NTHREADS) {
            const int kk = e / D, d = e % D, key = j0 + kk;
            __half kv = __float2half_rn(0.f), vv = kv;
            if (key < kv_hi) {
                kv = to_half(kb[static_cast<int64_t>(key) * ks.n + d]);
                vv = to_half(vb[static_cast<int64_t>(key) * vs.n + d]);
            }
            ksm[kk * DP + d] = kv;
            vts[d * KP + kk] = vv;
        }
        __syncthreads();
        // S = Q K^T for this warp's 16 rows x 64 keys
        float sacc[8][4];
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.f;
#pragma unroll 4
        for (int kt = 0; kt < D / 16; ++kt) {
            const __half *qa = qsm + rw * DP + kt * 16 + t4 * 2;
            const uint32_t a0 = ld32(qa), a1 = ld32(qa + 8 * DP), a2 = ld32(qa + 8), a3 = ld32(qa + 8 * DP + 8);
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
                const __half *kp = ksm + (nt * 8 + g) * DP + kt * 16 + t4 * 2;
                mma16816(sacc[nt], a0, a1, a2, a3, ld32(kp), ld32(kp + 8));
            }
        }
        // scale, bounds, mask; online softmax for rows a (c = 0, 1) and b (c = 2, 3)
        float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int key = j0 + nt * 8 + t4 * 2 + (c & 1);
                float s = sacc[nt][c] * scale_log2;
                const MT *mr = c < 2 ? mrow_a : mrow_b;
                if (key >= kv_hi) {
                    s = -INFINITY;
                } else if (mr) {
                    const float mv = mask_f(mr[key]);
                    s = mv == -INFINITY ? -INFINITY : fmaf(mv, LOG2E, s);
                }
                sacc[nt][c] = s;
            }
            mx_a = fmaxf(mx_a, fmaxf(sacc[nt][0], sacc[nt][1]));
            mx_b = fmaxf(mx_b, fmaxf(sacc[nt][2], sacc[nt][3]));
        }
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
        const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
        const float al_a = mn_a == -INFINITY ? 1.f : exp2f(m_a - mn_a);
        const float al_b = mn_b == -INFINITY ? 1.f : exp2f(m_b - mn_b);
        const float ms_a = mn_a == -INFINITY ? 0.f : mn_a, ms_b = mn_b == -INFINITY ? 0.f : mn_b;
        m_a = mn_a;
        m_b = mn_b;
        l_a *= al_a;
        l_b *= al_b;
#pragma unroll
        for (int i = 0; i < DT; ++i) {
            oacc[i][0] *= al_a;
            oacc[i][1] *= al_a;
            oacc[i][2] *= al_b;
            oacc[i][3] *= al_b;
        }
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            sacc[nt][0] = exp2f(sacc[nt][0] - ms_a);
            sacc[nt][1] = exp2f(sacc[nt][1] - ms_a);
            sacc[nt][2] = exp2f(sacc[nt][2] - ms_b);
            sacc[nt][3] = exp2f(sacc[nt][3] - ms_b);
            l_a += sacc[nt][0] + sacc[nt][1];
            l_b += sacc[nt][2] + sacc[nt][3];
        }
        // O += P V: P's accumulator layout is the A-fragment layout of 16-key steps
#pragma unroll
        for (int ks2 = 0; ks2 < 4; ++ks2) {
            const uint32_t a0 = pack_half2(sacc[2 * ks2][0], sacc[2 * ks2][1]);
            const uint32_t a1 = pack_half2(sacc[2 * ks2][2], sacc[2 * ks2][3]);
            const uint32_t a2 = pack_half2(sacc[2 * ks2 + 1][0], sacc[2 * ks2 + 1][1]);
            const uint32_t a3 = pack_half2(sacc[2 * ks2 + 1][2], sacc[2 * ks2 + 1][3]);
#pragma unroll
            for (int dt = 0; dt < DT; ++dt) {
                const __half *vp = vts + (dt * 8 + g) * KP + ks2 * 16 + t4 * 2;
                mma16816(oacc[dt], a0, a1, a2, a3, ld32(vp), ld32(vp + 8));
            }
        }
    }
    l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
    l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
    if (part_o) {  // split-KV partial: unnormalised accumulator + (max, sum) per row
        const int64_t base = (static_cast<int64_t>(blockIdx.z) * gridDim.y + blockIdx.y) * NQ;
        if (t4 == 0) {
            if (row_a < NQ) part_ml[base + row_a] = make_float2(m_a, l_a);
            if (row_b < NQ) part_ml[base + row_b] = make_float2(m_b, l_b);
        }
#pragma unroll
        for (int dt = 0; dt < DT; ++dt) {
            const int d = dt * 8 + t4 * 2;
            if (row_a < NQ) *reinterpret_cast<float2 *>(part_o + (base + row_a) * D + d) = make_float2(oacc[dt][0], oacc[dt][1]);
            if (row_b < NQ) *reinterpret_cast<float2 *>(part_o + (base + row_b) * D + d) = make_float2(oacc[dt][2], oacc[dt][3]);
        }
        return;
    }
    const float inv_a = l_a > 0.f ? 1.f / l_a : 0.f, inv_b = l_b > 0.f ? 1.f / l_b : 0.f;
    float *ob = o + b * os.b + h * os.h;
#pragma unroll
    for (int dt = 0; dt < DT; ++dt) {
        const int d = dt * 8 + t4 * 2;
        if (row_a < NQ) {
            ob[static_cast<int64_t>(row_a) * os.n + d] = oacc[dt][0] * inv_a;
            ob[static_cast<int64_t>(row_a) * os.n + d + 1] = oacc[dt][1] * inv_a;
        }
        if (row_b < NQ) {
            ob[static_cast<int64_t>(row_b) * os.n + d] = oacc[dt][2] * inv_b;
            ob[static_cast<int64_t>(row_b) * os.n + d + 1] = oacc[dt][3] * inv_b;
        }
    }
}

// out(row, :) = sum_z 2^(m_z - M) acc_z / sum_z 2^(m_z - M) l_z over the splits (M = max_z m_z)
template <int D>
__global__ void attn_combine_kernel(const float *__restrict__ part_o, const float2 *__restrict__ part_ml, int splits,
                                    int NQ, int heads, float *__restrict__ o, AttnStrides os) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t BH = static_cast<int64_t>(gridDim.y);
    if (i >= static_cast<int64_t>(NQ) * D) return;
    const int row = static_cast<int>(i / D), d = static_cast<int>(i % D), bh = blockIdx.y;
    float M = -INFINITY;
    for (int z = 0; z < splits; ++z) M = fmaxf(M, part_ml[(z * BH + bh) * NQ + row].x);
    float num = 0.f, den = 0.f;
    if (M != -INFINITY)
        for (int z = 0; z < splits; ++z) {
            const int64_t r = (z * BH + bh) * NQ + row;
            const float2 ml = part_ml[r];
            const float w = ml.x == -INFINITY ? 0.f : exp2f(ml.x - M);
            num = fmaf(w, part_o[r * D + d], num);
            den = fmaf(w, ml.y, den);
        }
    const int b = bh / heads, h = bh % heads;
    o[b * os.b + h * os.h + static_cast<int64_t>(row) * os.n + d] = den > 0.f ? num / den : 0.f;
}

template <int D, typename KVT, typename MT = __half>
cudaError_t launch_mma(const float *q, AttnStrides qs, int NQ, const KVT *k, AttnStrides ks, const KVT *v,
                       AttnStrides vs, int NKV, int batch, int heads, const MT *mask, int64_t mask_ld, float scale,
                       float *o, AttnStrides os, int splits, float *part_o, float2 *part_ml, cudaStream_t s,
                       int64_t mask_hs = 0) {
    const int smem = ((BQ + BK) * (D + 8) + D * (BK + 8)) * 2;
    cudaError_t e =
        cudaFuncSetAttribute(attn_mma_kernel<D, KVT, MT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    const int chunk = splits > 1 ? ((NKV + splits - 1) / splits + BK - 1) / BK * BK : NKV;
    const int nz = (NKV + chunk - 1) / chunk;
    dim3 grid((NQ + BQ - 1) / BQ, static_cast<unsigned>(batch * heads), static_cast<unsigned>(nz));
    attn_mma_kernel<D, KVT, MT><<<grid, NTHREADS, smem, s>>>(q, qs, NQ, k, ks, v, vs, NKV, heads, mask, mask_ld,
                                                              mask_hs, scale * 1.4426950408889634f, o, os, chunk,
                                                          nz > 1 ? part_o : nullptr, part_ml);
    if ((e = cudaGetLastError()) != cudaSuccess || nz == 1) return e;
    dim3 cgrid(static_cast<unsigned>((static_cast<int64_t>(NQ) * D + 255) / 256), static_cast<unsigned>(batch * heads));
    attn_combine_kernel<D><<<cgrid, 256, 0, s>>>(part_o, part_ml, nz, NQ, heads, o, os);
    return cudaGetLastError();
}

}  // namespace

bool attention_mma_supported(int D) { return D == 32 || D == 64 || D == 128 || D == 256; }

cudaError_t attention_mma(int D, const float *q, AttnStrides qs, int NQ, const float *k, AttnStrides ks,
                          const float *v, AttnStrides vs, int NKV, int batch, int heads, const __half *mask,
                          int64_t mask_ld, float scale, float *o, AttnStrides os, cudaStream_t s) {
    if (NQ <= 0 || NKV <= 0 || batch <= 0 || heads <= 0 || static_cast<int64_t>(batch) * heads > 65535 ||
        (mask && mask_ld < NKV))
        return cudaErrorInvalidValue;
    switch (D) {
    case 32: return launch_mma<32, float>(q, qs, NQ, k, ks, v, vs, NKV, batch, heads, mask, mask_ld, scale, o, os, 1, nullptr, nullptr, s);
    case 64: return launch_mma<64, float>(q, qs, NQ, k, ks, v, vs, NKV, batch, heads, mask, mask_ld, scale, o, os, 1, nullptr, nullptr, s);
    case 128: return launch_mma<128, float>(q, qs, NQ, k, ks, v, vs, NKV, batch, heads, mask, mask_ld, scale, o, os, 1, nullptr, nullptr, s);
    case 256: return launch_mma<256, float>(q, qs, NQ, k, ks, v, vs, NKV, batch, heads, mask, mask_ld, scale, o, os, 1, nullptr, nullptr, s);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t attention_mma_f32mask(int D, const float *q, AttnStrides qs, int NQ, const float *k, AttnStrides ks,
                                  const float *v, AttnStrides vs, int NKV, int batch, int heads, const float *mask,
                                  int64_t mask_ld, int64_t mask_hs, float scale, float *o, AttnStrides os,
                                  cudaStream_t s) {
    if (NQ <= 0 || NKV <= 0 || batch <= 0 || heads <= 0 || static_cast<int64_t>(batch) * heads > 65535 ||
        (mask && (mask_ld < NKV || mask_hs < 0)))
        return cudaErrorInvalidValue;
    switch (D) {
    case 32: return launch_mma<32, float, float>(q, qs, NQ, k, ks, v, vs, NKV, batch, heads, mask, mask_ld, scale, o, os, 1, nullptr, nullptr, s, mask_hs);
    case 64: return launch_mma<64, float, float>(q, qs, NQ, k, ks, v, vs, NKV, batch, heads, mask, mask_ld, scale, o, os, 1, nullptr, nullptr, s, mask_hs);
    case 128: return launch_mma<128, float, float>(q, qs, NQ, k, ks, v, vs, NKV, batch, heads, mask, mask_ld, scale, o, os, 1, nullptr, nullptr, s, mask_hs);
    case 256: return launch_mma<256, float, float>(q, qs, NQ, k, ks, v, vs, NKV, batch, heads, mask, mask_ld, scale, o, os, 1, nullptr, nullptr, s, mask_hs);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t attention_combine(int D, const float *part_o, const float2 *part_ml, int splits, int NQ, int batch,
                              int heads, float *o, AttnStrides os, cudaStream_t s) {
    if (NQ <= 0 || splits < 1 || batch < 1 || heads < 1) return cudaErrorInvalidValue;
    const dim3 cgrid(static_cast<unsigned>((static_cast<int64_t>(NQ) * D + 255) / 256),
                     static_cast<unsigned>(batch * heads));
    switch (D) {
    case 16: attn_combine_kernel<16><<<cgrid, 256, 0, s>>>(part_o, part_ml, splits, NQ, heads, o, os); break;
    case 32: attn_combine_kernel<32><<<cgrid, 256, 0, s>>>(part_o, part_ml, splits, NQ, heads, o, os); break;
    case 64: attn_combine_kernel<64><<<cgrid, 256, 0, s>>>(part_o, part_ml, splits, NQ, heads, o, os); break;
    case 128: attn_combine_kernel<128><<<cgrid, 256, 0, s>>>(part_o, part_ml, splits, NQ, heads, o, os); break;
    case 256: attn_combine_kernel<256><<<cgrid, 256, 0, s>>>(part_o, part_ml, splits, NQ, heads, o, os); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t attention_mma_f16kv_split(int D, const float *q, AttnStrides qs, int NQ, const __half *k, AttnStrides ks,
                                      const __half *v, AttnStrides vs, int NKV, int batch, int heads, float scale,
                                      float *o, AttnStrides os, int splits, float *part_o, float2 *part_ml,
                                      cudaStream_t s) {
    if (NQ <= 0 || NKV <= 0 || batch <= 0 || heads <= 0 || static_cast<int64_t>(batch) * heads > 65535 ||
        splits < 1 || splits > 64 || (splits > 1 && (!part_o || !part_ml)))
        return cudaErrorInvalidValue;
    switch (D) {
    case 64: return launch_mma<64, __half, __half>(q, qs, NQ, k, ks, v, vs, NKV, batch, heads, nullptr, 0, scale, o, os, splits, part_o, part_ml, s);
    case 128: return launch_mma<128, __half, __half>(q, qs, NQ, k, ks, v, vs, NKV, batch, heads, nullptr, 0, scale, o, os, splits, part_o, part_ml, s);
    case 256: return launch_mma<256, __half, __half>(q, qs, NQ, k, ks, v, vs, NKV, batch, heads, nullptr, 0, scale, o, os, splits, part_o, part_ml, s);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace b200
