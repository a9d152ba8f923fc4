// attn_simt.cu -- the general attention loop (see attn_simt.cuh).
//
// One CTA per (64 query rows, batch x head); 4 threads per query row, each
// owning D/4 dimensions of q and of the output accumulator; 64-key tiles of k
// and v staged in shared memory; online softmax in base 2 (scale and log2(e)
// folded into q, the mask scaled by log2(e)).
#include "attn_simt.cuh"
#include "attn_mma.cuh"

#include <cmath>

namespace b200 {
namespace {

// head dimension owned by register i of row-thread `part` (see attn_simt_kernel)
template <int DQ, bool VEC>
__device__ __forceinline__ int dim_of(int i, int part) {
    return VEC ? (i >> 2) * 16 + part * 4 + (i & 3) : part * DQ + i;
}

__device__ __forceinline__ float mask_value(__half m) { return __half2float(m); }
__device__ __forceinline__ float mask_value(float m) { return m; }

template <int DQ, typename MT>
__global__ void __launch_bounds__(256) attn_simt_kernel(const float *__restrict__ q, AttnStrides qs, int NQ,
                                                        const float *__restrict__ k, AttnStrides ks,
                                                        const float *__restrict__ v, AttnStrides vs, int NKV, int heads,
                                                        const MT *__restrict__ mask, int64_t mask_ld, int64_t mask_hs,
                                                        float scale_log2, float *__restrict__ o, AttnStrides os,
                                                        int chunk, float *__restrict__ part_o,
                                                        float2 *__restrict__ part_ml) {
    constexpr int HD = 4 * DQ, KT = 64;
    constexpr float LOG2E = 1.4426950408889634f;
    // Dimension ownership: with DQ % 4 == 0 the 4 threads of a row own
    // interleaved 4-float chunks (thread p: dims 16 j + 4 p + 0..3), so their
    // 16-byte shared-memory reads of one key row fall in distinct banks (a
    // contiguous DQ-float slice per thread would put all four in one bank
    // group: 4-way conflicts on every read); otherwise contiguous slices.
    constexpr bool VEC = DQ % 4 == 0;
    extern __shared__ float sm[];
    float *ksm = sm, *vsm = sm + KT * HD;
    const int b = blockIdx.y / heads, h = blockIdx.y % heads;
    const int row = blockIdx.x * (blockDim.x >> 2) + (threadIdx.x >> 2), part = threadIdx.x & 3;
    const bool valid = row < NQ;
    const float *kb = k + b * ks.b + h * ks.h;
    const float *vb = v + b * vs.b + h * vs.h;
    float qv[DQ], acc[DQ];
    const float *qr = q + b * qs.b + h * qs.h + static_cast<int64_t>(valid ? row : 0) * qs.n;
#pragma unroll
    for (int i = 0; i < DQ; ++i) {
        qv[i] = valid ? qr[dim_of<DQ, VEC>(i, part)] * scale_log2 : 0.f;
        acc[i] = 0.f;
    }
    const MT *mrow = mask ? mask + h * mask_hs + static_cast<int64_t>(valid ? row : 0) * mask_ld : nullptr;
    float m = -INFINITY, l = 0.f;
    // split over keys (part_o given): this CTA's keys [kv_lo, kv_hi), blockIdx.z = the split
    const int kv_lo = part_o ? blockIdx.z * chunk : 0;
    const int kv_hi = part_o ? min(NKV, kv_lo + chunk) : NKV;
    for (int j0 = kv_lo; j0 < kv_hi; j0 += KT) {
        __syncthreads();
        for (int e = threadIdx.x; e < KT * HD; e += blockDim.x) {
            const int kk = e / HD, d = e % HD, key = j0 + kk;
            float kv = 0.f, vv = 0.f;
            if (key < kv_hi) {
                kv = kb[static_cast<int64_t>(key) * ks.n + d];
                vv = vb[static_cast<int64_t>(key) * vs.n + d];
            }
            ksm[e] = kv;
            vsm[e] = vv;
        }
        __syncthreads();
        const int nk = kv_hi - j0 < KT ? kv_hi - j0 : KT;
        for (int kk = 0; kk < nk; ++kk) {
            float s = 0.f;
            if constexpr (VEC) {
                const float4 *kr = reinterpret_cast<const float4 *>(ksm + kk * HD) + part;
#pragma unroll
                for (int i = 0; i < DQ; i += 4) {
                    const float4 kv4 = kr[i];  // dims 16 (i / 4) + 4 part + 0..3
                    s = fmaf(qv[i], kv4.x, s);
                    s = fmaf(qv[i + 1], kv4.y, s);
                    s = fmaf(qv[i + 2], kv4.z, s);
                    s = fmaf(qv[i + 3], kv4.w, s);
                }
            } else {
                const float *kr = ksm + kk * HD + part * DQ;
#pragma unroll
                for (int i = 0; i < DQ; ++i) s = fmaf(qv[i], kr[i], s);
            }
            s += __shfl_xor_sync(0xffffffffu, s, 1);
            s += __shfl_xor_sync(0xffffffffu, s, 2);
            if (mrow) {
                const float mv = mask_value(mrow[j0 + kk]);
                if (mv == -INFINITY) continue;  // the 4 threads of a row agree
                s = fmaf(mv, LOG2E, s);
            }
            if (s > m) {
                const float alpha = exp2f(m - s);
                l *= alpha;
#pragma unroll
                for (int i = 0; i < DQ; ++i) acc[i] *= alpha;
                m = s;
            }
            const float p = exp2f(s - m);
            l += p;
            if constexpr (VEC) {
                const float4 *vr = reinterpret_cast<const float4 *>(vsm + kk * HD) + part;
#pragma unroll
                for (int i = 0; i < DQ; i += 4) {
                    const float4 vv4 = vr[i];
                    acc[i] = fmaf(p, vv4.x, acc[i]);
                    acc[i + 1] = fmaf(p, vv4.y, acc[i + 1]);
                    acc[i + 2] = fmaf(p, vv4.z, acc[i + 2]);
                    acc[i + 3] = fmaf(p, vv4.w, acc[i + 3]);
                }
            } else {
                const float *vr = vsm + kk * HD + part * DQ;
#pragma unroll
                for (int i = 0; i < DQ; ++i) acc[i] = fmaf(p, vr[i], acc[i]);
            }
        }
    }
    if (valid && part_o) {  // unnormalised partial result and (max in log2 units, sum) for the combine pass
        const int64_t r = (static_cast<int64_t>(blockIdx.z) * gridDim.y + blockIdx.y) * NQ + row;
#pragma unroll
        for (int i = 0; i < DQ; ++i) part_o[r * HD + dim_of<DQ, VEC>(i, part)] = acc[i];
        if (part == 0) part_ml[r] = make_float2(m, l);
    } else if (valid) {
        const float inv = l > 0.f ? 1.0f / l : 0.f;
        float *orow = o + b * os.b + h * os.h + static_cast<int64_t>(row) * os.n;
#pragma unroll
        for (int i = 0; i < DQ; ++i) orow[dim_of<DQ, VEC>(i, part)] = acc[i] * inv;
    }
}

template <int DQ, typename MT>
cudaError_t launch(const float *q, AttnStrides qs, int NQ, const float *k, AttnStrides ks, const float *v,
                   AttnStrides vs, int NKV, int batch, int heads, const MT *mask, int64_t mask_ld, int64_t mask_hs,
                   float scale, float *o, AttnStrides os, cudaStream_t s, int splits = 1, float *part_o = nullptr,
                   float2 *part_ml = nullptr) {
    const int smem = 2 * 64 * 4 * DQ * 4;
    cudaError_t e =
        cudaFuncSetAttribute(attn_simt_kernel<DQ, MT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    const int chunk = part_o ? (NKV + splits - 1) / splits : NKV;
    const int nz = part_o ? (NKV + chunk - 1) / chunk : 1;
    dim3 grid((NQ + 63) / 64, static_cast<unsigned>(batch * heads), static_cast<unsigned>(nz));
    attn_simt_kernel<DQ, MT><<<grid, 256, smem, s>>>(q, qs, NQ, k, ks, v, vs, NKV, heads, mask, mask_ld, mask_hs,
                                                     scale * 1.4426950408889634f, o, os, chunk, part_o, part_ml);
    e = cudaGetLastError();
    if (e != cudaSuccess || !part_o) return e;
    return attention_combine(4 * DQ, part_o, part_ml, nz, NQ, batch, heads, o, os, s);
}

template <typename MT>
cudaError_t dispatch(int D, const float *q, AttnStrides qs, int NQ, const float *k, AttnStrides ks, const float *v,
                     AttnStrides vs, int NKV, int batch, int heads, const MT *mask, int64_t mask_ld, int64_t mask_hs,
                     float scale, float *o, AttnStrides os, cudaStream_t s, int splits = 1, float *part_o = nullptr,
                     float2 *part_ml = nullptr) {
    if (NQ <= 0 || NKV <= 0 || batch <= 0 || heads <= 0 || static_cast<int64_t>(batch) * heads > 65535 ||
        (mask && (mask_ld < NKV || mask_hs < 0)))
        return cudaErrorInvalidValue;
#define B200_ATTN_CASE(d)                                                                                            \
    case 4 * d:                                                                                                      \
        return launch<d, MT>(q, qs, NQ, k, ks, v, vs, NKV, batch, heads, mask, mask_ld, mask_hs, scale, o, os, s, \
                             splits, part_o, part_ml)
    switch (D) {
        B200_ATTN_CASE(4);
        B200_ATTN_CASE(8);
        B200_ATTN_CASE(12);
        B200_ATTN_CASE(14);
        B200_ATTN_CASE(16);
        B200_ATTN_CASE(18);
        B200_ATTN_CASE(24);
        B200_ATTN_CASE(28);
        B200_ATTN_CASE(32);
        B200_ATTN_CASE(64);
    default: return cudaErrorInvalidValue;
    }
#undef B200_ATTN_CASE
}

}  // namespace

cudaError_t attention_simt(int D, const float *q, AttnStrides qs, int NQ, const float *k, AttnStrides ks,
                           const float *v, AttnStrides vs, int NKV, int batch, int heads, const __half *mask,
                           int64_t mask_ld, float scale, float *o, AttnStrides os, cudaStream_t s) {
    return dispatch<__half>(D, q, qs, NQ, k, ks, v, vs, NKV, batch, heads, mask, mask_ld, 0, scale, o, os, s);
}

cudaError_t attention_simt_split(int D, const float *q, AttnStrides qs, int NQ, const float *k, AttnStrides ks,
                                 const float *v, AttnStrides vs, int NKV, int batch, int heads, float scale, float *o,
                                 AttnStrides os, int splits, float *part_o, float2 *part_ml, cudaStream_t s) {
    if (splits < 1 || (splits > 1 && (!part_o || !part_ml)) || (D != 16 && D != 32 && D != 64)) return cudaErrorInvalidValue;
    if (splits == 1) return attention_simt(D, q, qs, NQ, k, ks, v, vs, NKV, batch, heads, nullptr, 0, scale, o, os, s);
    return dispatch<__half>(D, q, qs, NQ, k, ks, v, vs, NKV, batch, heads, nullptr, 0, 0, scale, o, os, s, splits, part_o,
                            part_ml);
}

cudaError_t attention_simt_f32mask(int D, const float *q, AttnStrides qs, int NQ, const float *k, AttnStrides ks,
                                   const float *v, AttnStrides vs, int NKV, int batch, int heads, const float *mask,
                                   int64_t mask_ld, int64_t mask_hs, float scale, float *o, AttnStrides os,
                                   cudaStream_t s) {
    return dispatch<float>(D, q, qs, NQ, k, ks, v, vs, NKV, batch, heads, mask, mask_ld, mask_hs, scale, o, os, s);
}

}  // namespace b200
