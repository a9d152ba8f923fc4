// attn_simt.cu -- the general attention loop (see attn_simt.cuh).
//
// One CTA per (64 query rows, batch x head); 4 threads per query row, each
// owning D/4 dimensions of q and of the output accumulator; 64-key tiles of k
// and v staged in shared memory; online softmax in base 2 (scale and log2(e)
// folded into q, the mask scaled by log2(e)).
#include "attn_simt.cuh"

#include <cmath>

namespace b200 {
namespace {

template <int DQ>
__global__ void __launch_bounds__(256) attn_simt_kernel(const float *__restrict__ q, AttnStrides qs, int NQ,
                                                        const float *__restrict__ k, AttnStrides ks,
                                                        const float *__restrict__ v, AttnStrides vs, int NKV, int heads,
                                                        const __half *__restrict__ mask, int64_t mask_ld,
                                                        float scale_log2, float *__restrict__ o, AttnStrides os) {
    constexpr int HD = 4 * DQ, KT = 64;
    constexpr float LOG2E = 1.4426950408889634f;
    extern __shared__ float sm[];
    float *ksm = sm, *vsm = sm + KT * HD;
    const int b = blockIdx.y / heads, h = blockIdx.y % heads;
    const int row = blockIdx.x * 64 + (threadIdx.x >> 2), part = threadIdx.x & 3;
    const bool valid = row < NQ;
    const float *kb = k + b * ks.b + h * ks.h;
    const float *vb = v + b * vs.b + h * vs.h;
    float qv[DQ], acc[DQ];
    const float *qr = q + b * qs.b + h * qs.h + static_cast<int64_t>(valid ? row : 0) * qs.n + part * DQ;
#pragma unroll
    for (int i = 0; i < DQ; ++i) {
        qv[i] = valid ? qr[i] * scale_log2 : 0.f;
        acc[i] = 0.f;
    }
    const __half *mrow = mask ? mask + static_cast<int64_t>(valid ? row : 0) * mask_ld : nullptr;
    float m = -INFINITY, l = 0.f;
    for (int j0 = 0; j0 < NKV; j0 += KT) {
        __syncthreads();
        for (int e = threadIdx.x; e < KT * HD; e += blockDim.x) {
            const int kk = e / HD, d = e % HD, key = j0 + kk;
            float kv = 0.f, vv = 0.f;
            if (key < NKV) {
                kv = kb[static_cast<int64_t>(key) * ks.n + d];
                vv = vb[static_cast<int64_t>(key) * vs.n + d];
            }
            ksm[e] = kv;
            vsm[e] = vv;
        }
        __syncthreads();
        const int nk = NKV - j0 < KT ? NKV - j0 : KT;
        for (int kk = 0; kk < nk; ++kk) {
            const float *kr = ksm + kk * HD + part * DQ;
            float s = 0.f;
#pragma unroll
            for (int i = 0; i < DQ; ++i) s = fmaf(qv[i], kr[i], s);
            s += __shfl_xor_sync(0xffffffffu, s, 1);
            s += __shfl_xor_sync(0xffffffffu, s, 2);
            if (mrow) {
                const float mv = __half2float(mrow[j0 + kk]);
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
            const float *vr = vsm + kk * HD + part * DQ;
#pragma unroll
            for (int i = 0; i < DQ; ++i) acc[i] = fmaf(p, vr[i], acc[i]);
        }
    }
    if (valid) {
        const float inv = l > 0.f ? 1.0f / l : 0.f;
        float *orow = o + b * os.b + h * os.h + static_cast<int64_t>(row) * os.n + part * DQ;
#pragma unroll
        for (int i = 0; i < DQ; ++i) orow[i] = acc[i] * inv;
    }
}

template <int DQ>
cudaError_t launch(const float *q, AttnStrides qs, int NQ, const float *k, AttnStrides ks, const float *v,
                   AttnStrides vs, int NKV, int batch, int heads, const __half *mask, int64_t mask_ld, float scale,
                   float *o, AttnStrides os, cudaStream_t s) {
    const int smem = 2 * 64 * 4 * DQ * 4;
    cudaError_t e = cudaFuncSetAttribute(attn_simt_kernel<DQ>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    dim3 grid((NQ + 63) / 64, static_cast<unsigned>(batch * heads));
    attn_simt_kernel<DQ><<<grid, 256, smem, s>>>(q, qs, NQ, k, ks, v, vs, NKV, heads, mask, mask_ld,
                                                 scale * 1.4426950408889634f, o, os);
    return cudaGetLastError();
}

}  // namespace

cudaError_t attention_simt(int D, const float *q, AttnStrides qs, int NQ, const float *k, AttnStrides ks,
                           const float *v, AttnStrides vs, int NKV, int batch, int heads, const __half *mask,
                           int64_t mask_ld, float scale, float *o, AttnStrides os, cudaStream_t s) {
    if (NQ <= 0 || NKV <= 0 || batch <= 0 || heads <= 0 || static_cast<int64_t>(batch) * heads > 65535 ||
        (mask && mask_ld < NKV))
        return cudaErrorInvalidValue;
    switch (D) {
    case 16: return launch<4>(q, qs, NQ, k, ks, v, vs, NKV, batch, heads, mask, mask_ld, scale, o, os, s);
    case 32: return launch<8>(q, qs, NQ, k, ks, v, vs, NKV, batch, heads, mask, mask_ld, scale, o, os, s);
    case 48: return launch<12>(q, qs, NQ, k, ks, v, vs, NKV, batch, heads, mask, mask_ld, scale, o, os, s);
    case 56: return launch<14>(q, qs, NQ, k, ks, v, vs, NKV, batch, heads, mask, mask_ld, scale, o, os, s);
    case 64: return launch<16>(q, qs, NQ, k, ks, v, vs, NKV, batch, heads, mask, mask_ld, scale, o, os, s);
    case 72: return launch<18>(q, qs, NQ, k, ks, v, vs, NKV, batch, heads, mask, mask_ld, scale, o, os, s);
    case 96: return launch<24>(q, qs, NQ, k, ks, v, vs, NKV, batch, heads, mask, mask_ld, scale, o, os, s);
    case 112: return launch<28>(q, qs, NQ, k, ks, v, vs, NKV, batch, heads, mask, mask_ld, scale, o, os, s);
    case 128: return launch<32>(q, qs, NQ, k, ks, v, vs, NKV, batch, heads, mask, mask_ld, scale, o, os, s);
    case 256: return launch<64>(q, qs, NQ, k, ks, v, vs, NKV, batch, heads, mask, mask_ld, scale, o, os, s);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace b200
