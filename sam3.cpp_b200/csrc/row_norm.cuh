// row_norm.cuh -- ggml_norm (+ ggml_mul by w, + ggml_add of b) over rows or
// channels of f32 maps, shared by the model runners.  ggml_norm forms the
// mean and the variance from double sums and rounds them to f32; the affine
// step is f32 ((x - mean) * scale * w + b, in that order).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace b200 {

__device__ __forceinline__ double rn_warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// rows of E contiguous floats (token-major maps): one warp per row
static __global__ void ln_rows_kernel(const float *__restrict__ x, int rows, int E, const float *__restrict__ w,
                                      const float *__restrict__ b, float eps, float *__restrict__ y) {
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (t >= rows) return;
    const float *xr = x + static_cast<int64_t>(t) * E;
    double s = 0.0;
    for (int c = lane; c < E; c += 32) s += static_cast<double>(xr[c]);
    s = rn_warp_sum_d(s);
    const float mean = static_cast<float>(s / E);
    double s2 = 0.0;
    for (int c = lane; c < E; c += 32) {
        const float d = __fsub_rn(xr[c], mean);
        s2 += static_cast<double>(__fmul_rn(d, d));
    }
    s2 = rn_warp_sum_d(s2);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(s2 / E), eps)));
    float *yr = y + static_cast<int64_t>(t) * E;
    for (int c = lane; c < E; c += 32)
        yr[c] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xr[c], mean), scale), w[c]), b[c]);
}

// channel-major maps x [C][P]: normalise over the C channels of every pixel
// (LayerNorm2d), one thread per pixel (coalesced across pixels)
static __global__ void ln_channels_kernel(const float *__restrict__ x, int C, int64_t P, const float *__restrict__ w,
                                          const float *__restrict__ b, float eps, float *__restrict__ y) {
    const int64_t p = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (p >= P) return;
    double s = 0.0;
    for (int c = 0; c < C; ++c) s += static_cast<double>(x[c * P + p]);
    const float mean = static_cast<float>(s / C);
    double s2 = 0.0;
    for (int c = 0; c < C; ++c) {
        const float d = __fsub_rn(x[c * P + p], mean);
        s2 += static_cast<double>(__fmul_rn(d, d));
    }
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(s2 / C), eps)));
    for (int c = 0; c < C; ++c)
        y[c * P + p] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x[c * P + p], mean), scale), w[c]), b[c]);
}

}  // namespace b200
