// eltwise.cuh -- elementwise kernels the model runners share (ggml's add,
// relu, the additive attention-bias mask), each rounding as the ggml node it
// replaces: one f32 operation per node, no contraction.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace b200 {

inline unsigned ew_blocks(int64_t n) { return static_cast<unsigned>((n + 255) / 256); }

// c = a + b (c may alias a or b)
static __global__ void ew_add_kernel(const float *a, const float *b, int64_t n, float *c) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) c[i] = __fadd_rn(a[i], b[i]);
}

// x = max(x, 0)
static __global__ void ew_relu_kernel(float *x, int64_t n) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) x[i] = fmaxf(x[i], 0.0f);
}

// mask[q][t] = fp16(bias[t]) for q < nq: sam3_expand_token_attn_bias
// (sam3.cpp:7550-7570) -- a token-padding bias repeated over the queries and
// cast to the fp16 mask FLASH_ATTN_EXT reads (-1e9 becomes -inf)
static __global__ void ew_bias_mask_kernel(const float *__restrict__ bias, int64_t nq, int nt,
                                           __half *__restrict__ mask) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < nq * nt) mask[i] = __float2half_rn(bias[i % nt]);
}

// y = fp16(x)
static __global__ void ew_to_half_kernel(const float *__restrict__ x, int64_t n, __half *__restrict__ y) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) y[i] = __float2half_rn(x[i]);
}

}  // namespace b200
