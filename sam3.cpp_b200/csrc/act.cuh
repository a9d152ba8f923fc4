// act.cuh -- the activation functions of the ggml graphs, as ggml's CPU
// backend evaluates them (shared by the MUL_MAT epilogue and the elementwise
// kernels of the model runners).
#pragma once

#include <cuda_fp16.h>

namespace b200 {

// ggml_gelu_erf: 0.5 x (1 + erf(x / sqrt(2)))
__device__ __forceinline__ float gelu_erf_f(float x) {
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, erff(__fmul_rn(x, 0.70710678118654752440f))));
}

// ggml_gelu on the CPU backend (GGML_GELU_FP16, the Hiera MLP, sam3.cpp:4453):
// 0 at x <= -10, x at x >= 10, else the fp16 table entry of the tanh form at
// fp16(x): fp16(0.5 x (1 + tanh(sqrt(2/pi) x (1 + 0.044715 x^2)))).
__device__ __forceinline__ float gelu_tanh_f16(float x) {
    if (x <= -10.0f) return 0.0f;
    if (x >= 10.0f) return x;
    const float h = __half2float(__float2half_rn(x));
    const float inner = __fmul_rn(__fmul_rn(0.79788456080286535587989211986876f, h),
                                  __fadd_rn(1.0f, __fmul_rn(__fmul_rn(0.044715f, h), h)));
    return __half2float(__float2half_rn(__fmul_rn(__fmul_rn(0.5f, h), __fadd_rn(1.0f, tanhf(inner)))));
}

}  // namespace b200
