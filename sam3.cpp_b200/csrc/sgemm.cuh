// sgemm.cuh -- fp32 C = A B^T (+ bias) with strided operands (see sgemm.cu).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace b200 {

// C[m * ldc + n] = sum_k A(m, k) B(n, k) + bias[n] (bias[m] with bias_rows); A(m, k) = a[m * a_m + k * a_k],
// B(n, k) = b[n * b_n + k * b_k]; a_f16 / b_f16 round that operand's elements to fp16 first (the input of an
// F16 kernel in ggml).
cudaError_t sgemm_nt(const float *a, int64_t a_m, int64_t a_k, const float *b, int64_t b_n, int64_t b_k, int M, int N,
                     int K, const float *bias, float *c, int64_t ldc, bool a_f16, cudaStream_t s, bool b_f16 = false,
                     bool bias_rows = false);

// im2col of a channel-major image [C][H][W] for a KxK kernel (stride S, padding P), rows of C*K*K in
// (c, ky, kx) order for the OH x OW output pixels.
cudaError_t im2col_chw(const float *x, int C, int H, int W, int K, int S, int P, int OH, int OW, float *col,
                       cudaStream_t s);

}  // namespace b200
