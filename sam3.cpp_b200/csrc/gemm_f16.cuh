// gemm_f16.cuh -- fp16 x fp16 -> fp32 tensor-core GEMM (tcgen05, TMA) used
// for the encoder's non-quantised contractions: the patch embedding
// (ggml_conv_2d_sk_p0, sam3.cpp:3819), and the SimpleFPN neck's transposed
// convolutions, 1x1 and 3x3 convolutions (sam3.cpp:3884-3922).
//
// C[m][n] = sum_k A[m][k] * B[n][k]; A fp16 [M, K] row-major, B fp16 [N, K]
// row-major, K a multiple of 8 (16-byte rows).  The epilogue adds bias[n],
// optionally applies GELU (erf form) and stores either fp32 or fp16, to a
// row-major [M, ldo] matrix or scattered as a 2x2 stride-2 transposed
// convolution output.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace b200 {

enum GemmStore : int {
    GEMM_STORE_ROWMAJOR = 0,  // out[m * ldo + n]
    GEMM_STORE_CONVT2X2 = 1,  // m = input pixel (iy, ix) of a win-wide map, n = (ky*2+kx)*cout + co
                              // -> out[((2iy+ky) * 2win + 2ix+kx) * cout + co]
};

struct GemmF16Args {
    const void *a;      // fp16 [M, K]
    const void *b;      // fp16 [N, K]
    int M, N, K;
    const float *bias;  // [N] or null (CONVT2X2: [cout], indexed by co)
    int gelu;           // apply GELU(erf) after the bias
    int out_f16;        // store fp16 instead of fp32
    void *out;
    int64_t ldo;
    int store;          // GemmStore
    int win, cout;      // CONVT2X2 geometry
    int *err;
};

cudaError_t gemm_f16(const GemmF16Args &args, int num_sms, cudaStream_t s);

}  // namespace b200
