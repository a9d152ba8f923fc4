// sgemm.cu -- fp32 C = A B^T + bias on the CUDA cores for the convolutions
// that ggml computes in f32 (F32 kernels: ggml_conv_2d's im2col + an f32
// MUL_MAT): the memory encoder's 1x1 convolutions (sam3.cpp:11560-11600) and
// the Hiera patch embedding (sam3.cpp:4474).  128 x 64 output tiles, K staged
// through shared memory 16 at a time, 8 x 4 outputs per thread; A and B are
// read through element strides, so channel-major and token-major operands
// both load coalesced (the lanes run along whichever stride is 1).
#include "sgemm.cuh"

#include <cuda_fp16.h>

namespace b200 {
namespace {

constexpr int BM = 128, BN = 64, BK = 16;

__global__ void __launch_bounds__(256) sgemm_nt_kernel(const float *__restrict__ a, int64_t a_m, int64_t a_k,
                                                       const float *__restrict__ b, int64_t b_n, int64_t b_k, int M,
                                                       int N, int K, const float *__restrict__ bias,
                                                       float *__restrict__ c, int64_t ldc, int flags) {
    const bool a_f16 = flags & 1, b_f16 = flags & 2, bias_rows = flags & 4;
    __shared__ float as[BK][BM + 4];
    __shared__ float bs[BK][BN + 4];
    const int tid = threadIdx.x;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int tx = tid & 15, ty = tid >> 4;  // 16 x 16 threads: columns tx + 16 j, rows ty + 16 i
    float acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
    const bool a_kfast = a_k == 1;  // lanes along k (token-major rows) or along m (channel-major)
    const bool b_kfast = b_k == 1;
    for (int k0 = 0; k0 < K; k0 += BK) {
#pragma unroll
        for (int r = 0; r < BM * BK / 256; ++r) {
            const int e = tid + 256 * r;
            const int kk = a_kfast ? e % BK : e / BM, mm = a_kfast ? e / BK : e % BM;
            const int m = m0 + mm, k = k0 + kk;
            float v = 0.f;
            if (m < M && k < K) {
                v = a[static_cast<int64_t>(m) * a_m + static_cast<int64_t>(k) * a_k];
                if (a_f16) v = __half2float(__float2half_rn(v));
            }
            as[kk][mm] = v;
        }
#pragma unroll
        for (int r = 0; r < BN * BK / 256; ++r) {
            const int e = tid + 256 * r;
            const int kk = b_kfast ? e % BK : e / BN, nn = b_kfast ? e / BK : e % BN;
            const int n = n0 + nn, k = k0 + kk;
            float v = 0.f;
            if (n < N && k < K) {
                v = b[static_cast<int64_t>(n) * b_n + static_cast<int64_t>(k) * b_k];
                if (b_f16) v = __half2float(__float2half_rn(v));
            }
            bs[kk][nn] = v;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            float av[8], bv[4];
#pragma unroll
            for (int i = 0; i < 8; ++i) av[i] = as[kk][ty + 16 * i];
#pragma unroll
            for (int j = 0; j < 4; ++j) bv[j] = bs[kk][tx + 16 * j];
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int m = m0 + ty + 16 * i;
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = n0 + tx + 16 * j;
            if (n < N)
                c[static_cast<int64_t>(m) * ldc + n] = bias ? __fadd_rn(acc[i][j], bias[bias_rows ? m : n]) : acc[i][j];
        }
    }
}

// im2col of a channel-major image [C][H][W] for a KxK kernel, stride S, padding P:
// col[(oy * OW + ox) * C*K*K + (c * K + ky) * K + kx], zero outside the image
__global__ void im2col_chw_kernel(const float *__restrict__ x, int C, int H, int W, int K, int S, int P, int OH,
                                  int OW, float *__restrict__ col) {
    const int64_t KK = static_cast<int64_t>(C) * K * K;
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<int64_t>(OH) * OW * KK) return;
    const int64_t p = i / KK;
    const int r = static_cast<int>(i % KK);
    const int kx = r % K, ky = (r / K) % K, cc = r / (K * K);
    const int oy = static_cast<int>(p / OW), ox = static_cast<int>(p % OW);
    const int iy = oy * S - P + ky, ix = ox * S - P + kx;
    col[i] = (iy >= 0 && iy < H && ix >= 0 && ix < W) ? x[(static_cast<int64_t>(cc) * H + iy) * W + ix] : 0.f;
}

}  // namespace

cudaError_t sgemm_nt(const float *a, int64_t a_m, int64_t a_k, const float *b, int64_t b_n, int64_t b_k, int M, int N,
                     int K, const float *bias, float *c, int64_t ldc, bool a_f16, cudaStream_t s, bool b_f16,
                     bool bias_rows) {
    if (M <= 0 || N <= 0 || K <= 0 || !a || !b || !c || (M + BM - 1) / BM > 65535) return cudaErrorInvalidValue;
    const dim3 grid(static_cast<unsigned>((N + BN - 1) / BN), static_cast<unsigned>((M + BM - 1) / BM));
    sgemm_nt_kernel<<<grid, 256, 0, s>>>(a, a_m, a_k, b, b_n, b_k, M, N, K, bias, c, ldc,
                                         (a_f16 ? 1 : 0) | (b_f16 ? 2 : 0) | (bias_rows ? 4 : 0));
    return cudaGetLastError();
}

cudaError_t im2col_chw(const float *x, int C, int H, int W, int K, int S, int P, int OH, int OW, float *col,
                       cudaStream_t s) {
    const int64_t n = static_cast<int64_t>(OH) * OW * C * K * K;
    if (n <= 0) return cudaErrorInvalidValue;
    im2col_chw_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(x, C, H, W, K, S, P, OH, OW, col);
    return cudaGetLastError();
}

}  // namespace b200
