// mmq.cuh -- device-side layouts and launch entry points of the quantised
// matrix multiply (ggml GGML_OP_MUL_MAT with Q8_0 / Q4_0 weights against
// activations quantised on the fly to Q8_0, sam3.cpp:3742,3783,3796,3799).
//
// Device layouts ("repacked" operands):
//   codes  : fp16 [rows, K] row-major, each value an exact small integer
//            (the block's int8 / nibble-8 code).  fp16 holds every int8
//            exactly, and a 32-term dot of such values accumulated by the
//            tensor core in fp32 is exact (|sum| <= 32*127*127 < 2^24), so
//            the MMA produces ggml's int32 block dot bit for bit.
//   scales : fp32 [K/32, ld] block-major: scales[b*ld + row] = fp16->fp32
//            of the block's d.  ld is rows rounded up to a multiple of 4 so
//            a TMA row is 16-byte aligned.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace b200 {

enum MmqOut : int {
    MMQ_OUT_F32 = 0,       // y[m*ldy + n] = acc (+ bias[n])
    MMQ_OUT_BLOCKDOTS = 1, // dump[(m*N + n)*nblk + b] = int32 block dot (debug/parity)
};

struct QMatrix {
    const void *codes;   // fp16 [rows, K]
    const float *scales; // fp32 [K/32, ld]
    int rows, K, ld;
};

struct MmqArgs {
    QMatrix a;           // activations, rows = M
    QMatrix b;           // weights, rows = N
    const float *bias;   // [N] or null
    float *y;            // [M, ldy]
    int64_t ldy;
    int32_t *dump;       // MMQ_OUT_BLOCKDOTS only
    int *err;            // device error word (0 = ok)
};

// Quantise f32 rows (ggml-cpu x86 activation rule) into the device layout.
cudaError_t quantize_rows_q8(const float *x, int64_t ldx, int M, int K, void *codes, float *scales, int ld,
                             cudaStream_t s);

// Repack ggml weight blocks (N rows of K) into the device layout.
// type: 8 = Q8_0, 2 = Q4_0.  Returns cudaErrorInvalidValue otherwise.
cudaError_t repack_weight_blocks(int type, const void *blocks, int N, int K, void *codes, float *scales, int ld,
                                 cudaStream_t s);

// tcgen05 tensor-core MMQ.
cudaError_t mmq_tc(const MmqArgs &args, int mode, int bn, int num_sms, cudaStream_t s);

// Straight SIMT version of the same arithmetic (small M, cross-checks).
cudaError_t mmq_simt(const MmqArgs &args, int mode, cudaStream_t s);

}  // namespace b200
