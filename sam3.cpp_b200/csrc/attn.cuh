// attn.cuh -- attention of the ViT blocks (ggml_flash_attn_ext, sam3.cpp:3778).
#pragma once

#include <cuda_runtime.h>

namespace b200 {

// Output of the attention, [B*N][heads*64] in row order: f32 rows, or (codes
// set) Q8_0 codes int8 [B*N][heads*64] + activation scale records
// [ceil(heads*64/256)][ld][8] fp16, the quantised layout the MUL_MAT reads.
struct AttnOut {
    float *f32 = nullptr;
    void *codes = nullptr;
    void *quads = nullptr;
    int ld = 0;
    // or (dq16 set) the same Q8_0 quantisation written dequantised,
    // fp16(q * fp16(d)) [B*N][heads*64] -- the A operand of mmq_dq16
    void *dq16 = nullptr;
};

// q, k: bf16 [B*heads][N][64]; vt: bf16 [B*heads][64][N] (V transposed).
// N must be a multiple of 8 (TMA row pitch).  Bounded waits report through
// *err (device word).
cudaError_t flash_attention(const void *q, const void *k, const void *vt, int B, int N, int heads, float scale,
                            const AttnOut &out, int *err, cudaStream_t s);

}  // namespace b200
