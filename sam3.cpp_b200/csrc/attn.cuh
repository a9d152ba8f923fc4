// attn.cuh -- attention of the ViT blocks (ggml_flash_attn_ext, sam3.cpp:3778).
#pragma once

#include <cuda_runtime.h>

namespace b200 {

// q, k: bf16 [B*heads][N][64]; vt: bf16 [B*heads][64][N] (V transposed);
// out: f32 [B*N][heads*64].  N must be a multiple of 8 (TMA row pitch).
// Bounded waits report through *err (device word).
cudaError_t flash_attention(const void *q, const void *k, const void *vt, int B, int N, int heads, float scale,
                            float *out, int *err, cudaStream_t s);

}  // namespace b200
