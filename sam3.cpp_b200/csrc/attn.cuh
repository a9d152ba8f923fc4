// attn.cuh -- attention of the ViT blocks (ggml_flash_attn_ext, sam3.cpp:3778).
#pragma once

#include <cuda_runtime.h>

namespace b200 {

// q, k, v: bf16 [B*heads][N][64]; out: f32 [B*N][heads*64].
cudaError_t flash_attention(const void *q, const void *k, const void *v, int B, int N, int heads, float scale,
                            float *out, cudaStream_t s);

}  // namespace b200
