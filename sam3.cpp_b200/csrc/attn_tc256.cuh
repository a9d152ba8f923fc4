// attn_tc256.cuh -- single-head width-256 attention on tcgen05 (see attn_tc256.cu).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace b200 {

// Key ranges per 128-query tile that fill num_sms SMs (at least two 64-key tiles per range).
int attention_tc256_splits(int NQ, int NK, int num_sms);

// v [NK][256] (row stride ld_v floats) -> fp16 v^T [256][ldt], keys contiguous, zero past NK
// (ldt >= NK, a multiple of 8).
cudaError_t v_to_half_transposed(const float *v, int NK, int ld_v, __half *vt, int ldt, cudaStream_t s);

// o [NQ][256] = softmax(q k^T scale) v: q fp16 [NQ][256], k fp16 [NK][256], vt fp16 [256][ldt];
// part_o (splits * NQ * 256 floats) and part_ml (splits * NQ) hold the key-range partials until the
// combine pass.  err: device word of the bounded pipeline waits.
cudaError_t attention_tc256(const __half *q, int NQ, const __half *k, int NK, const __half *vt, int ldt, float scale,
                            int splits, float *part_o, float2 *part_ml, float *o, int *err, cudaStream_t s);

}  // namespace b200
