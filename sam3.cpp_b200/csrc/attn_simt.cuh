// attn_simt.cuh -- softmax(q k^T * scale + mask) v on the CUDA cores in fp32
// for the attention shapes the tcgen05 kernel (attn.cu: head dim 64,
// self-attention, no mask) does not take: any head dimension in {16, 32, 48,
// 56, 64, 72, 96, 112, 128, 256}, query and key counts that differ, strided
// (permuted-view) operands and an optional fp16 additive mask, as
// GGML_OP_FLASH_ATTN_EXT allows (sam3.cpp:3778, 3934-3951, 4386).
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace b200 {

// Element strides of a [D, tokens, heads, batch] operand: token, head, batch.
// The D elements of one (token, head, batch) are contiguous.
struct AttnStrides {
    int64_t b, h, n;
};

// o(b, h, n, :) = softmax_k(scale * q(b, h, n, :) . k(b, h, k, :) + mask[n * mask_ld + k]) v(b, h, k, :)
// mask (fp16, may be null) is shared by every head and batch; a -inf entry
// removes the key; a query row with every key removed yields zeros.
cudaError_t attention_simt(int D, const float *q, AttnStrides qs, int NQ, const float *k, AttnStrides ks,
                           const float *v, AttnStrides vs, int NKV, int batch, int heads, const __half *mask,
                           int64_t mask_ld, float scale, float *o, AttnStrides os, cudaStream_t s);

// Few queries against many keys (a handful of prompt tokens over 4096 image
// tokens), no mask: the keys split into `splits` ranges, each CTA writes its
// unnormalised partial result and (max, sum) to part_o [splits][batch * heads]
// [NQ][D] / part_ml [splits][batch * heads][NQ], and attention_combine merges
// them into o.  D in {16, 32, 64}; splits == 1 is attention_simt.
cudaError_t attention_simt_split(int D, const float *q, AttnStrides qs, int NQ, const float *k, AttnStrides ks,
                                 const float *v, AttnStrides vs, int NKV, int batch, int heads, float scale, float *o,
                                 AttnStrides os, int splits, float *part_o, float2 *part_ml, cudaStream_t s);

// The same with an f32 mask per head: head h of query row n reads
// mask[h * mask_hs + n * mask_ld + k] (the SOFT_MAX_EXT mask the reference
// keeps in f32 for the detector's box-relative bias, sam3.cpp:8580-8590).
cudaError_t attention_simt_f32mask(int D, const float *q, AttnStrides qs, int NQ, const float *k, AttnStrides ks,
                                   const float *v, AttnStrides vs, int NKV, int batch, int heads, const float *mask,
                                   int64_t mask_ld, int64_t mask_hs, float scale, float *o, AttnStrides os,
                                   cudaStream_t s);

}  // namespace b200
