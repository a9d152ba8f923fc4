// attn_mma.cuh -- softmax(q k^T * scale + mask) v on the tensor cores
// (mma.sync, fp16 operands, fp32 accumulation) for head dims 32, 64, 128 and
// 256 with the strided operands and optional fp16 mask of attention_simt:
// the runners' attention where an fp16 rounding of q, k, v and of the
// probabilities is inside their tolerance (the tracker's memory attention,
// the detector's fusion / geometry encoders and segmentation head).
#pragma once

#include "attn_simt.cuh"

namespace b200 {

bool attention_mma_supported(int D);

// Same arguments and result layout as attention_simt (fp16 mask shared by the
// heads; a -inf entry removes the key; a row with every key removed yields zeros).
cudaError_t attention_mma(int D, const float *q, AttnStrides qs, int NQ, const float *k, AttnStrides ks,
                          const float *v, AttnStrides vs, int NKV, int batch, int heads, const __half *mask,
                          int64_t mask_ld, float scale, float *o, AttnStrides os, cudaStream_t s);

// The same with an f32 mask per head (head h of query row n reads
// mask[h * mask_hs + n * mask_ld + key]): the DETR decoder's box-relative bias.
cudaError_t attention_mma_f32mask(int D, const float *q, AttnStrides qs, int NQ, const float *k, AttnStrides ks,
                                  const float *v, AttnStrides vs, int NKV, int batch, int heads, const float *mask,
                                  int64_t mask_ld, int64_t mask_hs, float scale, float *o, AttnStrides os,
                                  cudaStream_t s);

// fp16 keys and values (already rounded: half the bytes to stage), no mask,
// keys split `splits` ways across CTAs (split-KV) so that few long query rows
// still fill the GPU: part_o (splits * batch * heads * NQ * D floats) and
// part_ml (splits * batch * heads * NQ float2) hold the partial results until
// a combine pass writes o.  Head dims 64, 128, 256.
cudaError_t attention_mma_f16kv_split(int D, const float *q, AttnStrides qs, int NQ, const __half *k, AttnStrides ks,
                                      const __half *v, AttnStrides vs, int NKV, int batch, int heads, float scale,
                                      float *o, AttnStrides os, int splits, float *part_o, float2 *part_ml,
                                      cudaStream_t s);

// The combine pass of a split-KV attention: o = sum_z 2^(m_z - M) part_o_z / sum_z 2^(m_z - M) l_z per
// row (part_ml = (m in log2 units, l) per split and row, part_o unnormalised).  D in {16, 32, 64, 128, 256}.
cudaError_t attention_combine(int D, const float *part_o, const float2 *part_ml, int splits, int NQ, int batch,
                              int heads, float *o, AttnStrides os, cudaStream_t s);

}  // namespace b200
