// attn_tcw.cuh -- attention over many small windows (and long single
// sequences) on the 5th-generation tensor cores, for the Hiera blocks
// (sam2_hiera_block_forward, sam3.cpp:4299-4461): per (window, head)
// out = softmax(q k^T * scale) v, head dimension up to 128, query count NQ
// (Q-pooled blocks: NQ = N / 4) and key count N per window.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace b200 {

// Operand widths: the head dimension padded to 64 or 128, the per-window key
// stride padded to a multiple of 8 (every key tile starts 16-byte aligned).
inline int attn_tcw_dpad(int hd) { return hd <= 64 ? 64 : 128; }
inline int attn_tcw_kstride(int N) { return (N + 7) / 8 * 8; }

// Elements of the three staged fp16 operands for (Bw windows, heads):
// q [heads][Bw * NQ][Dp], k [heads][Bw * Ns][Dp], v^T [heads][Dp][Bw * Ns].
inline size_t attn_tcw_q_elems(int Bw, int NQ, int heads, int hd) {
    return static_cast<size_t>(heads) * Bw * NQ * attn_tcw_dpad(hd);
}
inline size_t attn_tcw_kv_elems(int Bw, int N, int heads, int hd) {
    return static_cast<size_t>(heads) * Bw * attn_tcw_kstride(N) * attn_tcw_dpad(hd);
}

// Stage window-major f32 rows into the operands: q row (w * NQ + i) at q + row
// * q_ld + h * hd, k / v rows (w * N + j) at k / v + row * kv_ld + h * hd;
// fp16 round to nearest, zeros in the padding.
cudaError_t attn_tcw_stage(const float *q, int64_t q_ld, const float *k, const float *v, int64_t kv_ld, int Bw,
                           int NQ, int N, int heads, int hd, __half *qh, __half *kh, __half *vth, cudaStream_t s);

// o row (w * NQ + i), columns h * hd .. + hd (row stride o_ld) = the attention
// of window w, head h.  fp16 operands and probabilities, fp32 accumulation
// and row sums.  err: the device error word of the bounded waits.
cudaError_t attn_tcw(const __half *qh, const __half *kh, const __half *vth, int Bw, int NQ, int N, int heads, int hd,
                     float scale, float *o, int64_t o_ld, int *err, cudaStream_t s);

}  // namespace b200
