// mmq.cuh -- device-side layouts and launch entry points of the quantised
// matrix multiply (ggml GGML_OP_MUL_MAT with Q8_0 / Q4_0 weights against
// activations quantised on the fly to Q8_0, sam3.cpp:3742,3783,3796,3799).
//
// Device layouts of a quantised operand ("QMatrix", rows x K):
//   codes : int8 [rows, K] row-major -- the block's int8 code (Q8_0), or
//           nibble - 8 (Q4_0).  A kind::i8 MMA of K = 32 over two such rows
//           is exactly ggml's int32 block dot.
//   quads : 16-byte scale records, the K-major no-swizzle core-matrix rows of
//           a K=16 MMA operand, from which one K=16 kind::f16 MMA forms the
//           exact outer product S_b = d_x[:, b] (x) d_w[:, b]:
//             activations (A side) -- fp16 [ceil(K/256)][ld][8], record
//               (g, m) holds the scales of blocks 8g .. 8g+7 of row m;
//             weights (B side)     -- fp16 [K/32][ld][8], record (b, n)
//               holds d_w[n][b] in slot b % 8 and zeros elsewhere,
//           so A-record . B-record = d_x[m][b] * d_w[n][b] exactly.
//           ld = rows rounded up to a multiple of 128; padding rows are 0.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace b200 {

enum MmqOut : int {
    MMQ_OUT_F32 = 0,       // y[r*ldy + n] (+)= acc + bias[n], r = rowmap ? rowmap[m] : m
    MMQ_OUT_BLOCKDOTS = 1, // dump[(m*N + n)*nblk + b] = int32 block dot (debug/parity)
    MMQ_OUT_Q8 = 2,        // v = acc + bias (GELU-erf if gelu), re-quantised to Q8_0 (ggml-cpu
                           // activation rule) into the QMatrix (out_codes, out_quads, out_ld)
    MMQ_OUT_QKV = 3,       // attention inputs of a ViT block (sam3.cpp:3742-3776): v = acc + bias over
                           // N = 3E columns (q | k | v thirds, 64-wide heads), RoPE on the q and k
                           // thirds (sam3.cpp:3671-3710), written as bf16 Q, K [win*heads][tokens][64]
                           // and V^T [win*heads][64][tokens]; row m = window * win_tokens + token
    MMQ_OUT_DQ16 = 4,      // v = acc + bias (GELU if gelu), quantised to Q8_0 exactly as MMQ_OUT_Q8 and
                           // written dequantised, fp16(q * fp16(d)), into out16 [M, N] (the A operand of
                           // the next mmq_dq16)
};

constexpr int MMQ_ROW_ALIGN = 128;

// Bytes of an activation operand's scale records: ceil(K/256) groups of ld 16-byte records.
__host__ __device__ constexpr size_t act_quad_bytes(int K, int ld) {
    return static_cast<size_t>((K + 255) / 256) * static_cast<size_t>(ld) * 16u;
}

// element offset (in fp16 units) of block b's scale of row m in an A-side
// (activation) quad array with `ld` rows per group
__host__ __device__ constexpr int64_t act_quad_index(int b, int m, int ld) {
    return (static_cast<int64_t>(b >> 3) * ld + m) * 8 + (b & 7);
}

#ifdef __CUDACC__
// The Q8_0 code of v = x * id (|v| <= 127) as a float: round half to even,
// like (float)__float2int_rn(v), but on the FMA pipe -- adding 1.5 * 2^23
// leaves no fraction bits and the IEEE add rounds to nearest even -- instead
// of a float -> int -> float conversion pair.  Bit-identical for |v| < 2^22.
__device__ __forceinline__ float q8_code_f(float v) {
    return __fsub_rn(__fadd_rn(v, 12582912.0f), 12582912.0f);
}

// Store the scale d of block b (of nblk) of row m into an A-side record
// array.  The writer of a row's last block also zeroes the record slots past
// it when nblk is not a multiple of 8: the scale MMA reads whole records and
// multiplies those slots by the weight record's zeros, so left unwritten
// (holding whatever a previous use of the buffer left, possibly a NaN or an
// infinity) they would turn the product into a NaN.
__device__ __forceinline__ void store_act_scale(__half *quads, int b, int m, int ld, int nblk, float d) {
    const int64_t base = (static_cast<int64_t>(b >> 3) * ld + m) * 8;
    quads[base + (b & 7)] = __float2half_rn(d);
    if (b == nblk - 1)
        for (int s = (b & 7) + 1; s < 8; ++s) quads[base + s] = __ushort_as_half(static_cast<unsigned short>(0));
}
#endif

struct QMatrix {
    const void *codes;  // int8 [rows, K], or (nib != 0) 4-bit codes [rows, K/2]
    const void *quads;  // A side: fp16 [ceil(K/256)][ld][8]; B side: fp16 [K/32][ld][8]
    int rows, K, ld;
    // 0: one int8 code per element.  1 (Q4_0) / 2 (Q4_1): the blocks' own nibble
    // bytes, 16 per 32-element block, byte j = element j (low nibble) and element
    // j + 16 (high nibble); the code is nibble - 8 (Q4_0) or the nibble (Q4_1).
    int nib = 0;
};

struct MmqArgs {
    QMatrix a;          // activations, rows = M
    QMatrix b;          // weights, rows = N
    const float *bias;  // [N] or null
    float *y;           // [M, ldy]
    int64_t ldy;
    int32_t *dump;      // MMQ_OUT_BLOCKDOTS only
    int *err;           // device error word (0 = ok)
    int add = 0;                    // MMQ_OUT_F32: y = y + (acc + bias)
    const int *rowmap = nullptr;    // MMQ_OUT_F32: output row of tile row m
    int gelu = 0;                   // MMQ_OUT_Q8: 0 none, 1 GELU-erf, 2 ggml_gelu (tanh form, fp16 table)
    void *out_codes = nullptr;      // MMQ_OUT_Q8: int8 [M, N]
    void *out_quads = nullptr;      // MMQ_OUT_Q8: A-side records [ceil(N/256)][out_ld][16 B]
    int out_ld = 0;
    void *q_out = nullptr;          // MMQ_OUT_QKV: bf16 outputs
    void *k_out = nullptr;
    void *vt_out = nullptr;
    const float *freqs = nullptr;   // MMQ_OUT_QKV: RoPE table [win_tokens][32][2] (cos, sin), or null
    int win_tokens = 0;             // MMQ_OUT_QKV: tokens per window
    int heads = 0;                  // MMQ_OUT_QKV: heads (N = 3 * 64 * heads)
    const void *b_mins = nullptr;   // Q4_1 weights: m_w records, fp16 [K/32][ld][8] (m_w in slot b % 8)
    const void *a_sums = nullptr;   // Q4_1 weights: Q8_1 sum fields of the activations (act_quad_index layout)
    void *out16 = nullptr;          // MMQ_OUT_DQ16: fp16 [M, N]
};

// Quantise f32 rows (ggml-cpu x86 activation rule) into the device layout.
// quads must hold ceil(K/256) * ld records; rows >= M are left untouched.
// sums (optional): the Q8_1 sum fields s = fp16(d * sum(q)) in the quads'
// element layout (act_quad_index), for Q4_1 weights.
cudaError_t quantize_rows_q8(const float *x, int64_t ldx, int M, int K, void *codes, void *quads, int ld,
                             cudaStream_t s, void *sums = nullptr);

// Repack ggml weight blocks (N rows of K) into the device layout.
// type: 8 = Q8_0, 2 = Q4_0, 3 = Q4_1 (codes = nibbles 0..15, block minima to
// `mins` as records fp16 [K/32][ld][8], m_w in slot b % 8 like the scale
// records).  Returns cudaErrorInvalidValue otherwise.
// Codes: int8 [N][K] for Q8_0; the nibble bytes [N][K/2] for Q4_0 / Q4_1
// (weight_code_bytes).
inline size_t weight_code_bytes(int type, int N, int K) {
    return static_cast<size_t>(N) * static_cast<size_t>(type == 8 ? K : K / 2);
}
inline int weight_nib(int type) { return type == 2 ? 1 : type == 3 ? 2 : 0; }
cudaError_t repack_weight_blocks(int type, const void *blocks, int N, int K, void *codes, void *quads, int ld,
                                 cudaStream_t s, void *mins = nullptr);

// tcgen05 tensor-core MMQ, tile 128 x bn (bn = 64 or 128).  cvt selects the
// epilogue's exact int32 -> fp32 conversion: 0 = cvt instruction, 1 =
// magic-number add.
// bn = 0 picks the tile width from K.
cudaError_t mmq_tc(const MmqArgs &args, int mode, int num_sms, cudaStream_t s, int cvt = 0, int bn = 0);

// Straight SIMT version of the same arithmetic (small M, cross-checks).
cudaError_t mmq_simt(const MmqArgs &args, int mode, cudaStream_t s);

// ---- DQ16 arithmetic ------------------------------------------------------
// The same Q8_0 activation codes and scales (ggml's quantiser) and the same
// weight blocks, each element dequantised to fp16 -- fp16(q * d), one
// rounding of an exact product, relative error <= 2^-11 -- and multiplied on
// the fp16 tensor cores with fp32 accumulation over the whole of K.  The sum
// differs from the exact block-ordered fold by rounding only (about 3e-4
// normwise), and one MMA pass over K replaces the per-block int32 -> fp32
// fold on the CUDA cores.

// Dequantise an activation QMatrix (codes + A-side records, `ld` rows per
// record group) into fp16 [M][K].
cudaError_t dequant_act_f16(const void *codes, const void *quads, int M, int K, int ld, void *out, cudaStream_t s);
// Dequantise a Q8_0 (nib 0) or Q4_0 (nib 1) weight QMatrix into fp16 [N][K].
cudaError_t dequant_weight_f16(const QMatrix &w, void *out, cudaStream_t s);
// y = a16 . b16^T with the epilogues of mmq_tc (MMQ_OUT_F32, MMQ_OUT_QKV,
// MMQ_OUT_Q8, MMQ_OUT_DQ16): a16 fp16 [M][K], b16 fp16 [N][K], M = args.a.rows,
// N = args.b.rows, K = args.a.K (a multiple of 64).  bn: 128 or 256 (tile
// width), 0 = chosen from the tile count.
cudaError_t mmq_dq16(const MmqArgs &args, const void *a16, const void *b16, int mode, int num_sms, cudaStream_t s,
                     int bn = 0);

}  // namespace b200
