// mmq.cu -- quantised matrix multiply for sm_100a (ggml GGML_OP_MUL_MAT with
// Q8_0 / Q4_0 weights, activations quantised on the fly to Q8_0).
//
// Reference semantics (ggml generic vec_dot, reached from ggml_mul_mat at
// sam3.cpp:3742,3783,3796,3799):
//     y[m][n] = sum_b  (float) I_b[m][n] * (d_w[n][b] * d_x[m][b])
//     I_b     = sum_{k in block b} q_w[n][k] * q_x[m][k]   (int32)
// summed block by block in order in fp32.
//
// How the tensor core does it, per 32-wide K block b of a 128 x 128 tile:
//   * one kind::i8 MMA (K = 32) over the int8 codes puts I_b, the exact
//     int32 block dot, into tensor memory;
//   * one kind::f16 MMA (K = 16, only column 0 populated) puts the outer
//     product S_b[m][n] = d_x[m][b] * d_w[n][b] next to it -- exact, since
//     a product of two fp16 values fits an fp32 significand;
//   * the epilogue warps convert I_b to fp32 (exact: |I_b| < 2^22) and fold
//     acc = fma(I_b, S_b, acc) in block order.
// That is the oracle's fma sequence, so results are bit-identical to it.
#include "act.cuh"
#include "mmq.cuh"
#include "ptx.cuh"
#include "tmap.h"

#include <atomic>
#include <cstdlib>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace b200 {

// ---------------------------------------------------------------------------
// Activation quantiser.  Rule of ggml-cpu's x86 quantize_row_q8_0:
// d = amax/127 stored as fp16, id = 127/amax, q = round-half-even(x * id).
// All operations are IEEE round-to-nearest (the library is built without
// fast-math; the intrinsics make it explicit).  Four threads per 32-element
// block, eight consecutive floats each (two 16-byte loads).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t pack4_s8(int a, int b, int c, int d) {
    return (static_cast<uint32_t>(a) & 0xFFu) | ((static_cast<uint32_t>(b) & 0xFFu) << 8) |
           ((static_cast<uint32_t>(c) & 0xFFu) << 16) | ((static_cast<uint32_t>(d) & 0xFFu) << 24);
}

template <bool VEC>
__global__ void quantize_rows_q8_kernel(const float *__restrict__ x, int64_t ldx, int M, int K,
                                        int8_t *__restrict__ codes, __half *__restrict__ quads,
                                        __half *__restrict__ sums, int ld) {
    const int per_row = K >> 3;  // threads per row
    const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const bool active = t < static_cast<int64_t>(M) * per_row;
    const int m = active ? static_cast<int>(t / per_row) : 0;
    const int e = active ? static_cast<int>(t % per_row) * 8 : 0;
    float v[8];
    if (active) {
        const float *src = x + static_cast<int64_t>(m) * ldx + e;
        if constexpr (VEC) {
            const float4 a = *reinterpret_cast<const float4 *>(src);
            const float4 b = *reinterpret_cast<const float4 *>(src + 4);
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
            v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = src[i];
        }
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0.f;
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
    // the 4 threads of a block are consecutive lanes (K % 32 == 0)
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const float d = __fdiv_rn(amax, 127.f);
    const float id = amax != 0.f ? __fdiv_rn(127.f, amax) : 0.f;
    int q[8], qsum = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        q[i] = __float2int_rn(__fmul_rn(v[i], id));
        qsum += q[i];
    }
    // Q8_1 sum field: s = d * sum(q) in fp32 (d unrounded), stored as fp16
    qsum += __shfl_xor_sync(0xffffffffu, qsum, 1);
    qsum += __shfl_xor_sync(0xffffffffu, qsum, 2);
    if (!active) return;
    *reinterpret_cast<uint2 *>(codes + static_cast<int64_t>(m) * K + e) =
        make_uint2(pack4_s8(q[0], q[1], q[2], q[3]), pack4_s8(q[4], q[5], q[6], q[7]));
    if ((e & 31) == 0) {
        store_act_scale(quads, e >> 5, m, ld, K >> 5, d);
        if (sums) sums[act_quad_index(e >> 5, m, ld)] = __float2half_rn(__fmul_rn(d, static_cast<float>(qsum)));
    }
}

cudaError_t quantize_rows_q8(const float *x, int64_t ldx, int M, int K, void *codes, void *quads, int ld,
                             cudaStream_t s, void *sums) {
    if (K % 32 != 0 || M < 0 || ld < M) return cudaErrorInvalidValue;
    if (M == 0) return cudaSuccess;
    const int64_t threads_total = static_cast<int64_t>(M) * (K / 8);
    const int threads = 256;
    const unsigned blocks = static_cast<unsigned>((threads_total + threads - 1) / threads);
    const bool vec = (ldx % 4 == 0) && (reinterpret_cast<uintptr_t>(x) % 16 == 0);
    if (vec)
        quantize_rows_q8_kernel<true><<<blocks, threads, 0, s>>>(x, ldx, M, K, static_cast<int8_t *>(codes),
                                                                 static_cast<__half *>(quads),
                                                                 static_cast<__half *>(sums), ld);
    else
        quantize_rows_q8_kernel<false><<<blocks, threads, 0, s>>>(x, ldx, M, K, static_cast<int8_t *>(codes),
                                                                  static_cast<__half *>(quads),
                                                                  static_cast<__half *>(sums), ld);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Weight repack: ggml blocks -> codes (int8 for Q8_0, the blocks' own nibble
// bytes for Q4_0 / Q4_1) + scale quads.
// ---------------------------------------------------------------------------
__global__ void repack_weight_kernel(int type, const uint8_t *__restrict__ blocks, int N, int K,
                                     int8_t *__restrict__ codes, uint4 *__restrict__ quads, uint4 *__restrict__ mins,
                                     int ld) {
    const int nblk = K >> 5;
    const int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (w >= static_cast<int64_t>(N) * nblk) return;
    const int n = static_cast<int>(w / nblk);
    const int b = static_cast<int>(w % nblk);
    const uint8_t *blk;
    if (type == 8) {  // Q8_0 {fp16 d; int8 qs[32]}
        blk = blocks + w * 34;
        codes[static_cast<int64_t>(n) * K + b * 32 + lane] = static_cast<int8_t>(blk[2 + lane]);
    } else {
        // Q4_0 {fp16 d; uint8 qs[16]} (code = nibble - 8), Q4_1 {fp16 d; fp16 m; uint8 qs[16]}
        // (code = nibble, value = d * code + m): the 16 nibble bytes are kept as they are
        blk = blocks + w * (type == 2 ? 18 : 20);
        if (lane < 16)
            codes[static_cast<int64_t>(n) * (K / 2) + b * 16 + lane] = static_cast<int8_t>(blk[(type == 2 ? 2 : 4) + lane]);
    }
    if (lane == 0) {  // fp16 records (d, and m for Q4_1) in slot b % 8, the rest zero: the scale MMA's B operand
        const int slot = b & 7;
        const uint32_t dbits = static_cast<uint32_t>(blk[0] | (blk[1] << 8));
        uint32_t rec[4] = {0u, 0u, 0u, 0u};
        rec[slot >> 1] = (slot & 1) ? (dbits << 16) : dbits;
        quads[static_cast<int64_t>(b) * ld + n] = make_uint4(rec[0], rec[1], rec[2], rec[3]);
        if (type == 3) {
            const uint32_t mbits = static_cast<uint32_t>(blk[2] | (blk[3] << 8));
            uint32_t mr[4] = {0u, 0u, 0u, 0u};
            mr[slot >> 1] = (slot & 1) ? (mbits << 16) : mbits;
            mins[static_cast<int64_t>(b) * ld + n] = make_uint4(mr[0], mr[1], mr[2], mr[3]);
        }
    }
}

cudaError_t repack_weight_blocks(int type, const void *blocks, int N, int K, void *codes, void *quads, int ld,
                                 cudaStream_t s, void *mins) {
    if (K % 32 != 0 || N <= 0 || ld < N || (type != 8 && type != 2 && type != 3) || (type == 3 && !mins))
        return cudaErrorInvalidValue;
    const int64_t warps = static_cast<int64_t>(N) * (K / 32);
    const int threads = 256;
    const unsigned grid = static_cast<unsigned>((warps * 32 + threads - 1) / threads);
    repack_weight_kernel<<<grid, threads, 0, s>>>(type, static_cast<const uint8_t *>(blocks), N, K,
                                                  static_cast<int8_t *>(codes), static_cast<uint4 *>(quads),
                                                  static_cast<uint4 *>(mins), ld);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// tcgen05 MMQ kernel.  CTA tile: 96 tokens x BN features (BN = 64 or 128),
// persistent over tiles.
//
// The MMAs are M = 128 and the TMEM lane quarter of sub-partition q is
// readable only by that sub-partition's warps.  Sub-partition 1 runs the MMA
// issuer and the TMA producer (measured: epilogue warps sharing a
// sub-partition with the MMA issuer hand TMEM slots back 350-1100 cycles
// late, and every slot waits for them), so its lane quarter (MMA rows
// 32..63) carries zero rows and the tile's 96 tokens sit in MMA rows 0..31
// and 64..127.  The tensor core has the headroom for the idle quarter.
//
// Warp roles (8 warps):
//   warp 1     : TMEM allocator + MMA issuer (one elected lane).  Per K-block
//                into TMEM slot `buf` (2 BN columns): I_b -> [0, BN) (int32),
//                S_b -> [BN, 2 BN) (fp32); commit to tfull[buf].
//   warp 5     : TMA producer (one elected lane).  A stage holds four
//                K-blocks: the A codes (three 32-row boxes into MMA rows 0..31
//                and 64..127), the B codes (128 int8 per row = one 128-byte
//                swizzle atom), the A scale records of the stage's 8-block
//                group and the four blocks' B scale records (bulk copies).
//   warps w with w % 4 != 1 : epilogue (EPQ = 2 or 4 per lane quarter).  Warp
//                w reads TMEM lane quarter w % 4 (0, 2 or 3: tile rows 0..31,
//                32..63, 64..95) and column slice w / 4 (BN / EPQ columns of
//                one output row per thread).
// Shared memory: STAGES stages (MMA rows 32..63 of the A codes and A records
// zero), a 2 KB zero region (the unused second K-chunk of every scale
// operand), barriers.
// ---------------------------------------------------------------------------
template <int BN_, int EPQ_ = 2, int NIB_ = 0>
struct TcCfg {
    // NIB: B codes as stored.  0 = int8 (Q8_0); 1 = Q4_0 nibbles, 2 = Q4_1 nibbles (each
    // stage's nibble bytes land in the RAW region, BN rows x 64 bytes, and warps 9 and 13
    // unpack them into the stage's swizzled int8 B operand).  Q4_1 adds the term m_w s_x
    // per block: its records (A: Q8_1 sum fields, B: minima) ride in the stage like the
    // scale records and a third MMA puts the product next to I and S.
    static constexpr int NIB = NIB_;
    static constexpr int BM = 128;                  // MMA rows
    static constexpr int ROWS = 96;                 // tokens per tile
    static constexpr int BN = BN_;
    static constexpr int BLK = 4;                   // K-blocks per stage
    static constexpr int BK = 32 * BLK;             // int8 per stage row: 128 bytes = one swizzle atom
    static constexpr int A_BYTES = BM * BK;         // 16 KB
    static constexpr int B_BYTES = BN * BK;
    static constexpr int Q_BYTES = BM * 16;         // the stage's A scale operand (one record group): 2 KB
    static constexpr int QB_BYTES = BN * 16;        // one block's B scale operand
    static constexpr int Q_OFF = A_BYTES + B_BYTES;                    // A scale group, then BLK B scale records
    static constexpr int MIN_OFF = Q_OFF + Q_BYTES + BLK * QB_BYTES;   // Q4_1: A sum group, then BLK B minima
    static constexpr int STAGE_BYTES = MIN_OFF + (NIB == 2 ? Q_BYTES + BLK * QB_BYTES : 0);
    // BN = 64 runs two CTAs per SM (3 stages and 256 TMEM columns each): one CTA's tile
    // stores and handshakes overlap the other's MMAs
    static constexpr int CTAS = BN == 64 ? 2 : 1;
    static constexpr int STAGES = NIB == 2 ? 3 : BN == 128 ? 4 : 3;
    static constexpr int ZERO_OFF = STAGES * STAGE_BYTES;
    static constexpr int BAR_OFF = ZERO_OFF + Q_BYTES;
    static constexpr int EPQ = EPQ_;                // epilogue warps per used lane quarter (2 or 4)
    static constexpr int THREADS = 128 * EPQ;       // warps w % 4 == 1 beyond warps 1 and 5 stay idle
    static constexpr int EPI_WARPS = 3 * EPQ;
    static constexpr int COLS = BN / EPQ;           // output columns per epilogue thread
    static constexpr int CHUNK = 32;
    static_assert(COLS % CHUNK == 0, "whole 32-column TMEM loads (and whole Q8_0 blocks) per thread");
    static constexpr int TERMS = NIB == 2 ? 3 : 2;  // TMEM per K-block: I, S (, M = m_w s_x), BN columns each
    static constexpr int SLOT_COLS = TERMS * BN;
    static constexpr int TMEM_COLS = 512 / CTAS;
    static constexpr int SLOTS = TMEM_COLS / SLOT_COLS;  // K-blocks in flight between MMA and epilogue
    static constexpr int RAW_STAGE = BN * BK / 2;
    static constexpr int RAW_OFF = BAR_OFF + 256;
    static constexpr int SMEM_BYTES = RAW_OFF + (NIB ? STAGES * RAW_STAGE : 0) + 1024;
    static_assert(!NIB || (BN == 128 && EPQ == 4), "4-bit B codes are unpacked by the idle warps 9 and 13");
    static_assert(STAGE_BYTES % 1024 == 0, "stage alignment");
    static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

enum : int {
    ERR_WAIT_EMPTY = 1,
    ERR_WAIT_FULL_MMA = 2,
    ERR_WAIT_TEMPTY = 4,
    ERR_WAIT_TFULL = 16,
    ERR_WAIT_RAW = 32,
};

// No-swizzle K-major operand descriptor for the K=16 scale MMA: core
// matrices of 8 rows x 16 bytes, 8-row groups 128 bytes apart (SBO), the
// second K-chunk `lbo` bytes after the first (it points at the zero region).
__device__ __forceinline__ uint64_t noswz_kmajor_desc(uint32_t smem_addr, uint32_t lbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>(128u >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    return d;  // layout type 0 = no swizzle
}

// Exact int32 -> fp32 for |v| < 2^22: place v in the significand of
// 1.5 * 2^23 and subtract that constant (one integer add, one fp add).
constexpr uint32_t MAGIC_BITS = 0x4B400000u;
constexpr float MAGIC_F = 12582912.0f;

struct MmqEpi {
    const float *bias;
    float *y;
    int64_t ldy;
    int32_t *dump;
    int add;
    const int *rowmap;
    int gelu;
    int8_t *qcodes;
    __half *qquads;
    int qld;
    __nv_bfloat16 *q, *k, *vt;
    const float *freqs;
    int win_tokens, heads;
    __half *o16;  // MMQ_OUT_DQ16
};

__device__ __forceinline__ uint32_t pack4_i8(int a, int b, int c, int d) {
    return (static_cast<uint32_t>(a) & 0xFFu) | ((static_cast<uint32_t>(b) & 0xFFu) << 8) |
           ((static_cast<uint32_t>(c) & 0xFFu) << 16) | ((static_cast<uint32_t>(d) & 0xFFu) << 24);
}

// Tile output of one epilogue thread: the COLS accumulators of tile row m for
// output columns [nb, nb + COLS) -- bias, then the mode's epilogue (residual
// add through the row map / GELU + Q8_0 re-quantisation / RoPE + head split).
template <int MODE, int COLS>
__device__ __forceinline__ void tile_store(const MmqEpi &ep, float (&acc)[COLS], int m, int M, int N, int nb) {
    const float *__restrict__ bias = ep.bias;
    if constexpr (MODE == MMQ_OUT_F32) {
        if (m < M) {
            const int r = ep.rowmap ? ep.rowmap[m] : m;
            float *yr = ep.y + static_cast<int64_t>(r) * ep.ldy + nb;
            const bool vec = ((ep.ldy & 3) == 0) && ((reinterpret_cast<uintptr_t>(ep.y) & 15) == 0);
#pragma unroll
            for (int j = 0; j < COLS; j += 4) {
                float o[4] = {acc[j], acc[j + 1], acc[j + 2], acc[j + 3]};
                if (vec && nb + j + 3 < N) {
                    if (bias) {
                        const float4 bb = *reinterpret_cast<const float4 *>(bias + nb + j);
                        o[0] = __fadd_rn(o[0], bb.x);
                        o[1] = __fadd_rn(o[1], bb.y);
                        o[2] = __fadd_rn(o[2], bb.z);
                        o[3] = __fadd_rn(o[3], bb.w);
                    }
                    if (ep.add) {
                        const float4 prev = *reinterpret_cast<const float4 *>(yr + j);
                        o[0] = __fadd_rn(prev.x, o[0]);
                        o[1] = __fadd_rn(prev.y, o[1]);
                        o[2] = __fadd_rn(prev.z, o[2]);
                        o[3] = __fadd_rn(prev.w, o[3]);
                    }
                    *reinterpret_cast<float4 *>(yr + j) = make_float4(o[0], o[1], o[2], o[3]);
                } else {
                    for (int e = 0; e < 4; ++e) {
                        if (nb + j + e >= N) break;
                        float val = bias ? __fadd_rn(o[e], bias[nb + j + e]) : o[e];
                        if (ep.add) val = __fadd_rn(yr[j + e], val);
                        yr[j + e] = val;
                    }
                }
            }
        }
    } else if constexpr (MODE == MMQ_OUT_QKV) {
        // this thread's COLS columns lie inside one 64-wide head of the q, k or v third
        if (m < M) {
            const int E = N / 3;
            const int part = nb / E, c0 = nb - part * E, hd = c0 >> 6, d0 = c0 & 63;
            const int win = m / ep.win_tokens, pos = m - win * ep.win_tokens;
            const int64_t bh = static_cast<int64_t>(win) * ep.heads + hd;
#pragma unroll
            for (int i = 0; i < COLS; ++i)
                if (bias) acc[i] = __fadd_rn(acc[i], bias[nb + i]);
            if (part < 2) {
                if (ep.freqs) {
                    const float *fr = ep.freqs + (static_cast<int64_t>(pos) * 32 + (d0 >> 1)) * 2;
#pragma unroll
                    for (int i = 0; i < COLS; i += 2) {
                        const float2 cs = *reinterpret_cast<const float2 *>(fr + i);
                        const float x0 = acc[i], x1 = acc[i + 1];
                        acc[i] = __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y));
                        acc[i + 1] = __fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(x1, cs.x));
                    }
                }
                __nv_bfloat16 *dst = (part == 0 ? ep.q : ep.k) + (bh * ep.win_tokens + pos) * 64 + d0;
#pragma unroll
                for (int i = 0; i < COLS; i += 8) {
                    uint4 u;
                    uint32_t *uw = reinterpret_cast<uint32_t *>(&u);
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const __nv_bfloat162 p2 = __floats2bfloat162_rn(acc[i + 2 * e], acc[i + 2 * e + 1]);
                        uw[e] = *reinterpret_cast<const uint32_t *>(&p2);
                    }
                    *reinterpret_cast<uint4 *>(dst + i) = u;
                }
            } else {
                // V^T: consecutive lanes hold consecutive tokens, so each store is 64 contiguous bytes
                __nv_bfloat16 *dst = ep.vt + (bh * 64 + d0) * ep.win_tokens + pos;
#pragma unroll
                for (int i = 0; i < COLS; ++i) dst[static_cast<int64_t>(i) * ep.win_tokens] = __float2bfloat16_rn(acc[i]);
            }
        }
    } else if constexpr (MODE == MMQ_OUT_Q8 || MODE == MMQ_OUT_DQ16) {
        // this thread's COLS columns are whole 32-wide Q8_0 blocks of the output row
        if (m < M) {
#pragma unroll
            for (int hb = 0; hb < COLS; hb += 32) {
                if (nb + hb >= N) break;
                float amax = 0.f;
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    float val = bias ? __fadd_rn(acc[hb + i], bias[nb + hb + i]) : acc[hb + i];
                    if (ep.gelu == 1) val = gelu_erf_f(val);
                    else if (ep.gelu == 2) val = gelu_tanh_f16(val);
                    acc[hb + i] = val;
                    amax = fmaxf(amax, fabsf(val));
                }
                const float d = __fdiv_rn(amax, 127.f);
                const float id = amax != 0.f ? __fdiv_rn(127.f, amax) : 0.f;
                if constexpr (MODE == MMQ_OUT_DQ16) {
                    // the block's codes times its stored (fp16) scale, rounded once to fp16
                    const float dh = __half2float(__float2half_rn(d));
                    uint4 *dst = reinterpret_cast<uint4 *>(ep.o16 + static_cast<int64_t>(m) * N + nb + hb);
#pragma unroll
                    for (int i = 0; i < 32; i += 8) {
                        uint32_t hw[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float q0 = q8_code_f(__fmul_rn(acc[hb + i + 2 * e], id));
                            const float q1 = q8_code_f(__fmul_rn(acc[hb + i + 2 * e + 1], id));
                            const __half2 h2 = __floats2half2_rn(__fmul_rn(q0, dh), __fmul_rn(q1, dh));
                            hw[e] = *reinterpret_cast<const uint32_t *>(&h2);
                        }
                        dst[i >> 3] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                    }
                } else {
                    uint32_t pk[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        pk[i] = pack4_i8(__float2int_rn(__fmul_rn(acc[hb + 4 * i], id)),
                                         __float2int_rn(__fmul_rn(acc[hb + 4 * i + 1], id)),
                                         __float2int_rn(__fmul_rn(acc[hb + 4 * i + 2], id)),
                                         __float2int_rn(__fmul_rn(acc[hb + 4 * i + 3], id)));
                    uint4 *dst = reinterpret_cast<uint4 *>(ep.qcodes + static_cast<int64_t>(m) * N + nb + hb);
                    dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                    dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
                    store_act_scale(ep.qquads, (nb + hb) >> 5, m, ep.qld, N >> 5, d);
                }
            }
        }
    }
}

template <int MODE, int CVT, int BN, int EPQ, int NIB>
__global__ void __launch_bounds__(TcCfg<BN, EPQ>::THREADS, TcCfg<BN, EPQ>::CTAS)
    mmq_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                  const uint8_t *__restrict__ quads_a, const uint8_t *__restrict__ quads_b, int M, int N, int nblk,
                  int lda_q, int ldb_q, const MmqEpi ep, int *__restrict__ err, const uint8_t *__restrict__ sums_a,
                  const uint8_t *__restrict__ mins_b) {
    int32_t *__restrict__ dump = ep.dump;
    using C = TcCfg<BN, EPQ, NIB>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
    uint64_t *empty = full + C::STAGES;
    uint64_t *tfull = empty + C::STAGES;
    uint64_t *tempty = tfull + C::SLOTS;
    uint64_t *rfull = tempty + C::SLOTS;  // NIB: a stage's nibble bytes have landed
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(rfull + C::STAGES);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int num_m = (M + C::ROWS - 1) / C::ROWS;
    const int num_n = (N + C::BN - 1) / C::BN;
    const int num_tiles = num_m * num_n;
    const int kstages = (nblk + C::BLK - 1) / C::BLK;

    // zero region read by every scale MMA as its second K-chunk, and the
    // idle lane quarter's MMA rows 32..63 of every stage's A codes and records
    for (int i = threadIdx.x; i < C::Q_BYTES / 16; i += blockDim.x)
        reinterpret_cast<uint4 *>(smem + C::ZERO_OFF)[i] = make_uint4(0u, 0u, 0u, 0u);
    for (int i = threadIdx.x; i < C::STAGES * (32 * C::BK + 32 * 16) / 16; i += blockDim.x) {
        const int st = i / ((32 * C::BK + 32 * 16) / 16), j = i % ((32 * C::BK + 32 * 16) / 16);
        uint8_t *sb = smem + st * C::STAGE_BYTES;
        uint8_t *dst = j < 32 * C::BK / 16 ? sb + 32 * C::BK + j * 16
                                           : sb + C::A_BYTES + C::B_BYTES + 32 * 16 + (j - 32 * C::BK / 16) * 16;
        *reinterpret_cast<uint4 *>(dst) = make_uint4(0u, 0u, 0u, 0u);
    }
    if constexpr (NIB == 2)  // and of the Q4_1 sum-field records
        for (int i = threadIdx.x; i < C::STAGES * 32; i += blockDim.x)
            *reinterpret_cast<uint4 *>(smem + (i >> 5) * C::STAGE_BYTES + C::MIN_OFF + (32 + (i & 31)) * 16) =
                make_uint4(0u, 0u, 0u, 0u);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&full[s], NIB ? 3 : 1);  // NIB: + one arrival per unpacking warp
            mbar_init(&empty[s], 1);
            mbar_init(&rfull[s], 1);
        }
        for (int i = 0; i < C::SLOTS; ++i) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], C::EPI_WARPS * 32);  // every epilogue lane arrives
        }
        fence_mbar_init();
        prefetch_tmap(&tm_a);
        prefetch_tmap(&tm_b);

    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 5) {
        // ---- TMA producer: warp-uniform loop, one elected lane issues ----
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
            const int m0 = (t % num_m) * C::ROWS;
            const int n0 = (t / num_m) * C::BN;
            // A scale records of rows [m0, m0 + 96) that exist (lda_q >= M; rows past it are never stored)
            const int r1 = lda_q - m0 < 32 ? (lda_q - m0 > 0 ? lda_q - m0 : 0) : 32;
            const int r2 = lda_q - m0 - 32 < 64 ? (lda_q - m0 - 32 > 0 ? lda_q - m0 - 32 : 0) : 64;
            for (int ks = 0; ks < kstages; ++ks) {
                if (!__all_sync(0xffffffffu, mbar_wait(&empty[stage], phase ^ 1u, err, ERR_WAIT_EMPTY))) {
                    ok = false;
                    break;
                }
                uint8_t *sb = smem + stage * C::STAGE_BYTES;
                uint8_t *q = sb + C::A_BYTES + C::B_BYTES;
                if (elect_one()) {
                    // scale records are contiguous per (group or block, tile): one bulk copy each
                    const int b0 = ks * C::BLK;
                    const int nb = nblk - b0 < C::BLK ? nblk - b0 : C::BLK;
                    mbar_arrive_expect_tx(&full[stage], 3 * 32 * C::BK + (NIB ? 0 : C::B_BYTES) +
                                                            (NIB == 2 ? 2 : 1) * ((r1 + r2) * 16 + nb * C::QB_BYTES));
                    tma_load_2d(sb, &tm_a, &full[stage], ks * C::BK, m0);                         // MMA rows 0..31
                    tma_load_2d(sb + 64 * C::BK, &tm_a, &full[stage], ks * C::BK, m0 + 32);       // 64..95
                    tma_load_2d(sb + 96 * C::BK, &tm_a, &full[stage], ks * C::BK, m0 + 64);       // 96..127
                    if constexpr (NIB) {
                        mbar_arrive_expect_tx(&rfull[stage], C::RAW_STAGE);
                        tma_load_2d(smem + C::RAW_OFF + stage * C::RAW_STAGE, &tm_b, &rfull[stage], ks * (C::BK / 2), n0);
                    } else {
                        tma_load_2d(sb + C::A_BYTES, &tm_b, &full[stage], ks * C::BK, n0);
                    }
                    const uint8_t *qa = quads_a + (static_cast<int64_t>(b0 >> 3) * lda_q + m0) * 16;
                    if (r1 > 0) bulk_load(q, qa, r1 * 16, &full[stage]);
                    if (r2 > 0) bulk_load(q + 64 * 16, qa + 32 * 16, r2 * 16, &full[stage]);
                    for (int j = 0; j < nb; ++j)
                        bulk_load(q + C::Q_BYTES + j * C::QB_BYTES,
                                  quads_b + (static_cast<int64_t>(b0 + j) * ldb_q + n0) * 16, C::QB_BYTES, &full[stage]);
                    if constexpr (NIB == 2) {  // the same records for m_w s_x: A sum fields, B minima
                        uint8_t *mq = sb + C::MIN_OFF;
                        const uint8_t *sa = sums_a + (static_cast<int64_t>(b0 >> 3) * lda_q + m0) * 16;
                        if (r1 > 0) bulk_load(mq, sa, r1 * 16, &full[stage]);
                        if (r2 > 0) bulk_load(mq + 64 * 16, sa + 32 * 16, r2 * 16, &full[stage]);
                        for (int j = 0; j < nb; ++j)
                            bulk_load(mq + C::Q_BYTES + j * C::QB_BYTES,
                                      mins_b + (static_cast<int64_t>(b0 + j) * ldb_q + n0) * 16, C::QB_BYTES,
                                      &full[stage]);
                    }
                }
                __syncwarp();
                if (++stage == C::STAGES) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
        }
    } else if (warp == 1) {
        // ---- MMA issuer: warp-uniform loop, one elected lane issues ----
        constexpr uint32_t idesc_i = NIB == 2 ? idesc_s8u8_s32(C::BM, C::BN) : idesc_s8_s32(C::BM, C::BN);
        constexpr uint32_t idesc_s = idesc_f16_f32(C::BM, C::BN);
        const uint32_t zero_addr = smem_u32(smem + C::ZERO_OFF);
        int stage = 0;
        uint32_t phase = 0;
        uint32_t blk = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
            for (int ks = 0; ks < kstages; ++ks) {
                if (!__all_sync(0xffffffffu, mbar_wait(&full[stage], phase, err, ERR_WAIT_FULL_MMA))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t a_addr = smem_u32(smem + stage * C::STAGE_BYTES);
                const uint32_t b_addr = a_addr + C::A_BYTES;
                const uint32_t q_addr = b_addr + C::B_BYTES;
                const uint64_t qa_desc = noswz_kmajor_desc(q_addr, zero_addr - q_addr);
                for (int j = 0; j < C::BLK; ++j) {
                    if (ks * C::BLK + j >= nblk) break;
                    const uint32_t buf = blk % C::SLOTS;
                    if (!__all_sync(0xffffffffu,
                                    mbar_wait(&tempty[buf], ((blk / C::SLOTS) & 1u) ^ 1u, err, ERR_WAIT_TEMPTY))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + buf * C::SLOT_COLS;
                    const uint32_t koff = static_cast<uint32_t>(j * 32);  // 32 int8 = 32 bytes
                    const uint64_t a_desc = sw128_kmajor_desc(a_addr + koff);
                    const uint64_t b_desc = sw128_kmajor_desc(b_addr + koff);
                    const uint32_t qb = q_addr + C::Q_BYTES + j * C::QB_BYTES;
                    const uint64_t qb_desc = noswz_kmajor_desc(qb, zero_addr - qb);
                    if (elect_one()) {
                        mma_i8(d_tmem, a_desc, b_desc, idesc_i, 0);
                        if constexpr (MODE != MMQ_OUT_BLOCKDOTS) mma_f16(d_tmem + C::BN, qa_desc, qb_desc, idesc_s, 0);
                        if constexpr (NIB == 2 && MODE != MMQ_OUT_BLOCKDOTS) {
                            const uint32_t sa = smem_u32(smem + stage * C::STAGE_BYTES + C::MIN_OFF);
                            const uint32_t mb = sa + C::Q_BYTES + j * C::QB_BYTES;
                            mma_f16(d_tmem + 2 * C::BN, noswz_kmajor_desc(sa, zero_addr - sa),
                                    noswz_kmajor_desc(mb, zero_addr - mb), idesc_s, 0);
                        }
                        mma_commit(&tfull[buf]);
                    }
                    __syncwarp();
                    ++blk;
                }
                if (!ok) break;
                if (elect_one()) mma_commit(&empty[stage]);
                __syncwarp();
                if (++stage == C::STAGES) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
        }
    } else if (NIB != 0 && (warp == 9 || warp == 13)) {
        // ---- nibble unpack (Q4_0 weights): the stage's BN x 64 nibble bytes -> the
        // int8 B operand in the layout a 128-byte-swizzled TMA load would have
        // left (row r at r * 128, its 16-byte chunk c at chunk c ^ (r % 8)).  One
        // 16-byte source chunk is one block's nibbles: low nibbles are elements
        // 0..15 (chunk 2j of the row), high nibbles 16..31 (chunk 2j + 1); the
        // code nibble - 8 of each byte is (nibble + 0x78) ^ 0x80, no carries. ----
        const int ct = (warp == 9 ? 0 : 32) + lane;
        const uint32_t off = NIB == 1 ? 0x78787878u : 0u, flip = NIB == 1 ? 0x80808080u : 0u;  // Q4_1: the nibble
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
            for (int ks = 0; ks < kstages; ++ks) {
                if (!__all_sync(0xffffffffu, mbar_wait(&rfull[stage], phase, err, ERR_WAIT_RAW))) {
                    ok = false;
                    break;
                }
                const uint8_t *raw = smem + C::RAW_OFF + stage * C::RAW_STAGE;
                uint8_t *dst = smem + stage * C::STAGE_BYTES + C::A_BYTES;
#pragma unroll
                for (int i = 0; i < C::BN * 4 / 64; ++i) {
                    const int c = ct + 64 * i, r = c >> 2, j = c & 3;
                    const uint4 x = *reinterpret_cast<const uint4 *>(raw + r * 64 + j * 16);
                    uint4 lo, hi;
                    lo.x = ((x.x & 0x0F0F0F0Fu) + off) ^ flip;
                    lo.y = ((x.y & 0x0F0F0F0Fu) + off) ^ flip;
                    lo.z = ((x.z & 0x0F0F0F0Fu) + off) ^ flip;
                    lo.w = ((x.w & 0x0F0F0F0Fu) + off) ^ flip;
                    hi.x = (((x.x >> 4) & 0x0F0F0F0Fu) + off) ^ flip;
                    hi.y = (((x.y >> 4) & 0x0F0F0F0Fu) + off) ^ flip;
                    hi.z = (((x.z >> 4) & 0x0F0F0F0Fu) + off) ^ flip;
                    hi.w = (((x.w >> 4) & 0x0F0F0F0Fu) + off) ^ flip;
                    *reinterpret_cast<uint4 *>(dst + r * 128 + (((2 * j) ^ (r & 7)) << 4)) = lo;
                    *reinterpret_cast<uint4 *>(dst + r * 128 + (((2 * j + 1) ^ (r & 7)) << 4)) = hi;
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the MMA's reads
                __syncwarp();
                if (lane == 0) mbar_arrive(&full[stage]);
                if (++stage == C::STAGES) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
        }
    } else if ((warp & 3) != 1) {
        // ---- epilogue warps ----
        constexpr int CHUNK = C::CHUNK;
        const int q = warp & 3;                              // TMEM lane quarter: 0, 2 or 3
        const int h = warp >> 2;                             // column slice
        const int row = (q == 0 ? 0 : (q - 1) * 32) + lane;  // tile row (token m0 + row)
        const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
        uint32_t blk = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
            const int m0 = (t % num_m) * C::ROWS;
            const int n0 = (t / num_m) * C::BN;
            const int m = m0 + row;
            float acc[C::COLS];
#pragma unroll
            for (int i = 0; i < C::COLS; ++i) acc[i] = 0.f;
            for (int b = 0; b < nblk; ++b) {
                const uint32_t buf = blk % C::SLOTS;
                if (!__all_sync(0xffffffffu, mbar_wait(&tfull[buf], (blk / C::SLOTS) & 1u, err, ERR_WAIT_TFULL))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t ta = tmem_base + lane_addr + buf * C::SLOT_COLS + h * C::COLS;
#pragma unroll
                for (int c0 = 0; c0 < C::COLS; c0 += CHUNK) {
                    uint32_t vi[CHUNK], vs[CHUNK];
                    tmem_ld_32x32b_x32(ta + c0, vi);
                    if constexpr (MODE != MMQ_OUT_BLOCKDOTS) tmem_ld_32x32b_x32(ta + C::BN + c0, vs);
                    tmem_wait_ld();
                    constexpr bool MINS = NIB == 2 && MODE != MMQ_OUT_BLOCKDOTS;  // Q4_1: + m_w s_x after the fma
                    if (!MINS && c0 + CHUNK == C::COLS) {
                        // the whole buffer is in registers: hand it back to the MMA warp
                        // (all 32 lanes arrive: no divergent branch on the per-block path, 2% faster)
                        tc_fence_before();
                        mbar_arrive(&tempty[buf]);
                    }
                    if constexpr (MODE != MMQ_OUT_BLOCKDOTS) {
#pragma unroll
                        for (int i = 0; i < CHUNK; i += 2) {
                            float f0, f1;
                            if constexpr (CVT == 0) {
                                f0 = __int2float_rn(static_cast<int>(vi[i]));
                                f1 = __int2float_rn(static_cast<int>(vi[i + 1]));
                            } else {
                                fadd2(f0, f1, __uint_as_float(vi[i] + MAGIC_BITS), __uint_as_float(vi[i + 1] + MAGIC_BITS),
                                      -MAGIC_F, -MAGIC_F);
                            }
                            ffma2(acc[c0 + i], acc[c0 + i + 1], f0, f1, __uint_as_float(vs[i]),
                                  __uint_as_float(vs[i + 1]));
                        }
                        if constexpr (MINS) {
                            // M = m_w s_x is exact in fp32, so acc + M is ggml's fma(m_w, s_x, acc)
                            tmem_ld_32x32b_x32(ta + 2 * C::BN + c0, vs);
                            tmem_wait_ld();
                            if (c0 + CHUNK == C::COLS) {
                                tc_fence_before();
                                mbar_arrive(&tempty[buf]);
                            }
#pragma unroll
                            for (int i = 0; i < CHUNK; i += 2)
                                fadd2(acc[c0 + i], acc[c0 + i + 1], acc[c0 + i], acc[c0 + i + 1], __uint_as_float(vs[i]),
                                      __uint_as_float(vs[i + 1]));
                        }
                    } else {
                        if (m < M) {
                            for (int i = 0; i < CHUNK; ++i) {
                                const int n = n0 + h * C::COLS + c0 + i;
                                if (n < N)
                                    dump[(static_cast<int64_t>(m) * N + n) * nblk + b] = static_cast<int32_t>(vi[i]);
                            }
                        }
                    }
                }
                ++blk;
            }
            if (!ok) break;
            if constexpr (MODE != MMQ_OUT_BLOCKDOTS) tile_store<MODE, C::COLS>(ep, acc, m, M, N, n0 + h * C::COLS);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, C::TMEM_COLS);
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
template <int MODE, int CVT, int BN, int EPQ = 2, int NIB = 0>
static cudaError_t launch_tc_epq(const MmqArgs &a, int num_sms, cudaStream_t s) {
    using C = TcCfg<BN, EPQ, NIB>;
    const int M = a.a.rows, N = a.b.rows, K = a.a.K, nblk = K / 32;
    CUtensorMap tma, tmb;
    const uint64_t da[2] = {uint64_t(K), uint64_t(M)}, sk[1] = {uint64_t(K)};
    const uint32_t bxa[2] = {C::BK, 32};
    // B: int8 codes [N][K] in 128-byte-swizzled boxes, or (NIB) nibble bytes [N][K/2] in plain 64-byte rows
    const uint64_t db[2] = {uint64_t(NIB ? K / 2 : K), uint64_t(N)}, skb[1] = {uint64_t(NIB ? K / 2 : K)};
    const uint32_t bxb[2] = {NIB ? C::BK / 2 : C::BK, C::BN};
    if (!make_tmap(&tma, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.a.codes, 2, da, sk, bxa, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_tmap(&tmb, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.b.codes, 2, db, skb, bxb,
                   NIB ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    auto kern = mmq_tc_kernel<MODE, CVT, BN, EPQ, NIB>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    const int tiles = ((M + C::ROWS - 1) / C::ROWS) * ((N + C::BN - 1) / C::BN);
    const int grid = tiles < C::CTAS * num_sms ? tiles : C::CTAS * num_sms;
    MmqEpi ep;
    ep.bias = a.bias;
    ep.y = a.y;
    ep.ldy = a.ldy;
    ep.dump = a.dump;
    ep.add = a.add;
    ep.rowmap = a.rowmap;
    ep.gelu = a.gelu;
    ep.qcodes = static_cast<int8_t *>(a.out_codes);
    ep.qquads = static_cast<__half *>(a.out_quads);
    ep.qld = a.out_ld;
    ep.q = static_cast<__nv_bfloat16 *>(a.q_out);
    ep.k = static_cast<__nv_bfloat16 *>(a.k_out);
    ep.vt = static_cast<__nv_bfloat16 *>(a.vt_out);
    ep.freqs = a.freqs;
    ep.win_tokens = a.win_tokens;
    ep.heads = a.heads;
    kern<<<grid, C::THREADS, C::SMEM_BYTES, s>>>(tma, tmb, static_cast<const uint8_t *>(a.a.quads),
                                                  static_cast<const uint8_t *>(a.b.quads), M, N, nblk, a.a.ld, a.b.ld,
                                                  ep, a.err, static_cast<const uint8_t *>(a.a_sums),
                                                  static_cast<const uint8_t *>(a.b_mins));
    return cudaGetLastError();
}

// Epilogue warps per used lane quarter: 4 (default; measured 48.1 against
// 42.1 images/s with 2) or 2 (tuning: env SAM3B200_MMQ_EPQ=2).
static int mmq_epq() {
    static const int v = [] {
        const char *ev = getenv("SAM3B200_MMQ_EPQ");
        return ev && atoi(ev) == 2 ? 2 : 4;
    }();
    return v;
}

template <int MODE, int CVT, int BN>
static cudaError_t launch_tc(const MmqArgs &a, int num_sms, cudaStream_t s) {
    // Q4_0 / Q4_1 nibble codes: BN 128 with 4 epilogue warps per quarter, whose idle warps 9 and 13 unpack
    if (a.b.nib == 1) return launch_tc_epq<MODE, CVT, 128, 4, 1>(a, num_sms, s);
    if constexpr (MODE == MMQ_OUT_F32 || MODE == MMQ_OUT_BLOCKDOTS)
        if (a.b.nib == 2) return launch_tc_epq<MODE, CVT, 128, 4, 2>(a, num_sms, s);
    if (a.b.nib == 2) return cudaErrorInvalidValue;  // Q4_1: f32 output only
    if constexpr (BN == 128)  // 4 warps per quarter need BN / 4 >= 32 columns each
        if (mmq_epq() == 4) return launch_tc_epq<MODE, CVT, BN, 4>(a, num_sms, s);
    return launch_tc_epq<MODE, CVT, BN, 2>(a, num_sms, s);
}

static bool valid_args(const MmqArgs &a) {
    const int M = a.a.rows, N = a.b.rows, K = a.a.K;
    return K == a.b.K && K > 0 && K % 32 == 0 && M > 0 && N > 0 && a.a.ld >= M && a.b.ld >= N &&
           a.a.ld % MMQ_ROW_ALIGN == 0 && a.b.ld % MMQ_ROW_ALIGN == 0;
}

// 8 epilogue warps: each thread drains 32 (BN = 64) or 64 (BN = 128) columns,
// so a 32-wide Q8_0 output block stays inside one thread.  (16 warps with a
// software-pipelined drain measured slower on B200.)
template <int BN>
static cudaError_t dispatch_tc(const MmqArgs &a, int mode, int num_sms, cudaStream_t s, int cvt) {
    if (mode == MMQ_OUT_BLOCKDOTS) return launch_tc<MMQ_OUT_BLOCKDOTS, 0, BN>(a, num_sms, s);
    if (mode == MMQ_OUT_Q8) {
        if (a.b.rows % 32 != 0 || !a.out_codes || !a.out_quads || a.out_ld < a.a.rows) return cudaErrorInvalidValue;
        return cvt == 0 ? launch_tc<MMQ_OUT_Q8, 0, BN>(a, num_sms, s) : launch_tc<MMQ_OUT_Q8, 1, BN>(a, num_sms, s);
    }
    if (mode == MMQ_OUT_F32)
        return cvt == 0 ? launch_tc<MMQ_OUT_F32, 0, BN>(a, num_sms, s)
                        : launch_tc<MMQ_OUT_F32, 1, BN>(a, num_sms, s);
    if (mode == MMQ_OUT_QKV) {
        if (!a.q_out || !a.k_out || !a.vt_out || a.heads <= 0 || a.b.rows != 3 * 64 * a.heads ||
            a.win_tokens <= 0 || a.a.rows % a.win_tokens != 0)
            return cudaErrorInvalidValue;
        return cvt == 0 ? launch_tc<MMQ_OUT_QKV, 0, BN>(a, num_sms, s) : launch_tc<MMQ_OUT_QKV, 1, BN>(a, num_sms, s);
    }
    return cudaErrorInvalidValue;
}

cudaError_t mmq_tc(const MmqArgs &a, int mode, int num_sms, cudaStream_t s, int cvt, int bn) {
    // auto: short K (many tiles per CTA, the tile stores a large share) on the two-CTA BN = 64
    // configuration, long K (few tiles, long K loops) on BN = 128 (measured at the ViT shapes:
    // qkv -6%, fc1 -11%, proj -2% with BN = 64 x 2 CTAs; fc2, K = 4736, +4%)
    if (bn == 0) bn = a.a.K <= 2048 ? 64 : 128;
    if (!valid_args(a) || num_sms <= 0 || a.a.nib != 0 ||
        (a.b.nib == 2) != (a.b_mins != nullptr) || (a.b.nib == 2 && !a.a_sums))  // Q4_1: minima and sum fields
        return cudaErrorInvalidValue;
    if (bn == 64) return dispatch_tc<64>(a, mode, num_sms, s, cvt);
    if (bn == 128) return dispatch_tc<128>(a, mode, num_sms, s, cvt);
    return cudaErrorInvalidValue;
}

// ---------------------------------------------------------------------------
// SIMT MMQ: one thread per output, same block-ordered fma sequence.
// ---------------------------------------------------------------------------
__global__ void mmq_simt_kernel(const int8_t *__restrict__ ca, const uint4 *__restrict__ qa, int lda_q,
                                const int8_t *__restrict__ cb, const uint4 *__restrict__ qb, int ldb_q, int M, int N,
                                int K, const float *__restrict__ bias, float *__restrict__ y, int64_t ldy,
                                int32_t *__restrict__ dump, int mode, const __half *__restrict__ mins_b,
                                const __half *__restrict__ sums_a, int nib) {
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    const int m = blockIdx.y;
    if (n >= N || m >= M) return;
    const int nblk = K >> 5;
    const int8_t *ar = ca + static_cast<int64_t>(m) * K;
    const int8_t *br = cb + static_cast<int64_t>(n) * (nib ? K / 2 : K);
    float acc = 0.f;
    for (int b = 0; b < nblk; ++b) {
        int isum = 0;
        for (int j = 0; j < 32; ++j) {
            int w;
            if (nib == 0) {
                w = br[b * 32 + j];
            } else {  // the block's nibble bytes: byte j % 16, low nibble for j < 16
                const int byte = static_cast<uint8_t>(br[b * 16 + (j & 15)]);
                w = (j < 16 ? (byte & 15) : (byte >> 4)) - (nib == 1 ? 8 : 0);
            }
            isum += static_cast<int>(ar[b * 32 + j]) * w;
        }
        if (mode == MMQ_OUT_BLOCKDOTS) {
            dump[(static_cast<int64_t>(m) * N + n) * nblk + b] = isum;
        } else {
            const float dx = __half2float(reinterpret_cast<const __half *>(qa)[act_quad_index(b, m, lda_q)]);
            const float dw = __half2float(reinterpret_cast<const __half *>(qb)[(static_cast<int64_t>(b) * ldb_q + n) * 8 + (b & 7)]);
            acc = fmaf(static_cast<float>(isum), dx * dw, acc);
            if (mins_b)  // Q4_1 x Q8_1: + m_w * s_x per block (ggml vec_dot_q4_1_q8_1)
                acc = fmaf(__half2float(mins_b[(static_cast<int64_t>(b) * ldb_q + n) * 8 + (b & 7)]),
                           __half2float(sums_a[act_quad_index(b, m, lda_q)]), acc);
        }
    }
    if (mode == MMQ_OUT_F32) y[static_cast<int64_t>(m) * ldy + n] = bias ? acc + bias[n] : acc;
}

// Skinny MUL_MAT (at most 64 activation rows, f32 output, Q8_0 / Q4_0 codes):
// the same per-block arithmetic as mmq_simt_kernel -- exact int32 block dot,
// acc = fma(float(I), d_x * d_w, acc) in block order -- so its outputs are
// bit-identical to it, with 16-byte loads of both code rows, the dots formed
// by __dp4a and the block loop unrolled so several blocks' loads are in
// flight.  CTA: 32 weight rows x 8 activation rows, one output per thread.
constexpr int SKINNY_MAX_M = 64;

// Q4_0 nibble codes of 4 bytes -> the int8 codes (nibble - 8) of their low
// (elements j..j+3) or high (j+16..j+19) nibbles; (n + 0x78) ^ 0x80 per byte.
__device__ __forceinline__ int q4_lo(int v) { return static_cast<int>(((static_cast<uint32_t>(v) & 0x0F0F0F0Fu) + 0x78787878u) ^ 0x80808080u); }
__device__ __forceinline__ int q4_hi(int v) {
    return static_cast<int>((((static_cast<uint32_t>(v) >> 4) & 0x0F0F0F0Fu) + 0x78787878u) ^ 0x80808080u);
}

template <int NIB>
__global__ void __launch_bounds__(256) mmq_skinny_kernel(const int8_t *__restrict__ ca, const __half *__restrict__ qa,
                                                         int lda_q, const int8_t *__restrict__ cb,
                                                         const __half *__restrict__ qb, int ldb_q, int M, int N, int K,
                                                         const float *__restrict__ bias, float *__restrict__ y,
                                                         int64_t ldy) {
    const int n = blockIdx.x * 32 + (threadIdx.x & 31);
    const int m = blockIdx.y * 8 + (threadIdx.x >> 5);
    if (n >= N || m >= M) return;
    const int nblk = K >> 5;
    const int4 *br = reinterpret_cast<const int4 *>(cb + static_cast<int64_t>(n) * (NIB ? K / 2 : K));
    const int4 *ar = reinterpret_cast<const int4 *>(ca + static_cast<int64_t>(m) * K);
    float acc = 0.f;
#pragma unroll 4
    for (int b = 0; b < nblk; ++b) {
        int4 w0, w1;
        if constexpr (NIB) {  // one 16-byte load holds the block's 32 codes
            const int4 p = __ldg(br + b);
            w0 = make_int4(q4_lo(p.x), q4_lo(p.y), q4_lo(p.z), q4_lo(p.w));
            w1 = make_int4(q4_hi(p.x), q4_hi(p.y), q4_hi(p.z), q4_hi(p.w));
        } else {
            w0 = __ldg(br + 2 * b);
            w1 = __ldg(br + 2 * b + 1);
        }
        const int4 a0 = __ldg(ar + 2 * b), a1 = __ldg(ar + 2 * b + 1);
        const float dw = __half2float(qb[(static_cast<int64_t>(b) * ldb_q + n) * 8 + (b & 7)]);
        const float dx = __half2float(qa[act_quad_index(b, m, lda_q)]);
        int isum = 0;
        isum = __dp4a(a0.x, w0.x, isum);
        isum = __dp4a(a0.y, w0.y, isum);
        isum = __dp4a(a0.z, w0.z, isum);
        isum = __dp4a(a0.w, w0.w, isum);
        isum = __dp4a(a1.x, w1.x, isum);
        isum = __dp4a(a1.y, w1.y, isum);
        isum = __dp4a(a1.z, w1.z, isum);
        isum = __dp4a(a1.w, w1.w, isum);
        acc = fmaf(static_cast<float>(isum), dx * dw, acc);
    }
    y[static_cast<int64_t>(m) * ldy + n] = bias ? acc + bias[n] : acc;
}

cudaError_t mmq_simt(const MmqArgs &a, int mode, cudaStream_t s) {
    if (!valid_args(a) || a.a.rows > 65535 || (a.b_mins && !a.a_sums)) return cudaErrorInvalidValue;
    const int M = a.a.rows, N = a.b.rows, K = a.a.K;
    const bool aligned = (reinterpret_cast<uintptr_t>(a.a.codes) & 15) == 0 &&
                         (reinterpret_cast<uintptr_t>(a.b.codes) & 15) == 0;
    if (mode == MMQ_OUT_F32 && !a.b_mins && a.b.nib != 2 && M <= SKINNY_MAX_M && aligned) {
        auto kern = a.b.nib == 1 ? mmq_skinny_kernel<1> : mmq_skinny_kernel<0>;
        kern<<<dim3((N + 31) / 32, (M + 7) / 8), 256, 0, s>>>(
            static_cast<const int8_t *>(a.a.codes), static_cast<const __half *>(a.a.quads), a.a.ld,
            static_cast<const int8_t *>(a.b.codes), static_cast<const __half *>(a.b.quads), a.b.ld, M, N, K, a.bias,
            a.y, a.ldy);
        return cudaGetLastError();
    }
    dim3 grid((N + 127) / 128, M);
    mmq_simt_kernel<<<grid, 128, 0, s>>>(static_cast<const int8_t *>(a.a.codes), static_cast<const uint4 *>(a.a.quads),
                                         a.a.ld, static_cast<const int8_t *>(a.b.codes),
                                         static_cast<const uint4 *>(a.b.quads), a.b.ld, M, N, K, a.bias, a.y, a.ldy,
                                         a.dump, mode, static_cast<const __half *>(a.b_mins),
                                         static_cast<const __half *>(a.a_sums), a.b.nib);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// DQ16 arithmetic (mmq.cuh): Q8_0 / Q4_0 operands dequantised to fp16 and one
// kind::f16 MMA pass over the whole of K per tile.
// ---------------------------------------------------------------------------
__global__ void dequant_act_f16_kernel(const int8_t *__restrict__ codes, const __half *__restrict__ quads, int M, int K,
                                       int ld, __half *__restrict__ out) {
    const int kg = K >> 3;
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;  // 8-element group
    if (i >= static_cast<int64_t>(M) * kg) return;
    const int m = static_cast<int>(i / kg), k = static_cast<int>(i % kg) * 8;
    const uint2 c = *reinterpret_cast<const uint2 *>(codes + static_cast<int64_t>(m) * K + k);
    const float d = __half2float(quads[act_quad_index(k >> 5, m, ld)]);
    uint32_t hw[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const uint32_t word = e < 2 ? c.x : c.y;
        const int sh = (e & 1) * 16;
        const float q0 = static_cast<float>(static_cast<int8_t>((word >> sh) & 0xFFu));
        const float q1 = static_cast<float>(static_cast<int8_t>((word >> (sh + 8)) & 0xFFu));
        const __half2 h2 = __floats2half2_rn(__fmul_rn(q0, d), __fmul_rn(q1, d));
        hw[e] = *reinterpret_cast<const uint32_t *>(&h2);
    }
    *reinterpret_cast<uint4 *>(out + static_cast<int64_t>(m) * K + k) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
}

cudaError_t dequant_act_f16(const void *codes, const void *quads, int M, int K, int ld, void *out, cudaStream_t s) {
    if (M <= 0 || K <= 0 || K % 32 != 0 || ld < M) return cudaErrorInvalidValue;
    const int64_t groups = static_cast<int64_t>(M) * (K >> 3);
    dequant_act_f16_kernel<<<static_cast<unsigned>((groups + 255) / 256), 256, 0, s>>>(
        static_cast<const int8_t *>(codes), static_cast<const __half *>(quads), M, K, ld, static_cast<__half *>(out));
    return cudaGetLastError();
}

template <int NIB>
__global__ void dequant_weight_f16_kernel(const uint8_t *__restrict__ codes, const __half *__restrict__ quads, int N,
                                          int K, int ld, __half *__restrict__ out) {
    const int kg = K >> 3;
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<int64_t>(N) * kg) return;
    const int n = static_cast<int>(i / kg), k = static_cast<int>(i % kg) * 8, b = k >> 5;
    const float d = __half2float(quads[(static_cast<int64_t>(b) * ld + n) * 8 + (b & 7)]);
    int q[8];
    if constexpr (NIB == 0) {
        const uint2 c = *reinterpret_cast<const uint2 *>(codes + static_cast<int64_t>(n) * K + k);
#pragma unroll
        for (int e = 0; e < 8; ++e) q[e] = static_cast<int8_t>(((e < 4 ? c.x : c.y) >> (8 * (e & 3))) & 0xFFu);
    } else {
        // Q4_0 block bytes: byte j holds element j (low nibble) and j + 16 (high nibble); code = nibble - 8
        const int j0 = k & 31;
        const uint2 c = *reinterpret_cast<const uint2 *>(codes + static_cast<int64_t>(n) * (K / 2) + b * 16 + (j0 & 15));
        const int sh = j0 < 16 ? 0 : 4;
#pragma unroll
        for (int e = 0; e < 8; ++e)
            q[e] = static_cast<int>((((e < 4 ? c.x : c.y) >> (8 * (e & 3) + sh)) & 0xFu)) - 8;
    }
    uint32_t hw[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const __half2 h2 = __floats2half2_rn(__fmul_rn(static_cast<float>(q[2 * e]), d),
                                             __fmul_rn(static_cast<float>(q[2 * e + 1]), d));
        hw[e] = *reinterpret_cast<const uint32_t *>(&h2);
    }
    *reinterpret_cast<uint4 *>(out + static_cast<int64_t>(n) * K + k) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
}

cudaError_t dequant_weight_f16(const QMatrix &w, void *out, cudaStream_t s) {
    if (w.rows <= 0 || w.K <= 0 || w.K % 32 != 0 || w.ld < w.rows || (w.nib != 0 && w.nib != 1))
        return cudaErrorInvalidValue;
    const int64_t groups = static_cast<int64_t>(w.rows) * (w.K >> 3);
    const unsigned grid = static_cast<unsigned>((groups + 255) / 256);
    auto kern = w.nib == 1 ? dequant_weight_f16_kernel<1> : dequant_weight_f16_kernel<0>;
    kern<<<grid, 256, 0, s>>>(static_cast<const uint8_t *>(w.codes), static_cast<const __half *>(w.quads), w.rows, w.K,
                              w.ld, static_cast<__half *>(out));
    return cudaGetLastError();
}

// ---- warp-staged row segments (the DQ16 epilogue's stores) -----------------
// Every epilogue lane owns one output row (its TMEM lane), so a per-lane
// store touches 32 cache lines per instruction, and the L1 replays it 32
// times.  Instead each lane puts a 64-byte segment of its row into a per-warp
// 2 KB staging buffer -- 16-byte chunks XOR-swizzled by (row >> 1) & 3, which
// keeps both the row-per-lane writes and the 8-rows-per-instruction reads
// free of bank conflicts -- and the warp writes 8 rows x 64 bytes per
// instruction.  Row mappings (window order, head split) are per row, so any
// destination layout with 16-byte-aligned row segments works.
// (stage_idx / stage_put: ptx.cuh)

__device__ __forceinline__ uint32_t f2_bits(float a) { return __float_as_uint(a); }
__device__ __forceinline__ uint32_t bf2_bits(float a, float b) {
    const __nv_bfloat162 p = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&p);
}

// tile_store of the DQ16 kernel for MODE F32 / DQ16 / QKV, warp-collective
// (every lane of the warp calls it, rows m >= M included); m = this lane's tile
// row, the warp's rows are m - lane .. m - lane + 31.  Same arithmetic as
// tile_store, only the memory access pattern differs.
__device__ __forceinline__ bool f32_rows_vec(const MmqEpi &ep, int N) {
    return ((ep.ldy & 3) == 0) && ((reinterpret_cast<uintptr_t>(ep.y) & 15) == 0) && ((N & 3) == 0);
}

// The residual values tile_store_staged's MMQ_OUT_F32 path adds for COLS
// columns from nb (rounds of 16 columns, 8 rows x 64 bytes per load), read
// before the tile's accumulator is ready so their latency overlaps its MMAs.
template <int COLS>
__device__ __forceinline__ void prefetch_residual(const MmqEpi &ep, float4 (&pre)[COLS / 16][4], int m, int M, int N,
                                                  int nb, int lane) {
    const int myrow = m < M ? (ep.rowmap ? ep.rowmap[m] : m) : -1;
#pragma unroll
    for (int it = 0; it < 4; ++it) {
        const int r = it * 8 + (lane >> 2), ch = lane & 3;
        const int orow = __shfl_sync(0xffffffffu, myrow, r);
#pragma unroll
        for (int c = 0; c < COLS / 16; ++c) {
            const int n = nb + c * 16 + ch * 4;
            pre[c][it] = orow >= 0 && n < N
                             ? *reinterpret_cast<const float4 *>(ep.y + static_cast<int64_t>(orow) * ep.ldy + n)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
}

template <int MODE, int COLS>
__device__ __forceinline__ void tile_store_staged(const MmqEpi &ep, float (&acc)[COLS], int m, int M, int N, int nb,
                                                  uint4 *st, int lane, const float4 (*pre)[4] = nullptr) {
    constexpr unsigned FULL = 0xffffffffu;
    const float *__restrict__ bias = ep.bias;
    const int m_warp = m - lane;
    if constexpr (MODE == MMQ_OUT_F32) {
        const bool vec = f32_rows_vec(ep, N);
        if (!vec) {  // warp-uniform: the per-lane path handles any stride / width
            tile_store<MODE, COLS>(ep, acc, m, M, N, nb);
            return;
        }
        if (bias) {
#pragma unroll
            for (int i = 0; i < COLS; ++i)
                if (nb + i < N) acc[i] = __fadd_rn(acc[i], bias[nb + i]);
        }
        const int myrow = m < M ? (ep.rowmap ? ep.rowmap[m] : m) : -1;
#pragma unroll
        for (int c0 = 0; c0 < COLS; c0 += 16) {
            uint4 seg[4];
#pragma unroll
            for (int k = 0; k < 4; ++k)
                seg[k] = make_uint4(f2_bits(acc[c0 + 4 * k]), f2_bits(acc[c0 + 4 * k + 1]), f2_bits(acc[c0 + 4 * k + 2]),
                                    f2_bits(acc[c0 + 4 * k + 3]));
            stage_put(st, lane, seg);
#pragma unroll
            for (int it = 0; it < 4; ++it) {
                const int r = it * 8 + (lane >> 2), ch = lane & 3;
                const int orow = __shfl_sync(FULL, myrow, r);
                const int n = nb + c0 + ch * 4;
                if (orow >= 0 && n < N) {
                    const uint4 v = st[stage_idx(r, ch)];
                    float4 f = make_float4(__uint_as_float(v.x), __uint_as_float(v.y), __uint_as_float(v.z),
                                           __uint_as_float(v.w));
                    float *p = ep.y + static_cast<int64_t>(orow) * ep.ldy + n;
                    if (ep.add) {
                        const float4 prev = pre ? pre[c0 / 16][it] : *reinterpret_cast<const float4 *>(p);
                        f.x = __fadd_rn(prev.x, f.x);
                        f.y = __fadd_rn(prev.y, f.y);
                        f.z = __fadd_rn(prev.z, f.z);
                        f.w = __fadd_rn(prev.w, f.w);
                    }
                    *reinterpret_cast<float4 *>(p) = f;
                }
            }
        }
    } else if constexpr (MODE == MMQ_OUT_DQ16) {
        const int rowok = m < M;
#pragma unroll
        for (int hb = 0; hb < COLS; hb += 32) {
            if (nb + hb >= N) break;  // warp-uniform
            float amax = 0.f;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                float val = bias ? __fadd_rn(acc[hb + i], bias[nb + hb + i]) : acc[hb + i];
                if (ep.gelu == 1) val = gelu_erf_f(val);
                else if (ep.gelu == 2) val = gelu_tanh_f16(val);
                acc[hb + i] = val;
                amax = fmaxf(amax, fabsf(val));
            }
            const float d = __fdiv_rn(amax, 127.f);
            const float id = amax != 0.f ? __fdiv_rn(127.f, amax) : 0.f;
            const float dh = __half2float(__float2half_rn(d));  // the block's stored (fp16) scale
            uint32_t hw[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                const float q0 = q8_code_f(__fmul_rn(acc[hb + 2 * e], id));
                const float q1 = q8_code_f(__fmul_rn(acc[hb + 2 * e + 1], id));
                const __half2 h2 = __floats2half2_rn(__fmul_rn(q0, dh), __fmul_rn(q1, dh));
                hw[e] = *reinterpret_cast<const uint32_t *>(&h2);
            }
            const uint4 seg[4] = {make_uint4(hw[0], hw[1], hw[2], hw[3]), make_uint4(hw[4], hw[5], hw[6], hw[7]),
                                  make_uint4(hw[8], hw[9], hw[10], hw[11]), make_uint4(hw[12], hw[13], hw[14], hw[15])};
            stage_put(st, lane, seg);
#pragma unroll
            for (int it = 0; it < 4; ++it) {
                const int r = it * 8 + (lane >> 2), ch = lane & 3;
                if (__shfl_sync(FULL, rowok, r))
                    *reinterpret_cast<uint4 *>(ep.o16 + static_cast<int64_t>(m_warp + r) * N + nb + hb + ch * 8) =
                        st[stage_idx(r, ch)];
            }
        }
    } else if constexpr (MODE == MMQ_OUT_QKV) {
        // this thread's COLS columns lie inside one 64-wide head of the q, k or v third;
        // M is a multiple of win_tokens and a warp's 32 rows never straddle a window
        const int E = N / 3;
        const int part = nb / E, c0h = nb - part * E, hd = c0h >> 6, d0 = c0h & 63;
        const int win = m / ep.win_tokens, pos = m - win * ep.win_tokens;
        const int64_t bh = static_cast<int64_t>(win) * ep.heads + hd;
        if (bias) {
#pragma unroll
            for (int i = 0; i < COLS; ++i) acc[i] = __fadd_rn(acc[i], bias[nb + i]);
        }
        if (part < 2) {
            if (ep.freqs) {
                // the row's RoPE (cos, sin) pairs, gathered 8 rows x 64 bytes per instruction
#pragma unroll
                for (int c0 = 0; c0 < COLS; c0 += 16) {
                    __syncwarp();
#pragma unroll
                    for (int it = 0; it < 4; ++it) {
                        const int r = it * 8 + (lane >> 2), ch = lane & 3;
                        const int pr = __shfl_sync(FULL, pos, r);
                        st[stage_idx(r, ch)] = *reinterpret_cast<const uint4 *>(
                            ep.freqs + (static_cast<int64_t>(pr) * 32 + (d0 >> 1)) * 2 + c0 + ch * 4);
                    }
                    __syncwarp();
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const uint4 cs = st[stage_idx(lane, k)];  // cos, sin of pairs c0/2 + 2k, + 1
                        const int i = c0 + 4 * k;
                        float x0 = acc[i], x1 = acc[i + 1];
                        acc[i] = __fsub_rn(__fmul_rn(x0, __uint_as_float(cs.x)), __fmul_rn(x1, __uint_as_float(cs.y)));
                        acc[i + 1] = __fadd_rn(__fmul_rn(x0, __uint_as_float(cs.y)), __fmul_rn(x1, __uint_as_float(cs.x)));
                        x0 = acc[i + 2];
                        x1 = acc[i + 3];
                        acc[i + 2] = __fsub_rn(__fmul_rn(x0, __uint_as_float(cs.z)), __fmul_rn(x1, __uint_as_float(cs.w)));
                        acc[i + 3] = __fadd_rn(__fmul_rn(x0, __uint_as_float(cs.w)), __fmul_rn(x1, __uint_as_float(cs.z)));
                    }
                }
            }
            const int64_t base = m < M ? (bh * ep.win_tokens + pos) * 64 + d0 : -1;
            __nv_bfloat16 *dst = part == 0 ? ep.q : ep.k;
#pragma unroll
            for (int c0 = 0; c0 < COLS; c0 += 32) {
                uint4 seg[4];
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    seg[k] = make_uint4(bf2_bits(acc[c0 + 8 * k], acc[c0 + 8 * k + 1]),
                                        bf2_bits(acc[c0 + 8 * k + 2], acc[c0 + 8 * k + 3]),
                                        bf2_bits(acc[c0 + 8 * k + 4], acc[c0 + 8 * k + 5]),
                                        bf2_bits(acc[c0 + 8 * k + 6], acc[c0 + 8 * k + 7]));
                stage_put(st, lane, seg);
#pragma unroll
                for (int it = 0; it < 4; ++it) {
                    const int r = it * 8 + (lane >> 2), ch = lane & 3;
                    const long long b = __shfl_sync(FULL, static_cast<long long>(base), r);
                    if (b >= 0) *reinterpret_cast<uint4 *>(dst + b + c0 + ch * 8) = st[stage_idx(r, ch)];
                }
            }
        } else if (m < M) {
            // V^T: consecutive lanes hold consecutive tokens, so each store is 64 contiguous bytes
            __nv_bfloat16 *dst = ep.vt + (bh * 64 + d0) * ep.win_tokens + pos;
#pragma unroll
            for (int i = 0; i < COLS; ++i) dst[static_cast<int64_t>(i) * ep.win_tokens] = __float2bfloat16_rn(acc[i]);
        }
    } else {
        tile_store<MODE, COLS>(ep, acc, m, M, N, nb);
    }
}

// CTA tile 128 tokens x BN features, persistent over tiles, 576 threads:
//   warp 0      : TMA producer (one elected lane): 64-wide K stages of A
//                 (128 rows) and B (BN rows), 128-byte swizzle;
//   warp 1      : TMEM allocator + MMA issuer (one elected lane): four K = 16
//                 MMAs per stage into accumulator buffer (tile & 1), BN
//                 columns each, so a tile's epilogue overlaps the next
//                 tile's MMAs;
//   warps 2..17 : epilogue, four per TMEM lane quarter (warp w reads lane
//                 quarter w % 4, column slice (w - 2) / 4 of BN / 4 columns),
//                 then the mode's epilogue (bias, residual through the row
//                 map, RoPE + head split, GELU + Q8_0 re-quantisation) with
//                 its stores staged through shared memory (tile_store_staged).
template <int BN_>
struct DqCfg {
    static constexpr int BM = 128, BN = BN_, BK = 64;
    static constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGES = BN == 256 ? 4 : 6;
    static constexpr int BAR_OFF = STAGES * STAGE_BYTES;
    static constexpr int EPI_WARPS = 16;
    static constexpr int THREADS = 64 + 32 * EPI_WARPS;
    static constexpr int COLS = BN / 4;  // output columns per epilogue thread
    static constexpr int TMEM_COLS = 2 * BN;
    static constexpr int STAGE_OFF = BAR_OFF + 256;  // per-warp 2 KB row-segment staging (tile_store_staged)
    static constexpr int SMEM_BYTES = STAGE_OFF + EPI_WARPS * 2048 + 1024;
    static_assert(COLS % 32 == 0 && COLS <= 64, "whole 32-column TMEM loads, inside one 64-wide head");
    static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

template <int MODE, int BN>
__global__ void __launch_bounds__(DqCfg<BN>::THREADS, 1)
    mmq_dq16_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b, int M, int N,
                    int K, const MmqEpi ep, int *__restrict__ err) {
    using C = DqCfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
    uint64_t *empty = full + C::STAGES;
    uint64_t *tfull = empty + C::STAGES;
    uint64_t *tempty = tfull + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tempty + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int num_m = (M + C::BM - 1) / C::BM, num_n = (N + C::BN - 1) / C::BN;
    const int num_tiles = num_m * num_n;
    const int kstages = (K + C::BK - 1) / C::BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], C::EPI_WARPS);
        }
        fence_mbar_init();
        prefetch_tmap(&tm_a);
        prefetch_tmap(&tm_b);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
            const int m0 = (t % num_m) * C::BM, n0 = (t / num_m) * C::BN;
            for (int ks = 0; ks < kstages; ++ks) {
                if (!__all_sync(0xffffffffu, mbar_wait(&empty[stage], phase ^ 1u, err, ERR_WAIT_EMPTY))) {
                    ok = false;
                    break;
                }
                uint8_t *sb = smem + stage * C::STAGE_BYTES;
                if (elect_one()) {
                    mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
                    tma_load_2d(sb, &tm_a, &full[stage], ks * C::BK, m0);
                    tma_load_2d(sb + C::A_BYTES, &tm_b, &full[stage], ks * C::BK, n0);
                }
                __syncwarp();
                if (++stage == C::STAGES) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
        }
    } else if (warp == 1) {
        constexpr uint32_t idesc = idesc_f16_f32(C::BM, C::BN);
        int stage = 0;
        uint32_t phase = 0, it = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++it) {
            const uint32_t buf = it & 1u;
            if (!__all_sync(0xffffffffu, mbar_wait(&tempty[buf], ((it >> 1) & 1u) ^ 1u, err, ERR_WAIT_TEMPTY))) break;
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + buf * C::BN;
            for (int ks = 0; ks < kstages; ++ks) {
                if (!__all_sync(0xffffffffu, mbar_wait(&full[stage], phase, err, ERR_WAIT_FULL_MMA))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t a_addr = smem_u32(smem + stage * C::STAGE_BYTES);
                const uint32_t b_addr = a_addr + C::A_BYTES;
                if (elect_one()) {
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        mma_f16(d_tmem, sw128_kmajor_desc(a_addr + kk * 32), sw128_kmajor_desc(b_addr + kk * 32), idesc,
                                (ks | kk) != 0);
                    mma_commit(&empty[stage]);
                }
                __syncwarp();
                if (++stage == C::STAGES) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (!ok) break;
            if (elect_one()) mma_commit(&tfull[buf]);
            __syncwarp();
        }
    } else {
        const int q = warp & 3;
        const int cs = ((warp - 2) >> 2) * C::COLS;
        const int row = q * 32 + lane;
        const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
        uint32_t it = 0;
        // F32 with a residual add at 32 columns per thread (proj, fc2): the residual is read early
        constexpr bool PREF = MODE == MMQ_OUT_F32 && C::COLS == 32;
        const bool pref = PREF && ep.add && f32_rows_vec(ep, N);
        for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++it) {
            const uint32_t buf = it & 1u;
            const int m0 = (t % num_m) * C::BM, n0 = (t / num_m) * C::BN;
            float4 pre[PREF ? C::COLS / 16 : 1][4];
            if constexpr (PREF)
                if (pref) prefetch_residual<C::COLS>(ep, pre, m0 + row, M, N, n0 + cs, lane);
            if (!__all_sync(0xffffffffu, mbar_wait(&tfull[buf], (it >> 1) & 1u, err, ERR_WAIT_TFULL))) break;
            tc_fence_after();
            uint32_t v[C::COLS];
#pragma unroll
            for (int c = 0; c < C::COLS; c += 32)
                tmem_ld_32x32b_x32(tmem_base + lane_addr + buf * C::BN + cs + c, *reinterpret_cast<uint32_t(*)[32]>(v + c));
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[buf]);
            float acc[C::COLS];
#pragma unroll
            for (int i = 0; i < C::COLS; ++i) acc[i] = __uint_as_float(v[i]);
            tile_store_staged<MODE, C::COLS>(ep, acc, m0 + row, M, N, n0 + cs,
                                             reinterpret_cast<uint4 *>(smem + C::STAGE_OFF) + (warp - 2) * 128, lane,
                                             PREF && pref ? pre : nullptr);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, C::TMEM_COLS);
}

static MmqEpi dq16_epi(const MmqArgs &a) {
    MmqEpi ep;
    ep.bias = a.bias;
    ep.y = a.y;
    ep.ldy = a.ldy;
    ep.dump = nullptr;
    ep.add = a.add;
    ep.rowmap = a.rowmap;
    ep.gelu = a.gelu;
    ep.qcodes = static_cast<int8_t *>(a.out_codes);
    ep.qquads = static_cast<__half *>(a.out_quads);
    ep.qld = a.out_ld;
    ep.q = static_cast<__nv_bfloat16 *>(a.q_out);
    ep.k = static_cast<__nv_bfloat16 *>(a.k_out);
    ep.vt = static_cast<__nv_bfloat16 *>(a.vt_out);
    ep.freqs = a.freqs;
    ep.win_tokens = a.win_tokens;
    ep.heads = a.heads;
    ep.o16 = static_cast<__half *>(a.out16);
    return ep;
}

template <int MODE, int BN>
static cudaError_t launch_dq16(const MmqArgs &a, const void *a16, const void *b16, int num_sms, cudaStream_t s) {
    using C = DqCfg<BN>;
    const int M = a.a.rows, N = a.b.rows, K = a.a.K;
    CUtensorMap ta, tb;
    const uint64_t da[2] = {uint64_t(K), uint64_t(M)}, db[2] = {uint64_t(K), uint64_t(N)};
    const uint64_t st[1] = {uint64_t(K) * 2};
    const uint32_t bxa[2] = {C::BK, C::BM}, bxb[2] = {C::BK, C::BN};
    if (!make_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a16, 2, da, st, bxa, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, b16, 2, db, st, bxb, CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    auto kern = mmq_dq16_kernel<MODE, BN>;
    // the shared-memory opt-in, once per device and instantiation (a host call per launch otherwise)
    static std::atomic<uint64_t> attr_done{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = dev < 64 ? (uint64_t(1) << dev) : 0;
    if (!bit || !(attr_done.load(std::memory_order_relaxed) & bit)) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
        if (e != cudaSuccess) return e;
        attr_done.fetch_or(bit, std::memory_order_relaxed);
    }
    const int tiles = ((M + C::BM - 1) / C::BM) * ((N + C::BN - 1) / C::BN);
    const int grid = tiles < num_sms ? tiles : num_sms;
    kern<<<grid, C::THREADS, C::SMEM_BYTES, s>>>(ta, tb, M, N, K, dq16_epi(a), a.err);
    return cudaGetLastError();
}

template <int BN>
static cudaError_t dispatch_dq16(const MmqArgs &a, const void *a16, const void *b16, int mode, int num_sms,
                                 cudaStream_t s) {
    if (mode == MMQ_OUT_F32) return launch_dq16<MMQ_OUT_F32, BN>(a, a16, b16, num_sms, s);
    if (mode == MMQ_OUT_DQ16) {
        if (a.b.rows % 32 != 0 || !a.out16) return cudaErrorInvalidValue;
        return launch_dq16<MMQ_OUT_DQ16, BN>(a, a16, b16, num_sms, s);
    }
    if (mode == MMQ_OUT_Q8) {
        if (a.b.rows % 32 != 0 || !a.out_codes || !a.out_quads || a.out_ld < a.a.rows) return cudaErrorInvalidValue;
        return launch_dq16<MMQ_OUT_Q8, BN>(a, a16, b16, num_sms, s);
    }
    if (mode == MMQ_OUT_QKV) {
        if (!a.q_out || !a.k_out || !a.vt_out || a.heads <= 0 || a.b.rows != 3 * 64 * a.heads ||
            a.win_tokens <= 0 || a.a.rows % a.win_tokens != 0)
            return cudaErrorInvalidValue;
        return launch_dq16<MMQ_OUT_QKV, BN>(a, a16, b16, num_sms, s);
    }
    return cudaErrorInvalidValue;
}

// Tile width from the tile count: persistent CTAs take ceil(tiles / SMs)
// tiles each, and a BN-wide tile costs about BN + 64 columns' worth of time
// (the fixed part: its epilogue handshake and pipeline fill).
static int dq16_pick_bn(int M, int N, int num_sms) {
    static const int forced = [] {
        const char *ev = getenv("SAM3B200_DQ16_BN");
        return ev ? atoi(ev) : 0;
    }();
    if (forced == 128 || forced == 256) return forced;
    auto cost = [&](int bn) {
        const long long tiles = static_cast<long long>((M + 127) / 128) * ((N + bn - 1) / bn);
        return ((tiles + num_sms - 1) / num_sms) * (bn + 64);
    };
    return cost(256) <= cost(128) ? 256 : 128;
}

cudaError_t mmq_dq16(const MmqArgs &a, const void *a16, const void *b16, int mode, int num_sms, cudaStream_t s,
                     int bn) {
    const int M = a.a.rows, N = a.b.rows, K = a.a.K;
    if (!a16 || !b16 || M <= 0 || N <= 0 || K <= 0 || K % 8 != 0 || K != a.b.K || num_sms <= 0 ||
        (reinterpret_cast<uintptr_t>(a16) & 15) || (reinterpret_cast<uintptr_t>(b16) & 15))
        return cudaErrorInvalidValue;
    if (a.bias && (reinterpret_cast<uintptr_t>(a.bias) & 15)) return cudaErrorInvalidValue;
    if (bn == 0) bn = dq16_pick_bn(M, N, num_sms);
    if (bn == 128) return dispatch_dq16<128>(a, a16, b16, mode, num_sms, s);
    if (bn == 256) return dispatch_dq16<256>(a, a16, b16, mode, num_sms, s);
    return cudaErrorInvalidValue;
}

}  // namespace b200
