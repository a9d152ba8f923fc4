// attn.cu -- ggml_flash_attn_ext without mask (sam3.cpp:3778): per (window,
// head) out = softmax(Q K^T * scale) V, head_dim 64, on the 5th-generation
// tensor cores.  Q and K are bf16 [B*heads][N][64], V is stored transposed,
// bf16 [B*heads][64][N]; the output is [B*N][heads*64] (ggml's
// [HD, NH, N, B] result reshaped to [E, W, H, B], sam3.cpp:3780-3781), either
// f32 or -- for the proj MUL_MAT that follows -- quantised to Q8_0 with the
// ggml-cpu activation rule (each softmax thread holds two whole 32-wide
// blocks of its row), bit-identical to quantising the f32 output.
//
// A CTA owns two query tiles (t = 0, 1) of 96 queries of one (window, head)
// and streams the keys in tiles of 128.  The MMAs are M = 128; the TMEM lane
// quarter of sub-partition 1 (MMA rows 32..63), where the MMA issuer and the
// producer run, carries zero query rows, so no softmax warp shares their
// sub-partition (such warps fall behind and hold every hand-off back).  576
// and 5184 tokens are whole numbers of 192-query CTAs.
//   warp 5     : TMA producer -- both Q tiles once (three 32-row boxes into
//                MMA rows 0..31 and 64..127), then K and V^T tiles through a
//                STAGES-deep ring (128-byte swizzle, zero fill past N);
//   warp 1     : TMEM allocator + MMA issuer -- S_t(j) = Q_t K_j^T (M = 128,
//                N = 128 keys, K = 64) and, once softmax t has written
//                P_t(j), PV_t(j) = P_t(j) V_j (A = P read from tensor memory,
//                N = 64, K = 128 keys) followed by S_t(j+1), with one commit
//                (ready[t]) for the pair: commits hold the issuing thread far
//                longer than MMAs.  The tiles alternate, so the tensor core
//                works on one tile while the other tile's softmax runs;
//   warps w with w % 4 != 1 (12 of the 16): softmax.  Warp w serves tile
//                (w >> 2) & 1, TMEM lane quarter w % 4 (the only quarter its
//                sub-partition can read) and half w >> 3 of every query row:
//                keys 64 h .. 64 h + 63 of each key tile and output
//                dimensions 32 h .. 32 h + 31.  Per key tile each half reads
//                its 64 scores, takes their max, exchanges it with the other
//                half through shared memory (a named barrier of the two
//                warps), writes P = 2^(s c - m) as bf16 into tensor memory and
//                sums it; its 32 output dimensions stay in registers and
//                PV_t(j-1) is folded in as O = O 2^(m(j-2) - m(j-1)) + PV_t(j-1),
//                one step behind.  The two halves' row sums are added at the
//                end, and each half quantises its own 32-wide Q8_0 block.
// Tensor memory (512 columns): tile t at 256 t: S (128 columns), P (64: 128
// bf16 packed in pairs), PV (64).
#include "attn.cuh"
#include "mmq.cuh"
#include "ptx.cuh"
#include "tmap.h"

#include <cstdint>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace b200 {

namespace {

struct AttnCfg {
    static constexpr int BQ = 128, ROWS = 96, BKV = 128, HD = 64, QT = 2;
    static constexpr int STAGES = 3;
    static constexpr int Q_BYTES = BQ * HD * 2;         // 16 KB per query tile
    static constexpr int K_BYTES = BKV * HD * 2;        // 16 KB
    static constexpr int V_BYTES = HD * BKV * 2;        // 16 KB: two 64-key halves of 64 rows x 128 B
    static constexpr int STAGE_BYTES = K_BYTES + V_BYTES;
    static constexpr int KV_OFF = QT * Q_BYTES;
    static constexpr int BAR_OFF = KV_OFF + STAGES * STAGE_BYTES;  // 128 KB: one CTA per SM
    // softmax halves' exchange: values, then ok flags, each [2 parities][QT][4 quarters][2 halves][32 lanes]
    static constexpr int XCH_OFF = BAR_OFF + 256;
    static constexpr int XCH_BYTES = 2 * QT * 4 * 2 * 32 * 4;
    static constexpr int SMEM_BYTES = XCH_OFF + 2 * XCH_BYTES + 1024;
    static constexpr int THREADS = 512;
    static constexpr uint32_t S_COL = 0, P_COL = 128, PV_COL = 192, TILE_COLS = 256;
    static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

enum : int {
    AERR_Q = 1 << 8,
    AERR_KV_EMPTY = 1 << 9,
    AERR_KV_FULL = 1 << 10,
    AERR_S_EMPTY = 1 << 11,
    AERR_P_FULL = 1 << 12,
    AERR_PV_EMPTY = 1 << 13,
    AERR_S_FULL = 1 << 14,
    AERR_PV_FULL = 1 << 15,
};

// Row max over 32 scores (the keys past N are skipped when MASKED).
template <bool MASKED>
__device__ __forceinline__ float chunk_max(const uint32_t (&s)[32], float mx, int nvalid_here) {
#pragma unroll
    for (int i = 0; i < 32; ++i)
        if (!MASKED || i < nvalid_here) mx = fmaxf(mx, __uint_as_float(s[i]));
    return mx;
}

// p = 2^(s c - m) for 32 scores, packed as bf16 pairs; returns the sum of p.
template <bool MASKED>
__device__ __forceinline__ float chunk_exp(const uint32_t (&s)[32], float c, float neg_m, uint32_t (&pk)[16],
                                           int nvalid_here) {
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
        float p0 = ex2_approx(fmaf(__uint_as_float(s[i]), c, neg_m));
        float p1 = ex2_approx(fmaf(__uint_as_float(s[i + 1]), c, neg_m));
        if (MASKED) {
            if (i >= nvalid_here) p0 = 0.f;
            if (i + 1 >= nvalid_here) p1 = 0.f;
        }
        sum += p0 + p1;
        const __nv_bfloat162 h = __floats2bfloat162_rn(p0, p1);
        pk[i >> 1] = *reinterpret_cast<const uint32_t *>(&h);
    }
    return sum;
}

}  // namespace

__global__ void __launch_bounds__(AttnCfg::THREADS, 1)
    flash_attn_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, int N, int heads, float c_log2,
                         float *__restrict__ out, int8_t *__restrict__ qcodes, __half *__restrict__ qquads, int qld,
                         __half *__restrict__ o16,
                         int *__restrict__ err) {
    using C = AttnCfg;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *q_full = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
    uint64_t *kv_full = q_full + 1;
    uint64_t *kv_empty = kv_full + C::STAGES;
    // ready[t] phase j: S_t(j) (and PV_t(j-1)) are in tensor memory.
    // pdone[t] phase j: softmax t has read S_t(j), folded PV_t(j-1) and written P_t(j).
    uint64_t *ready = kv_empty + C::STAGES;  // [QT]
    uint64_t *pdone = ready + C::QT;         // [QT]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(pdone + C::QT);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int bh = blockIdx.y;
    const int q0 = blockIdx.x * C::QT * C::ROWS;
    const int ntiles = (N + C::BKV - 1) / C::BKV;
    const int nq = N - q0 > C::ROWS ? C::QT : 1;  // query tiles of this CTA that hold rows < N

    // MMA rows 32..63 of both Q tiles stay zero (TMA writes rows 0..31 and 64..127)
    for (int i = threadIdx.x; i < C::QT * 32 * 128 / 16; i += blockDim.x) {
        const int t = i / (32 * 128 / 16), j = i % (32 * 128 / 16);
        *reinterpret_cast<uint4 *>(smem + t * C::Q_BYTES + 32 * 128 + j * 16) = make_uint4(0u, 0u, 0u, 0u);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        for (int t = 0; t < C::QT; ++t) {
            mbar_init(&ready[t], 1);
            mbar_init(&pdone[t], 6);  // both halves of the three lane quarters
        }
        fence_mbar_init();
        prefetch_tmap(&tm_q);
        prefetch_tmap(&tm_k);
        prefetch_tmap(&tm_v);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 5) {
        // ---- TMA producer ----
        if (elect_one()) {
            mbar_arrive_expect_tx(q_full, nq * 3 * 32 * 128);
            for (int t = 0; t < nq; ++t) {
                uint8_t *qb = smem + t * C::Q_BYTES;
                const int r0 = q0 + t * C::ROWS;
                tma_load_3d(qb, &tm_q, q_full, 0, r0, bh);                 // MMA rows 0..31
                tma_load_3d(qb + 64 * 128, &tm_q, q_full, 0, r0 + 32, bh);  // 64..95
                tma_load_3d(qb + 96 * 128, &tm_q, q_full, 0, r0 + 64, bh);  // 96..127
            }
        }
        __syncwarp();
        for (int j = 0; j < ntiles; ++j) {
            const int st = j % C::STAGES;
            if (!__all_sync(0xffffffffu, mbar_wait(&kv_empty[st], ((j / C::STAGES) & 1) ^ 1, err, AERR_KV_EMPTY)))
                break;
            uint8_t *kb = smem + C::KV_OFF + st * C::STAGE_BYTES;
            if (elect_one()) {
                mbar_arrive_expect_tx(&kv_full[st], C::STAGE_BYTES);
                tma_load_3d(kb, &tm_k, &kv_full[st], 0, j * C::BKV, bh);
                tma_load_3d(kb + C::K_BYTES, &tm_v, &kv_full[st], j * C::BKV, 0, bh);
                tma_load_3d(kb + C::K_BYTES + C::V_BYTES / 2, &tm_v, &kv_full[st], j * C::BKV + 64, 0, bh);
            }
            __syncwarp();
        }
    } else if (warp == 1) {
        // ---- MMA issuer ----
        constexpr uint32_t idesc_s = idesc_bf16_f32(128, C::BKV);
        constexpr uint32_t idesc_pv = idesc_bf16_f32(128, C::HD);
        // S_t(j) = Q_t K_j^T (caller has waited for stage j and for S_t to be free)
        auto mma_s = [&](int t, int j) {
            const uint32_t q_addr = smem_u32(smem + t * C::Q_BYTES);
            const uint32_t k_addr = smem_u32(smem + C::KV_OFF + (j % C::STAGES) * C::STAGE_BYTES);
#pragma unroll
            for (int kk = 0; kk < C::HD / 16; ++kk)
                mma_f16(tmem + t * C::TILE_COLS + C::S_COL, sw128_kmajor_desc(q_addr + kk * 32),
                        sw128_kmajor_desc(k_addr + kk * 32), idesc_s, kk > 0);
        };
        // PV_t(j) = P_t(j) V_j
        auto mma_pv = [&](int t, int j) {
            const uint32_t v_addr = smem_u32(smem + C::KV_OFF + (j % C::STAGES) * C::STAGE_BYTES + C::K_BYTES);
#pragma unroll
            for (int kk = 0; kk < C::BKV / 16; ++kk) {
                // keys 16 kk .. +15: 64-key half kk / 4, 32-byte slice kk % 4 of its 128-byte rows
                const uint32_t va = v_addr + (kk >> 2) * (C::V_BYTES / 2) + (kk & 3) * 32;
                mma_f16_ts(tmem + t * C::TILE_COLS + C::PV_COL, tmem + t * C::TILE_COLS + C::P_COL + kk * 8,
                           sw128_kmajor_desc(va), idesc_pv, kk > 0);
            }
        };
        bool ok = __all_sync(0xffffffffu, mbar_wait(q_full, 0, err, AERR_Q)) &&
                  __all_sync(0xffffffffu, mbar_wait(&kv_full[0], 0, err, AERR_KV_FULL));
        if (ok) {
            tc_fence_after();
            if (elect_one()) {
                for (int t = 0; t < nq; ++t) {
                    mma_s(t, 0);
                    mma_commit(&ready[t]);
                }
            }
            __syncwarp();
        }
        for (int j = 0; j < ntiles && ok; ++j) {
            const bool more = j + 1 < ntiles;
            if (more && !__all_sync(0xffffffffu,
                                    mbar_wait(&kv_full[(j + 1) % C::STAGES], ((j + 1) / C::STAGES) & 1, err, AERR_KV_FULL))) {
                ok = false;
                break;
            }
            for (int t = 0; t < nq && ok; ++t) {
                // softmax t is done with S_t(j), PV_t(j-1) and has written P_t(j)
                if (!__all_sync(0xffffffffu, mbar_wait(&pdone[t], j & 1, err, AERR_P_FULL))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (elect_one()) {
                    mma_pv(t, j);
                    if (more) mma_s(t, j + 1);
                    mma_commit(&ready[t]);
                }
                __syncwarp();
            }
            if (!ok) break;
            if (elect_one()) mma_commit(&kv_empty[j % C::STAGES]);  // every reader of stage j has been issued
            __syncwarp();
        }
    } else if ((warp & 3) != 1) {
        // ---- softmax: each query row split over two threads (halves h = 0, 1 take keys 64 h .. 64 h + 63
        // of every key tile and output dimensions 32 h .. 32 h + 31), in two warps of one sub-partition
        // that exchange the row max per tile (and the row sum at the end) through shared memory ----
        const int t = (warp >> 2) & 1;
        const int half = warp >> 3;
        const int quarter = warp & 3;                             // 0, 2 or 3
        const int row = (quarter == 0 ? 0 : (quarter - 1) * 32) + lane;  // query q0 + 96 t + row
        const uint32_t base = tmem + t * C::TILE_COLS + (static_cast<uint32_t>(quarter * 32) << 16);
        const uint32_t bar_id = 1 + t * 4 + quarter;  // named barrier of the two halves (64 threads)
        float *xf = reinterpret_cast<float *>(smem + C::XCH_OFF);
        int *xok = reinterpret_cast<int *>(smem + C::XCH_OFF + C::XCH_BYTES);
        // exchange slot: [parity][t][quarter][half][lane]; parity alternates so a slot is rewritten only
        // after the partner passed the next barrier (and so finished reading it)
        auto slot = [&](int parity, int h) { return (((parity * 2 + t) * 4 + quarter) * 2 + h) * 32 + lane; };
        // both halves reach every exchange, failed waits included, and take the same decision after it
        auto exchange = [&](int parity, float v, bool ok_in, float &partner, bool &ok_both) {
            xf[slot(parity, half)] = v;
            xok[slot(parity, half)] = ok_in ? 1 : 0;
            asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(64) : "memory");
            partner = xf[slot(parity, half ^ 1)];
            ok_both = ok_in && xok[slot(parity, half ^ 1)] != 0;
        };
        if (t < nq) {
            float o[C::HD / 2];
#pragma unroll
            for (int i = 0; i < C::HD / 2; ++i) o[i] = 0.f;
            float m_run = -INFINITY, l_run = 0.f, alpha_prev = 0.f;
            bool ok = true;
            // O = O alpha + PV (this half's 32 output dimensions; PV_t(j-1) was formed against the running
            // max of step j-1); the caller has waited for ready[t] phase j
            auto fold_pv = [&](float alpha) {
                uint32_t pv[32];
                tmem_ld_32x32b_x32(base + C::PV_COL + 32 * half, pv);
                tmem_wait_ld();
#pragma unroll
                for (int d = 0; d < C::HD / 2; ++d) o[d] = fmaf(o[d], alpha, __uint_as_float(pv[d]));
            };
            for (int j = 0; j < ntiles; ++j) {
                const bool wok = __all_sync(0xffffffffu, mbar_wait(&ready[t], j & 1, err, AERR_S_FULL));
                const int nvalid = N - j * C::BKV - 64 * half;  // keys of this half-tile below N
                uint32_t s0[32];
                float mx = -INFINITY;
                if (wok) {
                    tc_fence_after();
                    uint32_t s1[32];
                    tmem_ld_32x32b_x32(base + C::S_COL + 64 * half, s0);
                    tmem_ld_32x32b_x32(base + C::S_COL + 64 * half + 32, s1);
                    tmem_wait_ld();
                    // row max of the raw scores (c > 0, so the max commutes with the scaling); the second
                    // 32 scores are read again for the exponentials (registers: the output row stays in them)
                    if (nvalid >= 64) {
                        mx = chunk_max<false>(s0, mx, 32);
                        mx = chunk_max<false>(s1, mx, 32);
                    } else {
                        mx = chunk_max<true>(s0, mx, nvalid);
                        mx = chunk_max<true>(s1, mx, nvalid - 32);
                    }
                }
                float mx_other;
                bool both;
                exchange(j & 1, mx, wok, mx_other, both);
                if (!both) {
                    ok = false;
                    break;
                }
                const float m_new = fmaxf(m_run, fmaxf(mx, mx_other) * c_log2);
                const float alpha = ex2_approx(m_run - m_new);
                // P = 2^(s c - m) of this half's 64 keys into tensor memory (PV_t(j-1), complete with
                // S_t(j), has read P_t(j-1)), row sum
                uint32_t pk[16];
                float rsum = nvalid >= 64 ? chunk_exp<false>(s0, c_log2, -m_new, pk, 32)
                                          : chunk_exp<true>(s0, c_log2, -m_new, pk, nvalid);
                tmem_st_32x32b_x16(base + C::P_COL + 32 * half, pk);
                tmem_ld_32x32b_x32(base + C::S_COL + 64 * half + 32, s0);
                tmem_wait_ld();
                rsum += nvalid >= 64 ? chunk_exp<false>(s0, c_log2, -m_new, pk, 32)
                                     : chunk_exp<true>(s0, c_log2, -m_new, pk, nvalid - 32);
                tmem_st_32x32b_x16(base + C::P_COL + 32 * half + 16, pk);
                // fold PV_t(j-1) before pdone lets PV_t(j) overwrite it (after the scores: fewer live registers)
                if (j > 0) fold_pv(alpha_prev);
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&pdone[t]);
                l_run = fmaf(l_run, alpha, rsum);
                m_run = m_new;
                alpha_prev = alpha;
            }
            if (ok) {
                const bool wok = __all_sync(0xffffffffu, mbar_wait(&ready[t], ntiles & 1, err, AERR_PV_FULL));
                if (wok) {
                    tc_fence_after();
                    fold_pv(alpha_prev);
                }
                float l_other;
                bool both;
                exchange(ntiles & 1, l_run, wok, l_other, both);
                const int n = q0 + t * C::ROWS + row;
                if (both && n < N) {
                    const int bb = bh / heads, h = bh % heads;
                    const float inv = 1.0f / (half == 0 ? l_run + l_other : l_other + l_run);
                    const int64_t r = static_cast<int64_t>(bb) * N + n;  // output row
                    const int hb = 32 * half;                             // this half's 32-wide Q8_0 block
#pragma unroll
                    for (int d = 0; d < C::HD / 2; ++d) o[d] = o[d] * inv;
                    const int E = heads * C::HD;
                    if (o16 || qcodes) {
                        float amax = 0.f;
#pragma unroll
                        for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(o[i]));
                        const float dq = __fdiv_rn(amax, 127.f);
                        const float id = amax != 0.f ? __fdiv_rn(127.f, amax) : 0.f;
                        if (o16) {  // Q8_0 of the block, written dequantised as fp16
                            const float dh = __half2float(__float2half_rn(dq));
                            uint4 *dst = reinterpret_cast<uint4 *>(o16 + r * E + h * C::HD + hb);
#pragma unroll
                            for (int i = 0; i < 32; i += 8) {
                                uint32_t hw[4];
#pragma unroll
                                for (int e = 0; e < 4; ++e) {
                                    const float a0 = q8_code_f(__fmul_rn(o[i + 2 * e], id));
                                    const float a1 = q8_code_f(__fmul_rn(o[i + 2 * e + 1], id));
                                    const __half2 h2 = __floats2half2_rn(__fmul_rn(a0, dh), __fmul_rn(a1, dh));
                                    hw[e] = *reinterpret_cast<const uint32_t *>(&h2);
                                }
                                dst[i >> 3] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                            }
                        } else {
                            uint32_t pk8[8];
#pragma unroll
                            for (int i = 0; i < 8; ++i) {
                                const int a0 = __float2int_rn(__fmul_rn(o[4 * i], id));
                                const int a1 = __float2int_rn(__fmul_rn(o[4 * i + 1], id));
                                const int a2 = __float2int_rn(__fmul_rn(o[4 * i + 2], id));
                                const int a3 = __float2int_rn(__fmul_rn(o[4 * i + 3], id));
                                pk8[i] = (static_cast<uint32_t>(a0) & 0xFFu) | ((static_cast<uint32_t>(a1) & 0xFFu) << 8) |
                                         ((static_cast<uint32_t>(a2) & 0xFFu) << 16) | ((static_cast<uint32_t>(a3) & 0xFFu) << 24);
                            }
                            uint4 *dst = reinterpret_cast<uint4 *>(qcodes + r * E + h * C::HD + hb);
                            dst[0] = make_uint4(pk8[0], pk8[1], pk8[2], pk8[3]);
                            dst[1] = make_uint4(pk8[4], pk8[5], pk8[6], pk8[7]);
                            store_act_scale(qquads, (h * C::HD + hb) >> 5, static_cast<int>(r), qld, E >> 5, dq);
                        }
                    } else {
                        float *dst = out + r * E + h * C::HD + hb;
#pragma unroll
                        for (int d = 0; d < 32; d += 4)
                            *reinterpret_cast<float4 *>(dst + d) = make_float4(o[d], o[d + 1], o[d + 2], o[d + 3]);
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, 512);
}

cudaError_t flash_attention(const void *q, const void *k, const void *vt, int B, int N, int heads, float scale,
                            const AttnOut &o, int *err, cudaStream_t s) {
    using C = AttnCfg;
    if (B <= 0 || N <= 0 || heads <= 0 || N % 8 != 0 || !err || (!o.f32 && !o.codes && !o.dq16) ||
        (o.codes && (!o.quads || o.ld < B * N)) || (reinterpret_cast<uintptr_t>(o.dq16) & 15))
        return cudaErrorInvalidValue;
    const uint64_t bhn = static_cast<uint64_t>(B) * heads;
    CUtensorMap tq, tk, tv;
    const uint64_t dqk[3] = {64, static_cast<uint64_t>(N), bhn};
    const uint64_t sqk[2] = {64 * 2, static_cast<uint64_t>(N) * 64 * 2};
    const uint32_t bq[3] = {64, 32, 1};
    const uint32_t bqk[3] = {64, 128, 1};
    const uint64_t dv[3] = {static_cast<uint64_t>(N), 64, bhn};
    const uint64_t sv[2] = {static_cast<uint64_t>(N) * 2, static_cast<uint64_t>(N) * 64 * 2};
    const uint32_t bv[3] = {64, 64, 1};
    if (!make_tmap(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, q, 3, dqk, sqk, bq, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_tmap(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, k, 3, dqk, sqk, bqk, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_tmap(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, vt, 3, dv, sv, bv, CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(flash_attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    dim3 grid((N + C::QT * C::ROWS - 1) / (C::QT * C::ROWS), static_cast<unsigned>(bhn));
    flash_attn_tc_kernel<<<grid, C::THREADS, C::SMEM_BYTES, s>>>(
        tq, tk, tv, N, heads, scale * 1.4426950408889634f, o.f32, static_cast<int8_t *>(o.codes),
        static_cast<__half *>(o.quads), o.ld, static_cast<__half *>(o.dq16), err);
    return cudaGetLastError();
}

}  // namespace b200
