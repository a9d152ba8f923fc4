// attn_tc256.cu -- single-head attention of width 256 on the 5th-generation
// tensor cores: the tracker's memory attention (sam3_build_mem_attn_graph,
// sam3.cpp:9228-9341: one head of d_model 256, 4096 current-frame queries
// against themselves and against up to 7 x 4096 memory tokens + 64 object-
// pointer tokens).  out = softmax(q k^T * scale) v with q, k, v rounded to fp16
// (the accuracy of the mma.sync path it replaces), fp32 accumulation.
//
// One CTA owns 128 queries and one contiguous range of keys (split-KV: the
// partial accumulators and (max, sum) of each range go through the same
// combine pass as attention_mma_f16kv_split).  Keys stream in tiles of 64.
//   warp 4     : TMA producer -- the Q tile once (four 64-column SW128
//                chunks), then K tiles (four chunks) and V^T tiles (one
//                256-row chunk) through two separate 2-deep rings, so a K
//                stage frees as soon as its S MMAs complete;
//   warp 5     : TMEM allocator + MMA issuer -- S(j) = Q K_j^T (M = 128,
//                N = 64, K = 256: 16 MMAs) into one of two S buffers, and
//                PV(j): O += P(j) V_j (A = P read from tensor memory, N = 256,
//                K = 64: 4 MMAs) once softmax has written P(j); S(j + 2) is
//                issued right after PV(j), so the tensor core computes
//                PV(j) and S(j + 2) while softmax works on S(j + 1);
//   warps 0-3  : softmax, one query row per thread (warp w reads TMEM lane
//                quarter w).  The row max m is kept in log2 units; P(j) =
//                2^(s c - m) goes to tensor memory as fp16.  O stays in
//                tensor memory: it is rescaled (ld, multiply, st) only when a
//                row's max grows by more than 2^8 (then after PV(j - 1) has
//                completed), otherwise P is formed against the stale max and
//                stays below 2^8 -- the lazy rescaling of FlashAttention-4.
// Tensor memory (512 columns): O 0..255, S buffers 256..383, P buffers 384..447.
#include "attn_mma.cuh"
#include "attn_tc256.cuh"
#include "ptx.cuh"
#include "tmap.h"

#include <cstdint>
#include <cuda_fp16.h>

namespace b200 {
namespace {

struct T256 {
    static constexpr int BQ = 128, BK = 64, D = 256, STAGES = 2;
    static constexpr int Q_CHUNK = BQ * 128;  // 128 rows x 64 fp16 (128 B), SW128
    static constexpr int Q_BYTES = 4 * Q_CHUNK;
    static constexpr int K_CHUNK = BK * 128;  // 64 keys x 64 fp16
    static constexpr int K_BYTES = 4 * K_CHUNK;
    static constexpr int V_BYTES = D * 128;   // V^T: 256 rows (d) x 64 keys
    static constexpr int K_OFF = Q_BYTES;
    static constexpr int V_OFF = K_OFF + STAGES * K_BYTES;
    static constexpr int BAR_OFF = V_OFF + STAGES * V_BYTES;  // 192 KB
    static constexpr int SMEM_BYTES = BAR_OFF + 256 + 1024;
    static constexpr int THREADS = 192;
    static constexpr uint32_t O_COL = 0, S_COL = 256, P_COL = 384;
    static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

constexpr float RESCALE_LOG2 = 8.0f;

enum : int {
    TERR_Q = 1 << 16,
    TERR_K_EMPTY = 1 << 17,
    TERR_K_FULL = 1 << 18,
    TERR_V_EMPTY = 1 << 19,
    TERR_V_FULL = 1 << 20,
    TERR_S_FULL = 1 << 21,
    TERR_P_FULL = 1 << 22,
    TERR_PV_DONE = 1 << 23,
};

__global__ void __launch_bounds__(T256::THREADS, 1)
    attn_tc256_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v, int NQ, int NK, int chunk, float c_log2,
                      float *__restrict__ part_o, float2 *__restrict__ part_ml, int *__restrict__ err) {
    using C = T256;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *q_full = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
    uint64_t *k_full = q_full + 1, *k_empty = k_full + 2, *v_full = k_empty + 2, *v_empty = v_full + 2;
    uint64_t *s_full = v_empty + 2, *p_full = s_full + 2, *pv_done = p_full + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(pv_done + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q0 = blockIdx.x * C::BQ, z = blockIdx.y;
    const int k0 = z * chunk, k1 = min(NK, k0 + chunk);
    const int nt = k1 > k0 ? (k1 - k0 + C::BK - 1) / C::BK : 0;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&k_full[b], 1);
            mbar_init(&k_empty[b], 1);
            mbar_init(&v_full[b], 1);
            mbar_init(&v_empty[b], 1);
            mbar_init(&s_full[b], 1);
            mbar_init(&p_full[b], 4);
            mbar_init(&pv_done[b], 1);
        }
        fence_mbar_init();
        prefetch_tmap(&tm_q);
        prefetch_tmap(&tm_k);
        prefetch_tmap(&tm_v);
    }
    if (warp == 5) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 4) {
        // ---- TMA producer ----
        if (nt > 0) {
            if (elect_one()) {
                mbar_arrive_expect_tx(q_full, C::Q_BYTES);
                for (int c = 0; c < 4; ++c) tma_load_2d(smem + c * C::Q_CHUNK, &tm_q, q_full, c * 64, q0);
            }
            __syncwarp();
        }
        for (int j = 0; j < nt; ++j) {
            const int b = j & 1;
            const uint32_t ph = ((j >> 1) & 1) ^ 1;
            if (!__all_sync(0xffffffffu, mbar_wait(&k_empty[b], ph, err, TERR_K_EMPTY))) break;
            if (elect_one()) {
                uint8_t *kb = smem + C::K_OFF + b * C::K_BYTES;
                mbar_arrive_expect_tx(&k_full[b], C::K_BYTES);
                for (int c = 0; c < 4; ++c) tma_load_2d(kb + c * C::K_CHUNK, &tm_k, &k_full[b], c * 64, k0 + j * C::BK);
            }
            __syncwarp();
            if (!__all_sync(0xffffffffu, mbar_wait(&v_empty[b], ph, err, TERR_V_EMPTY))) break;
            if (elect_one()) {
                mbar_arrive_expect_tx(&v_full[b], C::V_BYTES);
                tma_load_2d(smem + C::V_OFF + b * C::V_BYTES, &tm_v, &v_full[b], k0 + j * C::BK, 0);
            }
            __syncwarp();
        }
    } else if (warp == 5) {
        // ---- MMA issuer ----
        constexpr uint32_t idesc_s = idesc_f16_f32(128, C::BK);
        constexpr uint32_t idesc_pv = idesc_f16_f32(128, C::D);
        const uint32_t q_addr = smem_u32(smem);
        bool ok = nt > 0 && __all_sync(0xffffffffu, mbar_wait(q_full, 0, err, TERR_Q));
        // S(j) into S buffer j & 1; frees K stage j & 1 on completion
        auto issue_s = [&](int j) -> bool {
            const int b = j & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(&k_full[b], (j >> 1) & 1, err, TERR_K_FULL))) return false;
            tc_fence_after();
            if (elect_one()) {
                const uint32_t k_addr = smem_u32(smem + C::K_OFF + b * C::K_BYTES);
#pragma unroll
                for (int kk = 0; kk < C::D / 16; ++kk) {
                    const uint32_t off = (kk & 3) * 32u;  // 16-element K slice inside the 128-byte row
                    mma_f16(tmem + C::S_COL + b * C::BK, sw128_kmajor_desc(q_addr + (kk >> 2) * C::Q_CHUNK + off),
                            sw128_kmajor_desc(k_addr + (kk >> 2) * C::K_CHUNK + off), idesc_s, kk > 0);
                }
                mma_commit(&s_full[b]);
                mma_commit(&k_empty[b]);
            }
            __syncwarp();
            return true;
        };
        if (ok) ok = issue_s(0);
        if (ok && nt > 1) ok = issue_s(1);
        for (int j = 0; j < nt && ok; ++j) {
            const int b = j & 1;
            const uint32_t ph = (j >> 1) & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(&p_full[b], ph, err, TERR_P_FULL)) ||
                !__all_sync(0xffffffffu, mbar_wait(&v_full[b], ph, err, TERR_V_FULL))) {
                ok = false;
                break;
            }
            tc_fence_after();
            if (elect_one()) {
                const uint32_t v_addr = smem_u32(smem + C::V_OFF + b * C::V_BYTES);
#pragma unroll
                for (int kk = 0; kk < C::BK / 16; ++kk)
                    mma_f16_ts(tmem + C::O_COL, tmem + C::P_COL + b * 32 + kk * 8, sw128_kmajor_desc(v_addr + kk * 32),
                               idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
                mma_commit(&pv_done[b]);
                mma_commit(&v_empty[b]);
            }
            __syncwarp();
            if (j + 2 < nt) ok = issue_s(j + 2);
        }
    } else {
        // ---- softmax: query row q0 + 32 warp + lane ----
        const uint32_t lanes = static_cast<uint32_t>(warp * 32) << 16;
        const int row = q0 + warp * 32 + lane;
        float m_run = -INFINITY, l_run = 0.f;
        bool ok = true;
        for (int j = 0; j < nt; ++j) {
            const int b = j & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(&s_full[b], (j >> 1) & 1, err, TERR_S_FULL))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const int nvalid = min(C::BK, k1 - (k0 + j * C::BK));
            uint32_t s0[32], s1[32];
            tmem_ld_32x32b_x32(tmem + lanes + C::S_COL + b * C::BK, s0);
            tmem_ld_32x32b_x32(tmem + lanes + C::S_COL + b * C::BK + 32, s1);
            tmem_wait_ld();
            float mx = -INFINITY;
            if (nvalid >= C::BK) {
#pragma unroll
                for (int i = 0; i < 32; ++i) mx = fmaxf(mx, fmaxf(__uint_as_float(s0[i]), __uint_as_float(s1[i])));
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    if (i < nvalid) mx = fmaxf(mx, __uint_as_float(s0[i]));
                    if (i + 32 < nvalid) mx = fmaxf(mx, __uint_as_float(s1[i]));
                }
            }
            const float m_cand = fmaxf(m_run, mx * c_log2);
            // a row whose max grew by more than 2^8 takes the new max, its O and sum rescaled
            const bool grow = j == 0 || m_cand > m_run + RESCALE_LOG2;
            float alpha = 1.0f;
            if (j > 0 && __any_sync(0xffffffffu, grow)) {
                if (!__all_sync(0xffffffffu, mbar_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, err, TERR_PV_DONE))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                alpha = grow ? ex2_approx(m_run - m_cand) : 1.0f;
#pragma unroll 1
                for (int c = 0; c < C::D; c += 32) {
                    uint32_t o[32];
                    tmem_ld_32x32b_x32(tmem + lanes + C::O_COL + c, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                    tmem_st_32x32b_x32(tmem + lanes + C::O_COL + c, o);
                }
                tmem_wait_st();
            }
            const float m_use = grow ? m_cand : m_run;
            // P buffer b was read by PV(j - 2)
            if (j >= 2 &&
                !__all_sync(0xffffffffu, mbar_wait(&pv_done[b], ((j - 2) >> 1) & 1, err, TERR_PV_DONE))) {
                ok = false;
                break;
            }
            float rsum = 0.f;
            uint32_t pk[16];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint32_t(&sv)[32] = h ? s1 : s0;
#pragma unroll
                for (int i = 0; i < 32; i += 2) {
                    float p0 = ex2_approx(fmaf(__uint_as_float(sv[i]), c_log2, -m_use));
                    float p1 = ex2_approx(fmaf(__uint_as_float(sv[i + 1]), c_log2, -m_use));
                    if (h * 32 + i >= nvalid) p0 = 0.f;
                    if (h * 32 + i + 1 >= nvalid) p1 = 0.f;
                    const __half2 hp = __floats2half2_rn(p0, p1);
                    // the row sum of the probabilities the PV MMA multiplies (their fp16 values)
                    rsum += __low2float(hp) + __high2float(hp);
                    pk[i >> 1] = *reinterpret_cast<const uint32_t *>(&hp);
                }
                tmem_st_32x32b_x16(tmem + lanes + C::P_COL + b * 32 + h * 16, pk);
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[b]);
            l_run = fmaf(l_run, alpha, rsum);
            m_run = m_use;
        }
        // the partial result of this key range: unnormalised O, (max, sum)
        const int64_t base = static_cast<int64_t>(z) * NQ;
        if (ok && nt > 0 &&
            __all_sync(0xffffffffu, mbar_wait(&pv_done[(nt - 1) & 1], ((nt - 1) >> 1) & 1, err, TERR_PV_DONE))) {
            tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < C::D; c += 32) {
                uint32_t o[32];
                tmem_ld_32x32b_x32(tmem + lanes + C::O_COL + c, o);
                tmem_wait_ld();
                if (row < NQ) {
                    float4 *dst = reinterpret_cast<float4 *>(part_o + (base + row) * C::D + c);
#pragma unroll
                    for (int i = 0; i < 32; i += 4)
                        dst[i / 4] = make_float4(__uint_as_float(o[i]), __uint_as_float(o[i + 1]),
                                                 __uint_as_float(o[i + 2]), __uint_as_float(o[i + 3]));
                }
            }
            if (row < NQ) part_ml[base + row] = make_float2(m_run, l_run);
        } else if (nt == 0 && row < NQ) {
            part_ml[base + row] = make_float2(-INFINITY, 0.f);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 5) tmem_dealloc(tmem, 512);
}

// v [NK][256] f32 -> v^T fp16 [256][ldt] (keys contiguous), 32 x 32 tiles through shared memory
__global__ void v_to_half_t_kernel(const float *__restrict__ v, int NK, int ld_v, __half *__restrict__ vt, int ldt) {
    __shared__ float tile[32][33];
    const int k0 = blockIdx.x * 32, d0 = blockIdx.y * 32;
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const int k = k0 + r;
        tile[r][threadIdx.x] = k < NK ? v[static_cast<int64_t>(k) * ld_v + d0 + threadIdx.x] : 0.f;
    }
    __syncthreads();
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const int k = k0 + threadIdx.x;
        if (k < ldt) vt[static_cast<int64_t>(d0 + r) * ldt + k] = __float2half_rn(tile[threadIdx.x][r]);
    }
}

}  // namespace

int attention_tc256_splits(int NQ, int NK, int num_sms) {
    const int qtiles = (NQ + T256::BQ - 1) / T256::BQ;
    const int tiles = (NK + T256::BK - 1) / T256::BK;
    int splits = qtiles > 0 ? num_sms / qtiles : 1;
    splits = splits < 1 ? 1 : splits;
    const int most = tiles / 2 > 0 ? tiles / 2 : 1;  // at least two key tiles per CTA
    return splits < most ? splits : most;
}

cudaError_t v_to_half_transposed(const float *v, int NK, int ld_v, __half *vt, int ldt, cudaStream_t s) {
    if (NK <= 0 || ldt < NK || ldt % 8 != 0) return cudaErrorInvalidValue;
    dim3 grid(static_cast<unsigned>((ldt + 31) / 32), 256 / 32);
    v_to_half_t_kernel<<<grid, dim3(32, 8), 0, s>>>(v, NK, ld_v, vt, ldt);
    return cudaGetLastError();
}

cudaError_t attention_tc256(const __half *q, int NQ, const __half *k, int NK, const __half *vt, int ldt, float scale,
                            int splits, float *part_o, float2 *part_ml, float *o, int *err, cudaStream_t s) {
    using C = T256;
    if (NQ <= 0 || NK <= 0 || ldt < NK || ldt % 8 != 0 || splits < 1 || !part_o || !part_ml || !o || !err)
        return cudaErrorInvalidValue;
    // key ranges of whole 64-key tiles: every V^T load starts on a 16-byte boundary
    int chunk = (NK + splits - 1) / splits;
    chunk = (chunk + C::BK - 1) / C::BK * C::BK;
    const int nz = (NK + chunk - 1) / chunk;
    CUtensorMap tq, tk, tv;
    const uint64_t dq[2] = {256, static_cast<uint64_t>(NQ)}, dk[2] = {256, static_cast<uint64_t>(NK)};
    const uint64_t dv[2] = {static_cast<uint64_t>(NK), 256};
    const uint64_t sqk[1] = {256 * 2}, sv[1] = {static_cast<uint64_t>(ldt) * 2};
    const uint32_t bq[2] = {64, C::BQ}, bk[2] = {64, C::BK}, bv[2] = {C::BK, 256};
    if (!make_tmap(&tq, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, q, 2, dq, sqk, bq, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_tmap(&tk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, k, 2, dk, sqk, bk, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_tmap(&tv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, vt, 2, dv, sv, bv, CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(attn_tc256_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    dim3 grid(static_cast<unsigned>((NQ + C::BQ - 1) / C::BQ), static_cast<unsigned>(nz));
    attn_tc256_kernel<<<grid, C::THREADS, C::SMEM_BYTES, s>>>(tq, tk, tv, NQ, NK, chunk, scale * 1.4426950408889634f,
                                                              part_o, part_ml, err);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    return attention_combine(256, part_o, part_ml, nz, NQ, 1, 1, o, AttnStrides{0, 0, 256}, s);
}

}  // namespace b200
