// attn_tcw.cu -- windowed and global attention of the Hiera blocks on the
// 5th-generation tensor cores (sam2_hiera_block_forward, sam3.cpp:4299-4461:
// per window and head softmax(q k^T * scale) v; windows of 16-196 tokens,
// Q-pooled blocks with a quarter of the queries, global blocks of 1024-4096
// tokens; head dimension 56 / 72 / 96 padded to 64 or 128).
//
// A CTA owns one 128-row query tile.  Windows whose queries and keys both fit
// a 128-row tile are packed: P = min(128 / NQ, 128 / Ns) whole windows share
// the query tile and one 128-key tile, and row r (window r / NQ of the group)
// sees only its window's keys (a block-diagonal mask, so the tensor core's
// work per window is that of a 128 x 128 tile divided by P).  Longer windows
// and global blocks take one window per CTA and stream its keys in 128-key
// tiles, FlashAttention style.
//   warp 4    : TMA producer -- the Q tile (Dp / 64 128-byte-swizzled
//               chunks), then K and V^T tiles through two 2-deep rings;
//   warp 5    : TMEM allocator + MMA issuer -- S(j) = Q K_j^T (M = 128,
//               N = 128, K = Dp) into one of two S buffers, PV(j): O +=
//               P(j) V_j with P read from tensor memory (N = Dp, K = 128);
//               S(j + 2) issued right after PV(j);
//   warps 0-3 : softmax, one query row per thread (warp w reads TMEM lane
//               quarter w): row max in log2 units over the row's valid keys,
//               P = 2^(s c - m) as fp16 into tensor memory, the row sum over
//               the fp16 values the PV MMA multiplies; O rescaled in tensor
//               memory only when a row's max grows by more than 2^8
//               (FlashAttention-4's lazy rescaling); at the end O / l to the
//               f32 output rows.
// Tensor memory (512 columns): O 0..Dp-1, S buffers 128..383, P buffers 384..511.
#include "attn_tcw.cuh"
#include "ptx.cuh"
#include "tmap.h"

#include <cstdint>

namespace b200 {
namespace {

template <int DP, bool PACK>
struct TW {
    static constexpr int BQ = 128, BK = 128, D = DP, CH = DP / 64;  // 64-element (128-byte) SW128 chunks
    static constexpr int Q_CHUNK = BQ * 128;                       // 128 rows x 64 fp16
    static constexpr int Q_BYTES = CH * Q_CHUNK;
    static constexpr int K_CHUNK = BK * 128;                       // 128 keys x 64 fp16
    static constexpr int K_BYTES = CH * K_CHUNK;
    static constexpr int V_CHUNK = D * 128;                        // V^T: D rows x 64 keys
    static constexpr int V_BYTES = 2 * V_CHUNK;                    // one 128-key tile
    static constexpr int K_OFF = Q_BYTES;
    static constexpr int V_OFF = K_OFF + 2 * K_BYTES;
    static constexpr int BAR_OFF = V_OFF + 2 * V_BYTES;
    static constexpr int SMEM_BYTES = BAR_OFF + 256 + 1024;
    static constexpr int THREADS = 192;
    // Tensor memory: packed windows (one key tile) at head dimension 64 need O 64 + S 128 + P 64 = 256
    // columns, so two CTAs share an SM (one's TMA and setup under the other's MMAs and softmax);
    // otherwise O 0..Dp-1, two S buffers 128..383, two P buffers 384..511.
    static constexpr bool HALF_TMEM = PACK && DP == 64;
    static constexpr uint32_t TCOLS = HALF_TMEM ? 256 : 512;
    static constexpr uint32_t O_COL = 0, S_COL = HALF_TMEM ? 64 : 128, P_COL = HALF_TMEM ? 192 : 384;
    static constexpr int CTAS = HALF_TMEM ? 2 : 1;
    static_assert(DP == 64 || DP == 128, "head dimension padded to 64 or 128");
    static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

constexpr float TW_RESCALE_LOG2 = 8.0f;

enum : int {
    WERR_Q = 1 << 6,
    WERR_K_EMPTY = 1 << 7,
    WERR_K_FULL = 1 << 25,
    WERR_V_EMPTY = 1 << 26,
    WERR_V_FULL = 1 << 27,
    WERR_S_FULL = 1 << 28,
    WERR_P_FULL = 1 << 29,
    WERR_PV_DONE = 1 << 30,
};

// grid (query tiles per window, window groups, heads).  PACK (P > 0): P
// packed windows per group, one query tile and one key tile; otherwise (P = 0)
// one window per group, nt key tiles.
template <int DP, bool PACK>
__global__ void __launch_bounds__(TW<DP, PACK>::THREADS, TW<DP, PACK>::CTAS)
    attn_tcw_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, int Bw, int NQ, int N, int Ns, int hd, int P, int nt,
                    float c_log2, float *__restrict__ out, int64_t o_ld, int *__restrict__ err) {
    using C = TW<DP, PACK>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *q_full = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
    uint64_t *k_full = q_full + 1, *k_empty = k_full + 2, *v_full = k_empty + 2, *v_empty = v_full + 2;
    uint64_t *s_full = v_empty + 2, *p_full = s_full + 2, *pv_done = p_full + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(pv_done + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qt = blockIdx.x, g = blockIdx.y, h = blockIdx.z;
    // first query row and first key (within the head) of this CTA
    const int q_in_head = P ? g * P * NQ : g * NQ + qt * C::BQ;
    const int k_in_head = P ? g * P * Ns : g * Ns;

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
        tmem_alloc(tmem_slot, C::TCOLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 4) {
        // ---- TMA producer ----
        const int q_row = h * Bw * NQ + q_in_head, k_row = h * Bw * Ns + k_in_head;
        if (elect_one()) {
            mbar_arrive_expect_tx(q_full, C::Q_BYTES);
            for (int c = 0; c < C::CH; ++c) tma_load_2d(smem + c * C::Q_CHUNK, &tm_q, q_full, c * 64, q_row);
        }
        __syncwarp();
        for (int j = 0; j < nt; ++j) {
            const int b = j & 1;
            const uint32_t ph = ((j >> 1) & 1) ^ 1;
            if (!__all_sync(0xffffffffu, mbar_wait(&k_empty[b], ph, err, WERR_K_EMPTY))) break;
            if (elect_one()) {
                uint8_t *kb = smem + C::K_OFF + b * C::K_BYTES;
                mbar_arrive_expect_tx(&k_full[b], C::K_BYTES);
                for (int c = 0; c < C::CH; ++c)
                    tma_load_2d(kb + c * C::K_CHUNK, &tm_k, &k_full[b], c * 64, k_row + j * C::BK);
            }
            __syncwarp();
            if (!__all_sync(0xffffffffu, mbar_wait(&v_empty[b], ph, err, WERR_V_EMPTY))) break;
            if (elect_one()) {
                uint8_t *vb = smem + C::V_OFF + b * C::V_BYTES;
                mbar_arrive_expect_tx(&v_full[b], C::V_BYTES);
                for (int c = 0; c < 2; ++c)  // keys (x, 16-byte aligned: Ns % 8 == 0) x head rows (y)
                    tma_load_2d(vb + c * C::V_CHUNK, &tm_v, &v_full[b], k_in_head + j * C::BK + c * 64, h * C::D);
            }
            __syncwarp();
        }
    } else if (warp == 5) {
        // ---- MMA issuer ----
        constexpr uint32_t idesc_s = idesc_f16_f32(128, C::BK);
        constexpr uint32_t idesc_pv = idesc_f16_f32(128, C::D);
        const uint32_t q_addr = smem_u32(smem);
        bool ok = __all_sync(0xffffffffu, mbar_wait(q_full, 0, err, WERR_Q));
        auto issue_s = [&](int j) -> bool {
            const int b = j & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(&k_full[b], (j >> 1) & 1, err, WERR_K_FULL))) return false;
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
            if (!__all_sync(0xffffffffu, mbar_wait(&p_full[b], ph, err, WERR_P_FULL)) ||
                !__all_sync(0xffffffffu, mbar_wait(&v_full[b], ph, err, WERR_V_FULL))) {
                ok = false;
                break;
            }
            tc_fence_after();
            if (elect_one()) {
                const uint32_t v_addr = smem_u32(smem + C::V_OFF + b * C::V_BYTES);
#pragma unroll
                for (int kk = 0; kk < C::BK / 16; ++kk)
                    mma_f16_ts(tmem + C::O_COL, tmem + C::P_COL + b * 64 + kk * 8,
                               sw128_kmajor_desc(v_addr + (kk >> 2) * C::V_CHUNK + (kk & 3) * 32), idesc_pv,
                               (j > 0 || kk > 0) ? 1u : 0u);
                mma_commit(&pv_done[b]);
                mma_commit(&v_empty[b]);
            }
            __syncwarp();
            if (j + 2 < nt) ok = issue_s(j + 2);
        }
    } else {
        // ---- softmax: tile row r ----
        const uint32_t lanes = static_cast<uint32_t>(warp * 32) << 16;
        const int r = warp * 32 + lane;
        // the row's output row and its valid keys [klo, khi) relative to k_in_head
        int orow, klo, khi;
        bool rvalid;
        if (P) {
            const int wl = r / NQ, qi = r - wl * NQ, w = g * P + wl;
            rvalid = wl < P && w < Bw;
            orow = w * NQ + qi;
            klo = wl * Ns;
            khi = klo + N;
        } else {
            const int qi = qt * C::BQ + r;
            rvalid = qi < NQ;
            orow = g * NQ + qi;
            klo = 0;
            khi = N;
        }
        if (!rvalid) khi = klo;
        float m_run = -INFINITY, l_run = 0.f;
        bool ok = true;
        for (int j = 0; j < nt; ++j) {
            const int b = j & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(&s_full[b], (j >> 1) & 1, err, WERR_S_FULL))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const int lo = klo - j * C::BK, hi = khi - j * C::BK;  // valid tile columns [lo, hi)
            const uint32_t sb = tmem + lanes + C::S_COL + b * C::BK;
            float mx = -INFINITY;
            // long sequences: the whole S row stays in registers (one TMEM pass), and tiles whose 128
            // keys are valid for every row of the warp skip the masks
            uint32_t sr[PACK ? 1 : C::BK];
            bool all_full = false;
            if constexpr (PACK) {
#pragma unroll 1
                for (int c = 0; c < C::BK; c += 32) {
                    uint32_t sv[32];
                    tmem_ld_32x32b_x32(sb + c, sv);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (c + i >= lo && c + i < hi) mx = fmaxf(mx, __uint_as_float(sv[i]));
                }
            } else {
#pragma unroll
                for (int c = 0; c < C::BK; c += 32)
                    tmem_ld_32x32b_x32(sb + c, *reinterpret_cast<uint32_t(*)[32]>(sr + c));
                tmem_wait_ld();
                all_full = __all_sync(0xffffffffu, lo <= 0 && hi >= C::BK);
                if (all_full) {
#pragma unroll
                    for (int i = 0; i < C::BK; ++i) mx = fmaxf(mx, __uint_as_float(sr[i]));
                } else {
#pragma unroll
                    for (int i = 0; i < C::BK; ++i)
                        if (i >= lo && i < hi) mx = fmaxf(mx, __uint_as_float(sr[i]));
                }
            }
            const float m_cand = fmaxf(m_run, mx * c_log2);
            // a row whose max grew by more than 2^8 takes the new max, its O and sum rescaled
            const bool grow = j == 0 || m_cand > m_run + TW_RESCALE_LOG2;
            float alpha = 1.0f;
            if (j > 0 && __any_sync(0xffffffffu, grow)) {
                if (!__all_sync(0xffffffffu,
                                mbar_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, err, WERR_PV_DONE))) {
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
                !__all_sync(0xffffffffu, mbar_wait(&pv_done[b], ((j - 2) >> 1) & 1, err, WERR_PV_DONE))) {
                ok = false;
                break;
            }
            float rsum = 0.f;
            // P = 2^(s c - m) as fp16 pairs, zero outside the row's keys; the row sum over the fp16
            // values the PV MMA multiplies
            auto probs = [&](const uint32_t *sv, int c, bool masked, uint32_t(&pk)[16]) {
#pragma unroll
                for (int i = 0; i < 32; i += 2) {
                    float p0 = ex2_approx(fmaf(__uint_as_float(sv[i]), c_log2, -m_use));
                    float p1 = ex2_approx(fmaf(__uint_as_float(sv[i + 1]), c_log2, -m_use));
                    if (masked) {
                        if (!(c + i >= lo && c + i < hi)) p0 = 0.f;
                        if (!(c + i + 1 >= lo && c + i + 1 < hi)) p1 = 0.f;
                    }
                    const __half2 hp = __floats2half2_rn(p0, p1);
                    rsum += __low2float(hp) + __high2float(hp);
                    pk[i >> 1] = *reinterpret_cast<const uint32_t *>(&hp);
                }
            };
            if constexpr (PACK) {
#pragma unroll 1
                for (int c = 0; c < C::BK; c += 32) {
                    uint32_t sv[32], pk[16];
                    tmem_ld_32x32b_x32(sb + c, sv);
                    tmem_wait_ld();
                    probs(sv, c, true, pk);
                    tmem_st_32x32b_x16(tmem + lanes + C::P_COL + b * 64 + (c >> 1), pk);
                }
            } else {
#pragma unroll
                for (int c = 0; c < C::BK; c += 32) {
                    uint32_t pk[16];
                    if (all_full) probs(sr + c, c, false, pk);
                    else probs(sr + c, c, true, pk);
                    tmem_st_32x32b_x16(tmem + lanes + C::P_COL + b * 64 + (c >> 1), pk);
                }
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[b]);
            l_run = fmaf(l_run, alpha, rsum);
            m_run = m_use;
        }
        if (ok && __all_sync(0xffffffffu,
                             mbar_wait(&pv_done[(nt - 1) & 1], ((nt - 1) >> 1) & 1, err, WERR_PV_DONE))) {
            tc_fence_after();
            const float inv = rvalid && l_run > 0.f ? 1.0f / l_run : 0.f;
            float *dst = out + static_cast<int64_t>(orow) * o_ld + static_cast<int64_t>(h) * hd;
#pragma unroll 1
            for (int c = 0; c < C::D; c += 32) {
                uint32_t o[32];
                tmem_ld_32x32b_x32(tmem + lanes + C::O_COL + c, o);
                tmem_wait_ld();
                if (rvalid) {
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (c + i < hd) dst[c + i] = __uint_as_float(o[i]) * inv;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 5) tmem_dealloc(tmem, C::TCOLS);
}

// q or k rows -> [heads][Bw * stride][Dp] fp16 (8 elements per thread)
__global__ void tcw_stage_rows_kernel(const float *__restrict__ src, int64_t ld, int rows, int stride, int Bw,
                                      int heads, int hd, int Dp, __half *__restrict__ dst) {
    const int per = Dp / 8;
    const int64_t total = static_cast<int64_t>(heads) * Bw * stride * per;
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= total) return;
    const int d0 = static_cast<int>(i % per) * 8;
    int64_t rest = i / per;
    const int r = static_cast<int>(rest % stride);
    rest /= stride;
    const int w = static_cast<int>(rest % Bw), h = static_cast<int>(rest / Bw);
    const float *s = src + (static_cast<int64_t>(w) * rows + r) * ld + static_cast<int64_t>(h) * hd;
    uint32_t pk[4];
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
        const float a = (r < rows && d0 + e < hd) ? s[d0 + e] : 0.f;
        const float b = (r < rows && d0 + e + 1 < hd) ? s[d0 + e + 1] : 0.f;
        const __half2 hv = __floats2half2_rn(a, b);
        pk[e >> 1] = *reinterpret_cast<const uint32_t *>(&hv);
    }
    *reinterpret_cast<uint4 *>(dst + i * 8) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
}

// v rows -> v^T [heads][Dp][Bw * Ns] fp16, 32 keys x 32 dims per CTA through shared memory
__global__ void tcw_stage_vt_kernel(const float *__restrict__ v, int64_t ld, int N, int Ns, int Bw, int hd, int Dp,
                                    __half *__restrict__ vt) {
    __shared__ float tile[32][33];
    const int nk = Bw * Ns;  // < 2^31 (checked by the host)
    const int key0 = blockIdx.x * 32;
    const int d0 = blockIdx.y * 32, h = blockIdx.z;
    const float *vh = v + static_cast<int64_t>(h) * hd;
    for (int rr = threadIdx.y; rr < 32; rr += blockDim.y) {
        const int key = key0 + rr;
        const int d = d0 + threadIdx.x;
        float val = 0.f;
        if (key < nk && d < hd) {
            const int w = key / Ns, r = key - w * Ns;
            if (r < N) val = vh[static_cast<int64_t>(w * N + r) * ld + d];
        }
        tile[rr][threadIdx.x] = val;
    }
    __syncthreads();
    __half *vrow = vt + (static_cast<int64_t>(h) * Dp + d0) * nk;
    for (int rr = threadIdx.y; rr < 32; rr += blockDim.y) {
        const int key = key0 + threadIdx.x;
        if (key < nk) vrow[static_cast<int64_t>(rr) * nk + key] = __float2half_rn(tile[threadIdx.x][rr]);
    }
}

template <int DP, bool PACK>
cudaError_t launch_tcw(const __half *qh, const __half *kh, const __half *vth, int Bw, int NQ, int N, int heads, int hd,
                       float scale, float *o, int64_t o_ld, int *err, cudaStream_t s) {
    using C = TW<DP, PACK>;
    const int Ns = attn_tcw_kstride(N);
    const int P = (Ns <= C::BK && NQ <= C::BQ) ? (C::BQ / NQ < C::BK / Ns ? C::BQ / NQ : C::BK / Ns) : 0;
    const int nt = P ? 1 : (N + C::BK - 1) / C::BK;
    const int qtiles = P ? 1 : (NQ + C::BQ - 1) / C::BQ;
    const int groups = P ? (Bw + P - 1) / P : Bw;
    if (groups > 65535 || heads > 65535) return cudaErrorInvalidValue;
    CUtensorMap tq, tk, tv;
    const uint64_t dq[2] = {static_cast<uint64_t>(DP), static_cast<uint64_t>(heads) * Bw * NQ};
    const uint64_t dk[2] = {static_cast<uint64_t>(DP), static_cast<uint64_t>(heads) * Bw * Ns};
    const uint64_t dv[2] = {static_cast<uint64_t>(Bw) * Ns, static_cast<uint64_t>(heads) * DP};
    const uint64_t sqk[1] = {static_cast<uint64_t>(DP) * 2}, sv[1] = {static_cast<uint64_t>(Bw) * Ns * 2};
    const uint32_t bq[2] = {64, C::BQ}, bk[2] = {64, C::BK}, bv[2] = {64, static_cast<uint32_t>(DP)};
    if (!make_tmap(&tq, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, qh, 2, dq, sqk, bq, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_tmap(&tk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, kh, 2, dk, sqk, bk, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_tmap(&tv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, vth, 2, dv, sv, bv, CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    if ((P > 0) != PACK) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(attn_tcw_kernel<DP, PACK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    attn_tcw_kernel<DP, PACK><<<dim3(static_cast<unsigned>(qtiles), static_cast<unsigned>(groups),
                               static_cast<unsigned>(heads)),
                          C::THREADS, C::SMEM_BYTES, s>>>(tq, tk, tv, Bw, NQ, N, Ns, hd, P, nt,
                                                          scale * 1.4426950408889634f, o, o_ld, err);
    return cudaGetLastError();
}

}  // namespace

cudaError_t attn_tcw_stage(const float *q, int64_t q_ld, const float *k, const float *v, int64_t kv_ld, int Bw,
                           int NQ, int N, int heads, int hd, __half *qh, __half *kh, __half *vth, cudaStream_t s) {
    if (Bw <= 0 || NQ <= 0 || N <= 0 || heads <= 0 || hd <= 0 || hd > 128 || NQ > N ||
        static_cast<int64_t>(Bw) * attn_tcw_kstride(N) >= (int64_t{1} << 31))
        return cudaErrorInvalidValue;
    const int Dp = attn_tcw_dpad(hd), Ns = attn_tcw_kstride(N);
    const int64_t tq = static_cast<int64_t>(heads) * Bw * NQ * (Dp / 8);
    const int64_t tk = static_cast<int64_t>(heads) * Bw * Ns * (Dp / 8);
    tcw_stage_rows_kernel<<<static_cast<unsigned>((tq + 255) / 256), 256, 0, s>>>(q, q_ld, NQ, NQ, Bw, heads, hd, Dp,
                                                                                 qh);
    tcw_stage_rows_kernel<<<static_cast<unsigned>((tk + 255) / 256), 256, 0, s>>>(k, kv_ld, N, Ns, Bw, heads, hd, Dp,
                                                                                 kh);
    const int64_t nk = static_cast<int64_t>(Bw) * Ns;
    tcw_stage_vt_kernel<<<dim3(static_cast<unsigned>((nk + 31) / 32), static_cast<unsigned>(Dp / 32),
                               static_cast<unsigned>(heads)),
                          dim3(32, 8), 0, s>>>(v, kv_ld, N, Ns, Bw, hd, Dp, vth);
    return cudaGetLastError();
}

cudaError_t attn_tcw(const __half *qh, const __half *kh, const __half *vth, int Bw, int NQ, int N, int heads, int hd,
                     float scale, float *o, int64_t o_ld, int *err, cudaStream_t s) {
    if (Bw <= 0 || NQ <= 0 || N <= 0 || heads <= 0 || hd <= 0 || hd > 128 || NQ > N || !qh || !kh || !vth || !o ||
        !err)
        return cudaErrorInvalidValue;
    const int Ns = attn_tcw_kstride(N);
    const bool pack = Ns <= 128 && NQ <= 128;  // whole windows share 128-row tiles
    if (attn_tcw_dpad(hd) == 64)
        return pack ? launch_tcw<64, true>(qh, kh, vth, Bw, NQ, N, heads, hd, scale, o, o_ld, err, s)
                    : launch_tcw<64, false>(qh, kh, vth, Bw, NQ, N, heads, hd, scale, o, o_ld, err, s);
    return pack ? launch_tcw<128, true>(qh, kh, vth, Bw, NQ, N, heads, hd, scale, o, o_ld, err, s)
                : launch_tcw<128, false>(qh, kh, vth, Bw, NQ, N, heads, hd, scale, o, o_ld, err, s);
}

}  // namespace b200
