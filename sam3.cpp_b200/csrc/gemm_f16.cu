// gemm_f16.cu -- fp16 tcgen05 GEMM with TMEM accumulation over K (see
// gemm_f16.cuh).  CTA tile 128 x 128, persistent over tiles, 192 threads:
//   warp 0     : TMA producer (one lane), 64-wide K stages of A and B
//                (128-byte swizzle);
//   warp 1     : TMEM allocator + MMA issuer (one lane), four K=16 MMAs
//                per stage accumulating into TMEM buffer (tile & 1);
//   warps 2..17: epilogue, four warps per TMEM lane quarter (warp w reads
//                lane quarter w % 4 and the 32-column slice (w - 2) / 4 of a
//                row), while the MMA warp already works on the next tile in
//                the other buffer.  With a single epilogue warp per
//                sub-partition the drain of a 128 x 128 tile outlasted the
//                MMAs of the next one for K <= 1024.
#include "gemm_f16.cuh"
#include "ptx.cuh"
#include "tmap.h"

#include <cuda_fp16.h>

namespace b200 {

struct GCfg {
    static constexpr int BM = 128, BN = 128, BK = 64;
    static constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGES = 6;
    static constexpr int BAR_OFF = STAGES * STAGE_BYTES;
    static constexpr int EPI_WARPS = 16;
    static constexpr int THREADS = 64 + 32 * EPI_WARPS;
    static constexpr int COLS = BN / (EPI_WARPS / 4);  // columns per epilogue thread
    static constexpr int TMEM_COLS = 256;
    static constexpr int STAGE_OFF = BAR_OFF + 256;  // per-warp 2 KB row-segment staging (ptx.cuh stage_put)
    static constexpr int SMEM_BYTES = STAGE_OFF + EPI_WARPS * 2048 + 1024;
    static_assert(SMEM_BYTES <= 232448, "smem");
};

__device__ __forceinline__ float gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752440f)); }

__global__ void __launch_bounds__(GCfg::THREADS, 1)
    gemm_f16_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b, int M, int N,
                    int K, const float *__restrict__ bias, int gelu, int out_f16, void *__restrict__ out, int64_t ldo,
                    int store, int win, int cout, int *__restrict__ err) {
    using C = GCfg;
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
        // TMA producer: warp-uniform loop, one elected lane issues
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
            const int m0 = (t % num_m) * C::BM, n0 = (t / num_m) * C::BN;
            for (int ks = 0; ks < kstages; ++ks) {
                if (!__all_sync(0xffffffffu, mbar_wait(&empty[stage], phase ^ 1u, err, 1))) {
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
        // MMA issuer: warp-uniform loop, one elected lane issues
        constexpr uint32_t idesc = idesc_f16_f32(C::BM, C::BN);
        int stage = 0;
        uint32_t phase = 0, it = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++it) {
            const uint32_t buf = it & 1u;
            if (!__all_sync(0xffffffffu, mbar_wait(&tempty[buf], ((it >> 1) & 1u) ^ 1u, err, 4))) break;
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + buf * C::BN;
            for (int ks = 0; ks < kstages; ++ks) {
                if (!__all_sync(0xffffffffu, mbar_wait(&full[stage], phase, err, 2))) {
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
        const int cs = ((warp - 2) >> 2) * C::COLS;  // this warp's column slice
        const int row = q * 32 + lane;
        const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
        uint32_t it = 0;
        for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++it) {
            const uint32_t buf = it & 1u;
            if (!__all_sync(0xffffffffu, mbar_wait(&tfull[buf], (it >> 1) & 1u, err, 16))) break;
            tc_fence_after();
            const int m0 = (t % num_m) * C::BM, n0 = (t / num_m) * C::BN;
            const int m = m0 + row;
            for (int c = cs; c < cs + C::COLS; c += 32) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(tmem_base + lane_addr + buf * C::BN + c, v);
                tmem_wait_ld();
                if (c + 32 == cs + C::COLS) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tempty[buf]);
                }
                const int nc = n0 + c;
                // whole 32-column chunks with 16-byte-aligned row segments: the warp stores 8 rows x 64
                // bytes per instruction through its staging buffer (warp-uniform condition)
                const bool staged = nc + 32 <= N && (reinterpret_cast<uintptr_t>(out) & 15) == 0 &&
                                    (store == GEMM_STORE_CONVT2X2 || (ldo & (out_f16 ? 7 : 3)) == 0);
                if (staged) {
                    float f[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        float y = __uint_as_float(v[i]);
                        const int n = nc + i;
                        if (bias) y = y + bias[store == GEMM_STORE_CONVT2X2 ? n % cout : n];
                        if (gelu) y = gelu_erf(y);
                        f[i] = y;
                    }
                    long long base = -1;  // element offset of this lane's row segment; -1: row past M
                    if (m < M) {
                        if (store == GEMM_STORE_CONVT2X2) {
                            const int g = nc / cout, co = nc % cout;
                            const int iy = m / win, ix = m % win, ky = g >> 1, kx = g & 1;
                            base = (static_cast<long long>(2 * iy + ky) * (2 * win) + 2 * ix + kx) * cout + co;
                        } else {
                            base = static_cast<long long>(m) * ldo + nc;
                        }
                    }
                    uint4 *st = reinterpret_cast<uint4 *>(smem + C::STAGE_OFF) + (warp - 2) * 128;
                    if (out_f16) {
                        uint32_t hw[16];
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            const __half2 h2 = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
                            hw[i] = *reinterpret_cast<const uint32_t *>(&h2);
                        }
                        const uint4 seg[4] = {make_uint4(hw[0], hw[1], hw[2], hw[3]), make_uint4(hw[4], hw[5], hw[6], hw[7]),
                                              make_uint4(hw[8], hw[9], hw[10], hw[11]),
                                              make_uint4(hw[12], hw[13], hw[14], hw[15])};
                        stage_put(st, lane, seg);
#pragma unroll
                        for (int it = 0; it < 4; ++it) {
                            const int r = it * 8 + (lane >> 2), ch = lane & 3;
                            const long long b = __shfl_sync(0xffffffffu, base, r);
                            if (b >= 0) *reinterpret_cast<uint4 *>(static_cast<__half *>(out) + b + ch * 8) = st[stage_idx(r, ch)];
                        }
                    } else {
#pragma unroll
                        for (int c0 = 0; c0 < 32; c0 += 16) {
                            uint4 seg[4];
#pragma unroll
                            for (int k = 0; k < 4; ++k)
                                seg[k] = make_uint4(__float_as_uint(f[c0 + 4 * k]), __float_as_uint(f[c0 + 4 * k + 1]),
                                                    __float_as_uint(f[c0 + 4 * k + 2]), __float_as_uint(f[c0 + 4 * k + 3]));
                            stage_put(st, lane, seg);
#pragma unroll
                            for (int it = 0; it < 4; ++it) {
                                const int r = it * 8 + (lane >> 2), ch = lane & 3;
                                const long long b = __shfl_sync(0xffffffffu, base, r);
                                if (b >= 0)
                                    *reinterpret_cast<uint4 *>(static_cast<float *>(out) + b + c0 + ch * 4) =
                                        st[stage_idx(r, ch)];
                            }
                        }
                    }
                    continue;
                }
                if (m >= M || nc >= N) continue;
                float f[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    float y = __uint_as_float(v[i]);
                    const int n = nc + i;
                    if (bias && n < N) y = y + bias[store == GEMM_STORE_CONVT2X2 ? n % cout : n];
                    if (gelu) y = gelu_erf(y);
                    f[i] = y;
                }
                int64_t base;
                if (store == GEMM_STORE_CONVT2X2) {
                    const int g = nc / cout, co = nc % cout;  // 32 columns stay inside one (ky, kx) group
                    const int iy = m / win, ix = m % win, ky = g >> 1, kx = g & 1;
                    base = (static_cast<int64_t>(2 * iy + ky) * (2 * win) + 2 * ix + kx) * cout + co;
                } else {
                    base = static_cast<int64_t>(m) * ldo + nc;
                }
                const bool full_chunk = nc + 32 <= N;
                if (out_f16) {
                    __half *o = static_cast<__half *>(out) + base;
                    if (full_chunk && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
                        for (int i = 0; i < 32; i += 8) {
                            __half2 h0 = __floats2half2_rn(f[i], f[i + 1]), h1 = __floats2half2_rn(f[i + 2], f[i + 3]);
                            __half2 h2 = __floats2half2_rn(f[i + 4], f[i + 5]), h3 = __floats2half2_rn(f[i + 6], f[i + 7]);
                            uint4 u;
                            u.x = *reinterpret_cast<uint32_t *>(&h0);
                            u.y = *reinterpret_cast<uint32_t *>(&h1);
                            u.z = *reinterpret_cast<uint32_t *>(&h2);
                            u.w = *reinterpret_cast<uint32_t *>(&h3);
                            *reinterpret_cast<uint4 *>(o + i) = u;
                        }
                    } else {
                        for (int i = 0; i < 32 && nc + i < N; ++i) o[i] = __float2half_rn(f[i]);
                    }
                } else {
                    float *o = static_cast<float *>(out) + base;
                    if (full_chunk && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
                        for (int i = 0; i < 32; i += 4)
                            *reinterpret_cast<float4 *>(o + i) = make_float4(f[i], f[i + 1], f[i + 2], f[i + 3]);
                    } else {
                        for (int i = 0; i < 32 && nc + i < N; ++i) o[i] = f[i];
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, C::TMEM_COLS);
}

cudaError_t gemm_f16(const GemmF16Args &a, int num_sms, cudaStream_t s) {
    using C = GCfg;
    if (a.M <= 0 || a.N <= 0 || a.K <= 0 || a.K % 8 != 0 || num_sms <= 0) return cudaErrorInvalidValue;
    if (a.store == GEMM_STORE_CONVT2X2 && (a.cout % 32 != 0 || a.win <= 0 || a.N != 4 * a.cout))
        return cudaErrorInvalidValue;
    CUtensorMap ta, tb;
    const uint64_t da[2] = {uint64_t(a.K), uint64_t(a.M)}, db[2] = {uint64_t(a.K), uint64_t(a.N)};
    const uint64_t st[1] = {uint64_t(a.K) * 2};
    const uint32_t bx[2] = {C::BK, 128};
    if (!make_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.a, 2, da, st, bx, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.b, 2, db, st, bx, CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(gemm_f16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    const int tiles = ((a.M + 127) / 128) * ((a.N + 127) / 128);
    const int grid = tiles < num_sms ? tiles : num_sms;
    gemm_f16_kernel<<<grid, C::THREADS, C::SMEM_BYTES, s>>>(ta, tb, a.M, a.N, a.K, a.bias, a.gelu, a.out_f16, a.out,
                                                            a.ldo, a.store, a.win, a.cout, a.err);
    return cudaGetLastError();
}

}  // namespace b200
