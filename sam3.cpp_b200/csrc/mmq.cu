// mmq.cu -- quantised matrix multiply for sm_100a (ggml GGML_OP_MUL_MAT with
// Q8_0 / Q4_0 weights, activations quantised on the fly to Q8_0).
//
// Reference semantics (ggml generic vec_dot, reached from ggml_mul_mat at
// sam3.cpp:3742,3783,3796,3799):
//     y[m][n] = sum_b  (float) I_b[m][n] * (d_w[n][b] * d_x[m][b])
//     I_b     = sum_{k in block b} q_w[n][k] * q_x[m][k]   (int32)
// summed block by block in order in fp32.  This file computes exactly that:
// the tensor core forms every I_b (kind::f16 on integer-valued fp16 codes,
// exact in the fp32 accumulator), tensor memory holds it, and the epilogue
// warps fold it into per-thread fp32 accumulators with the two fp16 scales
// in block order -- the same fma sequence as the CPU oracle, so the result
// is bit-identical to it.
#include "mmq.cuh"
#include "ptx.cuh"

#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <mutex>

namespace b200 {

// ---------------------------------------------------------------------------
// Activation quantiser: one warp per 32-element block.  Rule of ggml-cpu's
// x86 quantize_row_q8_0: d = amax/127 stored as fp16, id = 127/amax,
// q = round-half-even(x * id).  (Division is IEEE-exact here: the library is
// built without fast-math.)
// ---------------------------------------------------------------------------
__global__ void quantize_rows_q8_kernel(const float *__restrict__ x, int64_t ldx, int M, int K,
                                        __half *__restrict__ codes, float *__restrict__ scales, int ld) {
    const int nblk = K >> 5;
    const int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (w >= static_cast<int64_t>(M) * nblk) return;
    const int m = static_cast<int>(w / nblk);
    const int b = static_cast<int>(w % nblk);
    const float v = x[static_cast<int64_t>(m) * ldx + b * 32 + lane];
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float d = __fdiv_rn(amax, 127.f);
    const float id = amax != 0.f ? __fdiv_rn(127.f, amax) : 0.f;
    const int q = __float2int_rn(__fmul_rn(v, id));
    codes[static_cast<int64_t>(m) * K + b * 32 + lane] = __int2half_rn(q);
    if (lane == 0) scales[static_cast<int64_t>(b) * ld + m] = __half2float(__float2half_rn(d));
}

cudaError_t quantize_rows_q8(const float *x, int64_t ldx, int M, int K, void *codes, float *scales, int ld,
                             cudaStream_t s) {
    if (K % 32 != 0 || M < 0) return cudaErrorInvalidValue;
    if (M == 0) return cudaSuccess;
    const int64_t warps = static_cast<int64_t>(M) * (K / 32);
    const int threads = 256;
    const int64_t blocks = (warps * 32 + threads - 1) / threads;
    quantize_rows_q8_kernel<<<static_cast<unsigned>(blocks), threads, 0, s>>>(x, ldx, M, K,
                                                                              static_cast<__half *>(codes), scales, ld);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Weight repack: ggml blocks -> integer fp16 codes + fp32 block scales.
// ---------------------------------------------------------------------------
__global__ void repack_q8_0_kernel(const uint8_t *__restrict__ blocks, int N, int K, __half *__restrict__ codes,
                                   float *__restrict__ scales, int ld) {
    const int nblk = K >> 5;
    const int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (w >= static_cast<int64_t>(N) * nblk) return;
    const int n = static_cast<int>(w / nblk);
    const int b = static_cast<int>(w % nblk);
    const uint8_t *blk = blocks + w * 34;
    const int8_t q = static_cast<int8_t>(blk[2 + lane]);
    codes[static_cast<int64_t>(n) * K + b * 32 + lane] = __int2half_rn(q);
    if (lane == 0) {
        const uint16_t dbits = *reinterpret_cast<const uint16_t *>(blk);
        scales[static_cast<int64_t>(b) * ld + n] = __half2float(__ushort_as_half(dbits));
    }
}

__global__ void repack_q4_0_kernel(const uint8_t *__restrict__ blocks, int N, int K, __half *__restrict__ codes,
                                   float *__restrict__ scales, int ld) {
    const int nblk = K >> 5;
    const int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (w >= static_cast<int64_t>(N) * nblk) return;
    const int n = static_cast<int>(w / nblk);
    const int b = static_cast<int>(w % nblk);
    const uint8_t *blk = blocks + w * 18;
    const uint8_t byte = blk[2 + (lane & 15)];
    const int nib = lane < 16 ? (byte & 0x0F) : (byte >> 4);
    codes[static_cast<int64_t>(n) * K + b * 32 + lane] = __int2half_rn(nib - 8);
    if (lane == 0) {
        const uint16_t dbits = *reinterpret_cast<const uint16_t *>(blk);
        scales[static_cast<int64_t>(b) * ld + n] = __half2float(__ushort_as_half(dbits));
    }
}

cudaError_t repack_weight_blocks(int type, const void *blocks, int N, int K, void *codes, float *scales, int ld,
                                 cudaStream_t s) {
    if (K % 32 != 0 || N <= 0) return cudaErrorInvalidValue;
    const int64_t warps = static_cast<int64_t>(N) * (K / 32);
    const int threads = 256;
    const unsigned grid = static_cast<unsigned>((warps * 32 + threads - 1) / threads);
    auto *b = static_cast<const uint8_t *>(blocks);
    auto *c = static_cast<__half *>(codes);
    if (type == 8) repack_q8_0_kernel<<<grid, threads, 0, s>>>(b, N, K, c, scales, ld);
    else if (type == 2) repack_q4_0_kernel<<<grid, threads, 0, s>>>(b, N, K, c, scales, ld);
    else return cudaErrorInvalidValue;
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// tcgen05 MMQ kernel.
//
// CTA tile 128 (tokens) x BN (output features); persistent over tiles.
// Warp roles (320 threads):
//   warp 0     : TMA producer (one lane) -- per stage two K-blocks of A and
//                B codes (128-byte swizzled) and their block scales.
//   warp 1     : TMEM allocator + MMA issuer (one lane) -- per K-block two
//                kind::f16 MMAs (K=16 each) into one of two TMEM buffers,
//                then tcgen05.commit to that buffer's "full" barrier.
//   warps 2..9 : epilogue -- per K-block read the int block dots from TMEM
//                and fold them in with d_x*d_w; at the end of the tile add
//                the bias and store.  Warp w reads TMEM lanes 32*(w%4)..+31
//                (the lane quarter it may access) and column half (w-2)/4.
// ---------------------------------------------------------------------------
template <int BN>
struct TcCfg {
    static constexpr int BM = 128;
    static constexpr int BK = 64;  // fp16 per stage row: 128 bytes = one swizzle atom
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int SA_BYTES = 2 * BM * 4;
    static constexpr int SB_BYTES = 2 * BN * 4;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + SA_BYTES + SB_BYTES;
    static constexpr int STAGES = BN == 256 ? 4 : 6;
    static constexpr int EPI_WARPS = 8;
    static constexpr int THREADS = 64 + EPI_WARPS * 32;
    static constexpr int COLS = BN / 2;
    static constexpr int TMEM_COLS = 2 * BN;
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 1024;
    static_assert(STAGE_BYTES % 1024 == 0, "stage alignment");
    static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

enum : int {
    ERR_WAIT_EMPTY = 1,
    ERR_WAIT_FULL_MMA = 2,
    ERR_WAIT_TEMPTY = 4,
    ERR_WAIT_FULL_EPI = 8,
    ERR_WAIT_TFULL = 16,
};

template <int BN, int MODE>
__global__ void __launch_bounds__(TcCfg<BN>::THREADS, 1)
    mmq_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                  const __grid_constant__ CUtensorMap tm_sa, const __grid_constant__ CUtensorMap tm_sb, int M, int N,
                  int nblk, const float *__restrict__ bias, float *__restrict__ y, int64_t ldy,
                  int32_t *__restrict__ dump, int *__restrict__ err) {
    using C = TcCfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::STAGES * C::STAGE_BYTES);
    uint64_t *empty = full + C::STAGES;
    uint64_t *tfull = empty + C::STAGES;
    uint64_t *tempty = tfull + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tempty + 2);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int num_m = (M + C::BM - 1) / C::BM;
    const int num_n = (N + BN - 1) / BN;
    const int num_tiles = num_m * num_n;
    const int kstages = (nblk + 1) >> 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1 + C::EPI_WARPS);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], C::EPI_WARPS);
        }
        fence_mbar_init();
        prefetch_tmap(&tm_a);
        prefetch_tmap(&tm_b);
        prefetch_tmap(&tm_sa);
        prefetch_tmap(&tm_sb);
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
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                const int m0 = (t % num_m) * C::BM;
                const int n0 = (t / num_m) * BN;
                for (int ks = 0; ks < kstages; ++ks) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, err, ERR_WAIT_EMPTY)) {
                        ok = false;
                        break;
                    }
                    uint8_t *sb = smem + stage * C::STAGE_BYTES;
                    mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
                    tma_load_2d(sb, &tm_a, &full[stage], ks * C::BK, m0);
                    tma_load_2d(sb + C::A_BYTES, &tm_b, &full[stage], ks * C::BK, n0);
                    tma_load_2d(sb + C::A_BYTES + C::B_BYTES, &tm_sa, &full[stage], m0, ks * 2);
                    tma_load_2d(sb + C::A_BYTES + C::B_BYTES + C::SA_BYTES, &tm_sb, &full[stage], n0, ks * 2);
                    if (++stage == C::STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16_f32(C::BM, BN);
            int stage = 0;
            uint32_t phase = 0;
            uint32_t blk = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                for (int ks = 0; ks < kstages; ++ks) {
                    if (!mbar_wait(&full[stage], phase, err, ERR_WAIT_FULL_MMA)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(smem + stage * C::STAGE_BYTES);
                    const uint32_t b_addr = a_addr + C::A_BYTES;
                    for (int j = 0; j < 2; ++j) {
                        if (ks * 2 + j >= nblk) break;
                        const uint32_t buf = blk & 1u;
                        if (!mbar_wait(&tempty[buf], ((blk >> 1) & 1u) ^ 1u, err, ERR_WAIT_TEMPTY)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t d_tmem = tmem_base + buf * BN;
#pragma unroll
                        for (int kk = 0; kk < 2; ++kk) {
                            const uint32_t koff = static_cast<uint32_t>((j * 2 + kk) * 32);  // 16 fp16 = 32 bytes
                            mma_f16(d_tmem, sw128_kmajor_desc(a_addr + koff), sw128_kmajor_desc(b_addr + koff), idesc,
                                    kk);
                        }
                        mma_commit(&tfull[buf]);
                        ++blk;
                    }
                    if (!ok) break;
                    mma_commit(&empty[stage]);
                    if (++stage == C::STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
        }
    } else {
        // ---- epilogue warps ----
        constexpr int CHUNK = C::COLS >= 128 ? 32 : 64;  // TMEM columns per batch (register budget)
        const int q = warp & 3;
        const int h = (warp - 2) >> 2;
        const int row = q * 32 + lane;
        const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
        int stage = 0;
        uint32_t phase = 0;
        uint32_t blk = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
            const int m0 = (t % num_m) * C::BM;
            const int n0 = (t / num_m) * BN;
            const int m = m0 + row;
            float acc[C::COLS];
#pragma unroll
            for (int i = 0; i < C::COLS; ++i) acc[i] = 0.f;
            for (int ks = 0; ks < kstages; ++ks) {
                // the stage's block scales have landed in shared memory
                if (!__all_sync(0xffffffffu, mbar_wait(&full[stage], phase, err, ERR_WAIT_FULL_EPI))) {
                    ok = false;
                    break;
                }
                const float *sa_s =
                    reinterpret_cast<const float *>(smem + stage * C::STAGE_BYTES + C::A_BYTES + C::B_BYTES);
                const float *sb_s = sa_s + 2 * C::BM;
                for (int j = 0; j < 2; ++j) {
                    const int b = ks * 2 + j;
                    if (b >= nblk) break;
                    const uint32_t buf = blk & 1u;
                    if (!__all_sync(0xffffffffu, mbar_wait(&tfull[buf], (blk >> 1) & 1u, err, ERR_WAIT_TFULL))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const float dx = sa_s[j * C::BM + row];
                    const float4 *dw4 = reinterpret_cast<const float4 *>(sb_s + j * BN + h * C::COLS);
#pragma unroll
                    for (int c0 = 0; c0 < C::COLS; c0 += CHUNK) {
                        uint32_t v[CHUNK];
                        const uint32_t ta = tmem_base + lane_addr + buf * BN + h * C::COLS + c0;
#pragma unroll
                        for (int c = 0; c < CHUNK; c += 32)
                            tmem_ld_32x32b_x32(ta + c, *reinterpret_cast<uint32_t(*)[32]>(&v[c]));
                        tmem_wait_ld();
                        if (c0 + CHUNK == C::COLS) {
                            // every column of this buffer is in registers: hand it back to the MMA warp
                            tc_fence_before();
                            __syncwarp();
                            if (lane == 0) mbar_arrive(&tempty[buf]);
                        }
                        if constexpr (MODE == MMQ_OUT_F32) {
#pragma unroll
                            for (int i = 0; i < CHUNK; i += 4) {
                                const float4 w4 = dw4[(c0 + i) >> 2];
                                float s0, s1, s2, s3;
                                fmul2(s0, s1, dx, dx, w4.x, w4.y);
                                fmul2(s2, s3, dx, dx, w4.z, w4.w);
                                ffma2(acc[c0 + i], acc[c0 + i + 1], __uint_as_float(v[i]), __uint_as_float(v[i + 1]),
                                      s0, s1);
                                ffma2(acc[c0 + i + 2], acc[c0 + i + 3], __uint_as_float(v[i + 2]),
                                      __uint_as_float(v[i + 3]), s2, s3);
                            }
                        } else {
                            if (m < M) {
                                for (int i = 0; i < CHUNK; ++i) {
                                    const int n = n0 + h * C::COLS + c0 + i;
                                    if (n < N)
                                        dump[(static_cast<int64_t>(m) * N + n) * nblk + b] =
                                            static_cast<int32_t>(__uint_as_float(v[i]));
                                }
                            }
                        }
                    }
                    ++blk;
                }
                if (!ok) break;
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[stage]);
                if (++stage == C::STAGES) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (!ok) break;
            if constexpr (MODE == MMQ_OUT_F32) {
                if (m < M) {
                    const int nb = n0 + h * C::COLS;
                    float *yr = y + static_cast<int64_t>(m) * ldy + nb;
                    const bool vec = ((ldy & 3) == 0) && ((reinterpret_cast<uintptr_t>(y) & 15) == 0);
#pragma unroll
                    for (int j = 0; j < C::COLS; j += 4) {
                        float4 o = make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
                        if (vec && nb + j + 3 < N) {
                            if (bias) {
                                const float4 bb = *reinterpret_cast<const float4 *>(bias + nb + j);
                                o.x += bb.x;
                                o.y += bb.y;
                                o.z += bb.z;
                                o.w += bb.w;
                            }
                            *reinterpret_cast<float4 *>(yr + j) = o;
                        } else {
                            const float ov[4] = {o.x, o.y, o.z, o.w};
                            for (int e = 0; e < 4; ++e)
                                if (nb + j + e < N) yr[j + e] = bias ? ov[e] + bias[nb + j + e] : ov[e];
                        }
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

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        void *p = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

static bool make_tmap_2d(CUtensorMap *map, CUtensorMapDataType dt, const void *base, uint64_t inner, uint64_t outer,
                         uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, dt, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, int MODE>
static cudaError_t launch_tc(const MmqArgs &a, int num_sms, cudaStream_t s) {
    using C = TcCfg<BN>;
    const int M = a.a.rows, N = a.b.rows, K = a.a.K;
    CUtensorMap tma, tmb, tmsa, tmsb;
    if (!make_tmap_2d(&tma, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.a.codes, K, M, uint64_t(K) * 2, C::BK, C::BM,
                      CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_tmap_2d(&tmb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.b.codes, K, N, uint64_t(K) * 2, C::BK, BN,
                      CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_tmap_2d(&tmsa, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a.a.scales, a.a.ld, K / 32, uint64_t(a.a.ld) * 4, C::BM,
                      2, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !make_tmap_2d(&tmsb, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a.b.scales, a.b.ld, K / 32, uint64_t(a.b.ld) * 4, BN, 2,
                      CU_TENSOR_MAP_SWIZZLE_NONE))
        return cudaErrorInvalidValue;
    auto kern = mmq_tc_kernel<BN, MODE>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    const int tiles = ((M + C::BM - 1) / C::BM) * ((N + BN - 1) / BN);
    const int grid = tiles < num_sms ? tiles : num_sms;
    kern<<<grid, C::THREADS, C::SMEM_BYTES, s>>>(tma, tmb, tmsa, tmsb, M, N, K / 32, a.bias, a.y, a.ldy, a.dump,
                                                  a.err);
    return cudaGetLastError();
}

cudaError_t mmq_tc(const MmqArgs &a, int mode, int bn, int num_sms, cudaStream_t s) {
    const int M = a.a.rows, N = a.b.rows, K = a.a.K;
    if (K != a.b.K || K % 32 != 0 || K % 8 != 0 || M <= 0 || N <= 0) return cudaErrorInvalidValue;
    if (a.a.ld % 4 != 0 || a.b.ld % 4 != 0 || a.a.ld < M || a.b.ld < N) return cudaErrorInvalidValue;
    if (num_sms <= 0) return cudaErrorInvalidValue;
    if (mode == MMQ_OUT_F32) {
        if (bn == 256) return launch_tc<256, MMQ_OUT_F32>(a, num_sms, s);
        if (bn == 128) return launch_tc<128, MMQ_OUT_F32>(a, num_sms, s);
    } else if (mode == MMQ_OUT_BLOCKDOTS) {
        if (bn == 256) return launch_tc<256, MMQ_OUT_BLOCKDOTS>(a, num_sms, s);
        if (bn == 128) return launch_tc<128, MMQ_OUT_BLOCKDOTS>(a, num_sms, s);
    }
    return cudaErrorInvalidValue;
}

// ---------------------------------------------------------------------------
// SIMT MMQ: one thread per output, same block-ordered fma sequence.
// ---------------------------------------------------------------------------
__global__ void mmq_simt_kernel(const __half *__restrict__ ca, const float *__restrict__ sa, int lda_s,
                                const __half *__restrict__ cb, const float *__restrict__ sb, int ldb_s, int M, int N,
                                int K, const float *__restrict__ bias, float *__restrict__ y, int64_t ldy,
                                int32_t *__restrict__ dump, int mode) {
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    const int m = blockIdx.y;
    if (n >= N || m >= M) return;
    const int nblk = K >> 5;
    const __half *ar = ca + static_cast<int64_t>(m) * K;
    const __half *br = cb + static_cast<int64_t>(n) * K;
    float acc = 0.f;
    for (int b = 0; b < nblk; ++b) {
        float isum = 0.f;
        for (int j = 0; j < 32; ++j) isum = fmaf(__half2float(ar[b * 32 + j]), __half2float(br[b * 32 + j]), isum);
        if (mode == MMQ_OUT_BLOCKDOTS) {
            dump[(static_cast<int64_t>(m) * N + n) * nblk + b] = static_cast<int32_t>(isum);
        } else {
            acc = fmaf(isum, sa[static_cast<int64_t>(b) * lda_s + m] * sb[static_cast<int64_t>(b) * ldb_s + n], acc);
        }
    }
    if (mode == MMQ_OUT_F32) y[static_cast<int64_t>(m) * ldy + n] = bias ? acc + bias[n] : acc;
}

cudaError_t mmq_simt(const MmqArgs &a, int mode, cudaStream_t s) {
    const int M = a.a.rows, N = a.b.rows, K = a.a.K;
    if (K != a.b.K || K % 32 != 0 || M <= 0 || N <= 0 || M > 65535) return cudaErrorInvalidValue;
    dim3 grid((N + 127) / 128, M);
    mmq_simt_kernel<<<grid, 128, 0, s>>>(static_cast<const __half *>(a.a.codes), a.a.scales, a.a.ld,
                                         static_cast<const __half *>(a.b.codes), a.b.scales, a.b.ld, M, N, K, a.bias,
                                         a.y, a.ldy, a.dump, mode);
    return cudaGetLastError();
}

}  // namespace b200
