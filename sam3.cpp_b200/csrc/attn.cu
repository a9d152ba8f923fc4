// attn.cu -- ggml_flash_attn_ext without mask (sam3.cpp:3778): per (window,
// head) out = softmax(Q K^T * scale) V, head_dim 64.  Q, K, V are bf16
// [B*heads][N][64]; the output is f32 [B*N][heads*64] (ggml's
// [HD, NH, N, B] result reshaped to [E, W, H, B], sam3.cpp:3780-3781).
//
// Flash-attention tiling: a CTA owns 64 query rows of one (window, head),
// four warps x 16 rows; keys stream through shared memory in 64-row tiles
// (double-buffered cp.async), scores and the running output stay in
// registers, the softmax is online (running max and sum per row).
#include "attn.cuh"

#include <cstdint>

#include <cuda_bf16.h>

namespace b200 {

namespace {

constexpr int BQ = 64, BKV = 64, HD = 64;

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// rows of 64 bf16 (128 bytes); 16-byte chunks XOR-swizzled by row % 8
__device__ __forceinline__ uint32_t swz(int row, int chunk) { return row * 128 + ((chunk ^ (row & 7)) << 4); }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, bool valid) {
    const int n = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}

// 64 rows x 128 bytes from global rows [row0, row0 + 64) (rows >= n are zero)
__device__ __forceinline__ void load_tile(uint8_t *sm, const __nv_bfloat16 *g, int row0, int n) {
    const uint32_t base = smem_addr(sm);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int c = threadIdx.x + i * 128;
        const int row = c >> 3, ch = c & 7;
        const bool valid = row0 + row < n;
        const __nv_bfloat16 *src = g + static_cast<int64_t>(valid ? row0 + row : 0) * HD + ch * 8;
        cp_async16(base + swz(row, ch), src, valid);
    }
}

}  // namespace

__global__ void __launch_bounds__(128) flash_attn_kernel(const __nv_bfloat16 *__restrict__ q,
                                                         const __nv_bfloat16 *__restrict__ k,
                                                         const __nv_bfloat16 *__restrict__ v, int N, int heads,
                                                         float scale_log2, float *__restrict__ out) {
    __shared__ __align__(128) uint8_t sq[BQ * 128];
    __shared__ __align__(128) uint8_t sk[2][BKV * 128];
    __shared__ __align__(128) uint8_t sv[2][BKV * 128];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int bh = blockIdx.y;
    const int q0 = blockIdx.x * BQ;
    const __nv_bfloat16 *qg = q + static_cast<int64_t>(bh) * N * HD;
    const __nv_bfloat16 *kg = k + static_cast<int64_t>(bh) * N * HD;
    const __nv_bfloat16 *vg = v + static_cast<int64_t>(bh) * N * HD;
    const int ntiles = (N + BKV - 1) / BKV;

    load_tile(sq, qg, q0, N);
    load_tile(sk[0], kg, 0, N);
    load_tile(sv[0], vg, 0, N);
    asm volatile("cp.async.commit_group;" ::: "memory");

    uint32_t qa[4][4];
    float o[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
    const int g = lane >> 2, tq = lane & 3;

    for (int it = 0; it < ntiles; ++it) {
        const int buf = it & 1;
        if (it + 1 < ntiles) {
            load_tile(sk[buf ^ 1], kg, (it + 1) * BKV, N);
            load_tile(sv[buf ^ 1], vg, (it + 1) * BKV, N);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        asm volatile("cp.async.wait_group 1;" ::: "memory");
        __syncthreads();
        if (it == 0) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const int row = warp * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
                const int ch = 2 * kk + (lane >> 4);
                ldsm_x4(smem_addr(sq) + swz(row, ch), qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3]);
            }
        }
        // S = Q K^T for this warp's 16 rows x 64 keys
        float s[8][4];
#pragma unroll
        for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
        const uint32_t kb = smem_addr(sk[buf]);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
            for (int j = 0; j < 8; j += 2) {
                const int row = 8 * j + (lane & 7) + 8 * (lane >> 4);
                const int ch = 2 * kk + ((lane >> 3) & 1);
                uint32_t b0, b1, b2, b3;
                ldsm_x4(kb + swz(row, ch), b0, b1, b2, b3);
                mma_bf16(s[j], qa[kk], b0, b1);
                mma_bf16(s[j + 1], qa[kk], b2, b3);
            }
        }
        // online softmax (rows g and g + 8 of the warp's 16)
        const int key0 = it * BKV;
        float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int key = key0 + 8 * j + 2 * tq + (e & 1);
                float val = key < N ? s[j][e] * scale_log2 : -INFINITY;
                s[j][e] = val;
                mx[e >> 1] = fmaxf(mx[e >> 1], val);
            }
        }
        float alpha[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
            const float m_new = fmaxf(m_run[r], mx[r]);
            alpha[r] = exp2f(m_run[r] - m_new);
            m_run[r] = m_new;
        }
        float rs[2] = {0.f, 0.f};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float p = exp2f(s[j][e] - m_run[e >> 1]);
                s[j][e] = p;
                rs[e >> 1] += p;
            }
        }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
            rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
            l_run[r] = l_run[r] * alpha[r] + rs[r];
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            o[j][0] *= alpha[0];
            o[j][1] *= alpha[0];
            o[j][2] *= alpha[1];
            o[j][3] *= alpha[1];
        }
        // O += P V
        const uint32_t vb = smem_addr(sv[buf]);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            uint32_t pa[4];
            pa[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
            pa[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
            pa[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
            pa[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
            for (int j = 0; j < 8; j += 2) {
                const int row = 16 * kk + (lane & 7) + 8 * ((lane >> 3) & 1);
                const int ch = j + (lane >> 4);
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(vb + swz(row, ch), b0, b1, b2, b3);
                mma_bf16(o[j], pa, b0, b1);
                mma_bf16(o[j + 1], pa, b2, b3);
            }
        }
        __syncthreads();
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");

    const int b = bh / heads, h = bh % heads;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int n = q0 + warp * 16 + g + 8 * r;
        if (n >= N) continue;
        const float inv = 1.0f / l_run[r];
        float *dst = out + (static_cast<int64_t>(b) * N + n) * heads * HD + h * HD;
#pragma unroll
        for (int j = 0; j < 8; ++j)
            *reinterpret_cast<float2 *>(dst + 8 * j + 2 * tq) = make_float2(o[j][2 * r] * inv, o[j][2 * r + 1] * inv);
    }
}

cudaError_t flash_attention(const void *q, const void *k, const void *v, int B, int N, int heads, float scale,
                            float *out, cudaStream_t s) {
    if (B <= 0 || N <= 0 || heads <= 0) return cudaErrorInvalidValue;
    dim3 grid((N + BQ - 1) / BQ, B * heads);
    flash_attn_kernel<<<grid, 128, 0, s>>>(static_cast<const __nv_bfloat16 *>(q),
                                           static_cast<const __nv_bfloat16 *>(k),
                                           static_cast<const __nv_bfloat16 *>(v), N, heads,
                                           scale * 1.4426950408889634f, out);
    return cudaGetLastError();
}

}  // namespace b200
