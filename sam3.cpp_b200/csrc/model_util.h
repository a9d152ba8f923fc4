// model_util.h -- device buffers and weight upload shared by the model-level
// runners (encoder.cu: SAM3 ViT + neck; hiera.cu: SAM2 Hiera + FPN).
#pragma once

#include <cstdint>
#include <cstring>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <vector>

#include "../../include/sam3_b200.h"
#include "backend_impl.h"
#include "mmq.cuh"

namespace b200 {

struct DevBuf {
    void *p = nullptr;
    size_t n = 0;
    DevBuf() = default;
    DevBuf(const DevBuf &) = delete;
    DevBuf &operator=(const DevBuf &) = delete;
    DevBuf(DevBuf &&o) noexcept : p(o.p), n(o.n) {
        o.p = nullptr;
        o.n = 0;
    }
    ~DevBuf() { release(); }
    bool alloc(size_t bytes) {
        if (p) cudaFree(p);
        p = nullptr;
        n = 0;
        if (!cuda_ok(cudaMalloc(&p, bytes ? bytes : 16), "cudaMalloc(encoder buffer)")) return false;
        n = bytes;
        return true;
    }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        n = 0;
    }
    template <class T>
    T *as() const { return static_cast<T *>(p); }
};

struct QWeight {  // a repacked linear weight (see mmq.cuh)
    DevBuf codes, quads;
    DevBuf w16;  // the same blocks dequantised to fp16 [N][K] (DQ16 arithmetic), when the runner uses it
    int K = 0, N = 0, ld = 0;
    int nib = 0;  // QMatrix::nib of the codes (0 Q8_0, 1 Q4_0)
    bool set = false;
};

inline bool upload(DevBuf &d, const void *h, size_t bytes, cudaStream_t s) {
    return d.alloc(bytes) && cuda_ok(cudaMemcpyAsync(d.p, h, bytes, cudaMemcpyHostToDevice, s), "upload") &&
           cuda_ok(cudaStreamSynchronize(s), "upload sync");
}

inline bool upload_f16(DevBuf &d, const std::vector<float> &v, cudaStream_t s) {
    std::vector<__half> h(v.size());
    for (size_t i = 0; i < v.size(); ++i) h[i] = __float2half_rn(v[i]);
    return upload(d, h.data(), h.size() * sizeof(__half), s);
}

inline int64_t type_row_bytes(int type, int64_t k) {
    switch (type) {
    case SAM3B200_TYPE_F32: return 4 * k;
    case SAM3B200_TYPE_F16: return 2 * k;
    case SAM3B200_TYPE_Q8_0: return k / 32 * 34;
    case SAM3B200_TYPE_Q4_0: return k / 32 * 18;
    case SAM3B200_TYPE_Q4_1: return k / 32 * 20;
    default: return -1;
    }
}

// F32 or F16 host data -> float vector
inline bool to_f32(int type, const void *data, int64_t n, std::vector<float> &out) {
    out.resize(static_cast<size_t>(n));
    if (type == SAM3B200_TYPE_F32) {
        memcpy(out.data(), data, static_cast<size_t>(n) * 4);
        return true;
    }
    if (type == SAM3B200_TYPE_F16) {
        const __half *h = static_cast<const __half *>(data);
        for (int64_t i = 0; i < n; ++i) out[i] = __half2float(h[i]);
        return true;
    }
    set_error("tensor type %d where F32/F16 is expected", type);
    return false;
}

inline bool upload_qweight(Backend *be, QWeight &w, int type, const void *data, int64_t K, int64_t N) {
    if ((type != SAM3B200_TYPE_Q8_0 && type != SAM3B200_TYPE_Q4_0) || K % 32 != 0) {
        set_error("linear weight must be Q8_0 or Q4_0 with ne0 %% 32 == 0 (got type %d, ne0 %lld)", type,
                  (long long)K);
        return false;
    }
    w.K = static_cast<int>(K);
    w.N = static_cast<int>(N);
    w.ld = (w.N + MMQ_ROW_ALIGN - 1) / MMQ_ROW_ALIGN * MMQ_ROW_ALIGN;
    w.nib = weight_nib(type);
    DevBuf raw;
    const size_t raw_bytes = static_cast<size_t>(type_row_bytes(type, K)) * N;
    const size_t qb = static_cast<size_t>(K / 32) * w.ld * 16;
    bool ok = raw.alloc(raw_bytes) && w.codes.alloc(weight_code_bytes(type, w.N, w.K)) && w.quads.alloc(qb) &&
              cuda_ok(cudaMemsetAsync(w.quads.p, 0, qb, be->stream), "memset quads") &&
              cuda_ok(cudaMemcpyAsync(raw.p, data, raw_bytes, cudaMemcpyHostToDevice, be->stream), "upload") &&
              cuda_ok(repack_weight_blocks(type, raw.p, w.N, w.K, w.codes.p, w.quads.p, w.ld, be->stream),
                      "repack") &&
              cuda_ok(cudaStreamSynchronize(be->stream), "repack sync");
    raw.release();
    w.set = ok;
    return ok;
}

// The fp16 dequantised copy of an uploaded weight (mmq.cuh, DQ16 arithmetic).
inline bool make_w16(Backend *be, QWeight &w) {
    return w.set && w.w16.alloc(static_cast<size_t>(w.N) * w.K * 2) &&
           cuda_ok(dequant_weight_f16(QMatrix{w.codes.p, w.quads.p, w.N, w.K, w.ld, w.nib}, w.w16.p, be->stream),
                   "dequant weight") &&
           cuda_ok(cudaStreamSynchronize(be->stream), "dequant sync");
}

// Upload rows [r0, r0 + rows) of a ggml [K, N] weight as a weight of its own
// (rows are independent in every type): the per-view MUL_MATs of a fused
// in_proj become separate weights.
inline sam3b200_weight *upload_weight_rows(Backend *be, int type, const void *data, int64_t K, int64_t r0,
                                           int64_t rows) {
    const int64_t rb = type_row_bytes(type, K);
    if (rb <= 0) {
        set_error("weight rows: type %d unsupported", type);
        return nullptr;
    }
    return sam3b200_weight_upload(reinterpret_cast<sam3b200_backend *>(be), type,
                                  static_cast<const char *>(data) + r0 * rb, K, rows);
}

}  // namespace b200
