// backend.cu -- the C ABI declared in include/sam3_b200.h: backend lifetime,
// device buffers, synchronous tensor copies, weight upload into the
// tensor-core layout, and the MUL_MAT node.
#include "../../include/sam3_b200.h"
#include "backend_impl.h"
#include "gemm_f16.cuh"
#include "mmq.cuh"
#include "vit_ops.cuh"

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

using namespace b200;

static thread_local std::string g_last_error;

void b200::set_error(const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
}

bool b200::cuda_ok(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return true;
    set_error("%s: %s", what, cudaGetErrorString(e));
    return false;
}

bool b200::Backend::ensure_scratch(size_t need_codes, size_t need_quads) {
    if (need_codes > act_codes_bytes) {
        if (act_codes) cudaFree(act_codes);
        act_codes = nullptr;
        act_codes_bytes = 0;
        if (!cuda_ok(cudaMalloc(&act_codes, need_codes), "cudaMalloc(activation codes)")) return false;
        act_codes_bytes = need_codes;
    }
    if (need_quads > act_quads_bytes) {
        if (act_quads) cudaFree(act_quads);
        act_quads = nullptr;
        act_quads_bytes = 0;
        if (!cuda_ok(cudaMalloc(&act_quads, need_quads), "cudaMalloc(activation scale quads)")) return false;
        if (!cuda_ok(cudaMemsetAsync(act_quads, 0, need_quads, stream), "cudaMemset(activation scale quads)"))
            return false;
        act_quads_bytes = need_quads;
    }
    return true;
}

void b200::Backend::prof_mark(int cls) {
    if (!profiling || cls < 0 || cls > 3) return;
    auto &v = prof_events[cls];
    if (prof_used[cls] == v.size()) {
        cudaEvent_t e;
        if (cudaEventCreate(&e) != cudaSuccess) return;
        v.push_back(e);
    }
    cudaEventRecord(v[prof_used[cls]++], stream);
}

extern "C" {

const char *sam3b200_last_error(void) { return g_last_error.c_str(); }

long long sam3b200_backend_launch_count(const sam3b200_backend *h) {
    auto *be = reinterpret_cast<const Backend *>(h);
    return be ? be->launches : -1;
}

int sam3b200_backend_profile(sam3b200_backend *h, int enable) {
    auto *be = reinterpret_cast<Backend *>(h);
    if (!be) return SAM3B200_STATUS_FAILED;
    be->profiling = enable;
    for (auto &u : be->prof_used) u = 0;
    return SAM3B200_STATUS_SUCCESS;
}

int sam3b200_backend_profile_read(sam3b200_backend *h, int cls, double *total_ms, int *n) {
    auto *be = reinterpret_cast<Backend *>(h);
    if (!be || cls < 0 || cls > 3) return SAM3B200_STATUS_FAILED;
    cudaSetDevice(be->device);
    if (!cuda_ok(cudaStreamSynchronize(be->stream), "profile sync")) return SAM3B200_STATUS_FAILED;
    double t = 0;
    const size_t pairs = be->prof_used[cls] / 2;
    for (size_t i = 0; i < pairs; ++i) {
        float ms = 0.f;
        if (!cuda_ok(cudaEventElapsedTime(&ms, be->prof_events[cls][2 * i], be->prof_events[cls][2 * i + 1]),
                     "event elapsed"))
            return SAM3B200_STATUS_FAILED;
        t += ms;
    }
    if (total_ms) *total_ms = t;
    if (n) *n = static_cast<int>(pairs);
    return SAM3B200_STATUS_SUCCESS;
}

sam3b200_backend *sam3b200_backend_init(int device) {
    int n = 0;
    if (!cuda_ok(cudaGetDeviceCount(&n), "cudaGetDeviceCount")) return nullptr;
    if (device < 0 || device >= n) {
        set_error("device %d out of range (%d devices)", device, n);
        return nullptr;
    }
    cudaDeviceProp prop;
    if (!cuda_ok(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties")) return nullptr;
    if (prop.major != 10) {
        set_error("device %d is sm_%d%d; this backend is built for sm_100a only", device, prop.major, prop.minor);
        return nullptr;
    }
    if (!cuda_ok(cudaSetDevice(device), "cudaSetDevice")) return nullptr;
    auto *be = new Backend();
    be->device = device;
    be->num_sms = prop.multiProcessorCount;
    if (const char *ev = getenv("SAM3B200_MMQ_CVT")) be->mmq_cvt = atoi(ev) == 0 ? 0 : 1;
    if (const char *ev = getenv("SAM3B200_MMQ_BN")) be->mmq_bn = atoi(ev) == 64 ? 64 : atoi(ev) == 128 ? 128 : 0;
    if (const char *ev = getenv("SAM3B200_ARITH"))
        be->mmq_arith = atoi(ev) == SAM3B200_ARITH_EXACT ? SAM3B200_ARITH_EXACT : SAM3B200_ARITH_DQ16;
    snprintf(be->name, sizeof(be->name), "B200[%d] %s", device, prop.name);
    if (!cuda_ok(cudaStreamCreateWithFlags(&be->stream, cudaStreamNonBlocking), "cudaStreamCreate") ||
        !cuda_ok(cudaMalloc(&be->err, sizeof(int)), "cudaMalloc(err)") ||
        !cuda_ok(cudaMemset(be->err, 0, sizeof(int)), "cudaMemset(err)")) {
        delete be;
        return nullptr;
    }
    return reinterpret_cast<sam3b200_backend *>(be);
}

void sam3b200_backend_free(sam3b200_backend *h) {
    auto *be = reinterpret_cast<Backend *>(h);
    if (!be) return;
    cudaSetDevice(be->device);
    cudaStreamSynchronize(be->stream);
    if (be->act_codes) cudaFree(be->act_codes);
    if (be->act_quads) cudaFree(be->act_quads);
    if (be->err) cudaFree(be->err);
    for (auto &v : be->prof_events)
        for (auto e : v) cudaEventDestroy(e);
    cudaStreamDestroy(be->stream);
    delete be;
}

const char *sam3b200_backend_name(const sam3b200_backend *h) {
    auto *be = reinterpret_cast<const Backend *>(h);
    return be ? be->name : "";
}

void *sam3b200_backend_stream(sam3b200_backend *h) {
    auto *be = reinterpret_cast<Backend *>(h);
    return be ? static_cast<void *>(be->stream) : nullptr;
}

int sam3b200_backend_synchronize(sam3b200_backend *h) {
    auto *be = reinterpret_cast<Backend *>(h);
    if (!be) return SAM3B200_STATUS_FAILED;
    cudaSetDevice(be->device);
    if (!cuda_ok(cudaStreamSynchronize(be->stream), "cudaStreamSynchronize")) return SAM3B200_STATUS_FAILED;
    int e = 0;
    if (!cuda_ok(cudaMemcpy(&e, be->err, sizeof(int), cudaMemcpyDeviceToHost), "read error word"))
        return SAM3B200_STATUS_FAILED;
    if (e != 0) {
        if (e == (1 << 20))  // ops.cu: a get_rows index outside the source rows
            set_error("get_rows: row index out of range (error word 0x%x)", e);
        else
            set_error("kernel pipeline wait timed out (error word 0x%x)", e);
        cudaMemset(be->err, 0, sizeof(int));
        return SAM3B200_STATUS_FAILED;
    }
    return SAM3B200_STATUS_SUCCESS;
}

void *sam3b200_buffer_alloc(sam3b200_backend *h, size_t size) {
    auto *be = reinterpret_cast<Backend *>(h);
    if (!be) return nullptr;
    cudaSetDevice(be->device);
    void *p = nullptr;
    if (!cuda_ok(cudaMalloc(&p, size ? size : 1), "cudaMalloc")) return nullptr;
    return p;
}

void sam3b200_buffer_free(sam3b200_backend *h, void *p) {
    auto *be = reinterpret_cast<Backend *>(h);
    if (!be || !p) return;
    cudaSetDevice(be->device);
    cudaStreamSynchronize(be->stream);
    cudaFree(p);
}

int sam3b200_tensor_set(sam3b200_backend *h, void *dev, const void *host, size_t offset, size_t size) {
    auto *be = reinterpret_cast<Backend *>(h);
    if (!be || (!dev && size)) return SAM3B200_STATUS_FAILED;
    cudaSetDevice(be->device);
    if (!cuda_ok(cudaMemcpyAsync(static_cast<char *>(dev) + offset, host, size, cudaMemcpyHostToDevice, be->stream),
                 "tensor_set") ||
        !cuda_ok(cudaStreamSynchronize(be->stream), "tensor_set sync"))
        return SAM3B200_STATUS_FAILED;
    return SAM3B200_STATUS_SUCCESS;
}

int sam3b200_tensor_get(sam3b200_backend *h, const void *dev, void *host, size_t offset, size_t size) {
    auto *be = reinterpret_cast<Backend *>(h);
    if (!be || (!dev && size)) return SAM3B200_STATUS_FAILED;
    cudaSetDevice(be->device);
    if (!cuda_ok(cudaMemcpyAsync(host, static_cast<const char *>(dev) + offset, size, cudaMemcpyDeviceToHost,
                                 be->stream),
                 "tensor_get") ||
        !cuda_ok(cudaStreamSynchronize(be->stream), "tensor_get sync"))
        return SAM3B200_STATUS_FAILED;
    return SAM3B200_STATUS_SUCCESS;
}

extern "C" int sam3b200_tensor_memset(sam3b200_backend *h, void *dev, int value, size_t offset, size_t size) {
    auto *be = reinterpret_cast<Backend *>(h);
    if (!be || (!dev && size)) {
        set_error("tensor_memset: null argument");
        return SAM3B200_STATUS_FAILED;
    }
    if (size == 0) return SAM3B200_STATUS_SUCCESS;
    cudaSetDevice(be->device);
    if (!cuda_ok(cudaMemsetAsync(static_cast<char *>(dev) + offset, value & 0xff, size, be->stream), "tensor_memset") ||
        !cuda_ok(cudaStreamSynchronize(be->stream), "tensor_memset sync"))
        return SAM3B200_STATUS_FAILED;
    return SAM3B200_STATUS_SUCCESS;
}

extern "C" int sam3b200_device_memory(int device, size_t *free_bytes, size_t *total_bytes) {
    if (!free_bytes || !total_bytes) {
        set_error("device_memory: null argument");
        return SAM3B200_STATUS_FAILED;
    }
    int prev = 0;
    cudaGetDevice(&prev);
    const bool ok = cuda_ok(cudaSetDevice(device), "cudaSetDevice") &&
                    cuda_ok(cudaMemGetInfo(free_bytes, total_bytes), "cudaMemGetInfo");
    cudaSetDevice(prev);
    return ok ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
}

extern "C" int sam3b200_device_count(int *count) {
    if (!count) {
        set_error("device_count: null argument");
        return SAM3B200_STATUS_FAILED;
    }
    *count = 0;
    return cuda_ok(cudaGetDeviceCount(count), "cudaGetDeviceCount") ? SAM3B200_STATUS_SUCCESS
                                                                     : SAM3B200_STATUS_FAILED;
}

sam3b200_weight *sam3b200_weight_upload(sam3b200_backend *h, int type, const void *host_blocks, int64_t ne0,
                                        int64_t ne1) {
    auto *be = reinterpret_cast<Backend *>(h);
    if (!be || !host_blocks) {
        set_error("weight_upload: null argument");
        return nullptr;
    }
    const bool quant = type == SAM3B200_TYPE_Q8_0 || type == SAM3B200_TYPE_Q4_0 || type == SAM3B200_TYPE_Q4_1;
    const bool dense = type == SAM3B200_TYPE_F16 || type == SAM3B200_TYPE_F32;
    if (!quant && !dense) {
        set_error("weight_upload: unsupported weight type %d (F32=0, F16=1, Q4_0=2, Q4_1=3, Q8_0=8)", type);
        return nullptr;
    }
    if (ne0 <= 0 || ne1 <= 0 || ne0 > (1 << 20) || ne1 > (1 << 24) || (quant && ne0 % 32 != 0) ||
        (dense && ne0 % 8 != 0)) {
        set_error("weight_upload: bad shape ne0=%lld ne1=%lld (ne0 must be a positive multiple of %d)",
                  (long long)ne0, (long long)ne1, quant ? 32 : 8);
        return nullptr;
    }
    cudaSetDevice(be->device);
    const int K = static_cast<int>(ne0), N = static_cast<int>(ne1);
    auto *w = new Weight();
    w->type = type;
    w->K = K;
    w->N = N;
    w->ld = (N + MMQ_ROW_ALIGN - 1) / MMQ_ROW_ALIGN * MMQ_ROW_ALIGN;
    void *raw = nullptr;
    bool ok;
    if (dense) {
        // F16 as is; F32 rounded to fp16 (the fp16 tensor-core GEMM computes both)
        const size_t elems = static_cast<size_t>(N) * K;
        ok = cuda_ok(cudaMalloc(&w->dense, elems * 2), "cudaMalloc(dense weight)");
        if (ok && type == SAM3B200_TYPE_F16) {
            ok = cuda_ok(cudaMemcpyAsync(w->dense, host_blocks, elems * 2, cudaMemcpyDefault, be->stream),
                         "weight upload");
        } else if (ok) {
            ok = cuda_ok(cudaMalloc(&raw, elems * 4), "cudaMalloc(weight staging)") &&
                 cuda_ok(cudaMemcpyAsync(raw, host_blocks, elems * 4, cudaMemcpyDefault, be->stream),
                         "weight upload") &&
                 cuda_ok(f32_rows_to_f16(static_cast<const float *>(raw), K, N, K, w->dense, be->stream), "to f16");
        }
        ok = ok && cuda_ok(cudaStreamSynchronize(be->stream), "weight upload sync");
    } else {
        const size_t block_bytes = type == SAM3B200_TYPE_Q8_0 ? 34 : type == SAM3B200_TYPE_Q4_0 ? 18 : 20;
        const size_t raw_bytes = static_cast<size_t>(N) * (K / 32) * block_bytes;
        const size_t quad_bytes = static_cast<size_t>(K / 32) * w->ld * 16;
        const size_t min_bytes = static_cast<size_t>(K / 32) * w->ld * 16;
        ok = cuda_ok(cudaMalloc(&raw, raw_bytes), "cudaMalloc(weight staging)") &&
             cuda_ok(cudaMalloc(&w->codes, weight_code_bytes(type, N, K)), "cudaMalloc(weight codes)") &&
             cuda_ok(cudaMalloc(&w->quads, quad_bytes), "cudaMalloc(weight scale quads)") &&
             cuda_ok(cudaMemsetAsync(w->quads, 0, quad_bytes, be->stream), "memset scale quads") &&
             (type != SAM3B200_TYPE_Q4_1 || (cuda_ok(cudaMalloc(&w->mins, min_bytes), "cudaMalloc(weight minima)") &&
                                             cuda_ok(cudaMemsetAsync(w->mins, 0, min_bytes, be->stream), "memset"))) &&
             cuda_ok(cudaMemcpyAsync(raw, host_blocks, raw_bytes, cudaMemcpyDefault, be->stream),
                     "weight upload") &&
             cuda_ok(repack_weight_blocks(type, raw, N, K, w->codes, w->quads, w->ld, be->stream, w->mins),
                     "weight repack") &&
             cuda_ok(cudaStreamSynchronize(be->stream), "weight upload sync");
    }
    if (raw) cudaFree(raw);
    if (!ok) {
        if (w->codes) cudaFree(w->codes);
        if (w->quads) cudaFree(w->quads);
        if (w->mins) cudaFree(w->mins);
        if (w->dense) cudaFree(w->dense);
        delete w;
        return nullptr;
    }
    return reinterpret_cast<sam3b200_weight *>(w);
}

void sam3b200_weight_free(sam3b200_backend *h, sam3b200_weight *wh) {
    auto *be = reinterpret_cast<Backend *>(h);
    auto *w = reinterpret_cast<Weight *>(wh);
    if (!w) return;
    if (be) {
        cudaSetDevice(be->device);
        cudaStreamSynchronize(be->stream);
    }
    cudaFree(w->codes);
    cudaFree(w->quads);
    cudaFree(w->mins);
    cudaFree(w->dense);
    cudaFree(w->w16);
    delete w;
}

int sam3b200_set_mmq_impl(sam3b200_backend *h, int impl) {
    auto *be = reinterpret_cast<Backend *>(h);
    if (!be) return -1;
    const int prev = be->mmq_impl;
    if (impl >= SAM3B200_MMQ_AUTO && impl <= SAM3B200_MMQ_SIMT) be->mmq_impl = impl;
    return prev;
}

int sam3b200_set_arith(sam3b200_backend *h, int arith) {
    auto *be = reinterpret_cast<Backend *>(h);
    if (!be) return -1;
    const int prev = be->mmq_arith;
    if (arith == SAM3B200_ARITH_EXACT || arith == SAM3B200_ARITH_DQ16) be->mmq_arith = arith;
    return prev;
}

}  // extern "C"

// Quantise x into the backend's activation scratch and run the MUL_MAT.
int b200::run_mul_mat(Backend *be, const Weight *w, const float *x, int64_t ldx, int64_t M, const float *bias,
                      float *dst, int64_t ldd, int32_t *dump) {
    if (!be || !w || !x || (!dst && !dump)) {
        set_error("mul_mat: null argument");
        return SAM3B200_STATUS_FAILED;
    }
    if (M <= 0 || M > (1 << 24) || ldx < w->K || (dst && ldd < w->N)) {
        set_error("mul_mat: bad shape M=%lld ldx=%lld ldd=%lld for K=%d N=%d", (long long)M, (long long)ldx,
                  (long long)ldd, w->K, w->N);
        return SAM3B200_STATUS_FAILED;
    }
    cudaSetDevice(be->device);
    const int Mi = static_cast<int>(M);
    if (w->dense) {
        // F16 / F32 weights: x -> fp16 (ggml's vec_dot_type for F16), fp16 tensor-core GEMM, f32 out
        if (dump) {
            set_error("mul_mat_block_dots: weight type %d has no integer block dots", w->type);
            return SAM3B200_STATUS_FAILED;
        }
        if (!be->ensure_scratch(static_cast<size_t>(Mi) * w->K * 2, 16)) return SAM3B200_STATUS_ALLOC_FAILED;
        GemmF16Args g;
        g.a = be->act_codes;
        g.b = w->dense;
        g.M = Mi;
        g.N = w->N;
        g.K = w->K;
        g.bias = bias;
        g.gelu = 0;
        g.out_f16 = 0;
        g.out = dst;
        g.ldo = ldd;
        g.store = GEMM_STORE_ROWMAJOR;
        g.win = 0;
        g.cout = 0;
        g.err = be->err;
        be->count(2);
        be->prof_mark(0);
        const bool ok = cuda_ok(f32_rows_to_f16(x, ldx, Mi, w->K, be->act_codes, be->stream), "x to f16") &&
                        cuda_ok(gemm_f16(g, be->num_sms, be->stream), "mul_mat f16 gemm");
        be->prof_mark(0);
        return ok ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
    }
    const int lda = (Mi + MMQ_ROW_ALIGN - 1) / MMQ_ROW_ALIGN * MMQ_ROW_ALIGN;
    const size_t quad_bytes = act_quad_bytes(w->K, lda);
    const bool q41 = w->type == SAM3B200_TYPE_Q4_1;  // Q8_1 activations: the sum fields follow the scales
    if (!be->ensure_scratch(static_cast<size_t>(Mi) * w->K, q41 ? 2 * quad_bytes : quad_bytes))
        return SAM3B200_STATUS_ALLOC_FAILED;
    void *sums = q41 ? static_cast<char *>(be->act_quads) + quad_bytes : nullptr;
    if (!cuda_ok(quantize_rows_q8(x, ldx, Mi, w->K, be->act_codes, be->act_quads, lda, be->stream, sums),
                 "quantize activations"))
        return SAM3B200_STATUS_FAILED;
    MmqArgs a;
    a.a = QMatrix{be->act_codes, be->act_quads, Mi, w->K, lda};
    a.b = QMatrix{w->codes, w->quads, w->N, w->K, w->ld, weight_nib(w->type)};
    a.bias = bias;
    a.y = dst;
    a.ldy = ldd;
    a.dump = dump;
    a.err = be->err;
    a.b_mins = w->mins;
    a.a_sums = sums;
    const int mode = dump ? MMQ_OUT_BLOCKDOTS : MMQ_OUT_F32;
    int impl = be->mmq_impl;
    if (impl == SAM3B200_MMQ_AUTO) impl = Mi < 64 ? SAM3B200_MMQ_SIMT : SAM3B200_MMQ_TC;
    cudaError_t e;
    be->count(2);
    be->prof_mark(0);
    if (impl == SAM3B200_MMQ_SIMT) e = mmq_simt(a, mode, be->stream);
    else e = mmq_tc(a, mode, be->num_sms, be->stream, be->mmq_cvt, be->mmq_bn);
    be->prof_mark(0);
    if (!cuda_ok(e, "mul_mat launch")) return SAM3B200_STATUS_FAILED;
    return SAM3B200_STATUS_SUCCESS;
}

extern "C" int sam3b200_mul_mat(sam3b200_backend *h, const sam3b200_weight *w, const float *x, int64_t ldx,
                                int64_t M, const float *bias, float *dst, int64_t ldd) {
    if (reinterpret_cast<uintptr_t>(bias) & 15) {  // the tensor-core epilogue reads the bias as float4
        set_error("mul_mat: bias must be 16-byte aligned");
        return SAM3B200_STATUS_FAILED;
    }
    return run_mul_mat(reinterpret_cast<Backend *>(h), reinterpret_cast<const Weight *>(w), x, ldx, M, bias, dst,
                       ldd, nullptr);
}

extern "C" int sam3b200_mul_mat_block_dots(sam3b200_backend *h, const sam3b200_weight *wh, const float *x, int64_t M,
                                           int32_t *dst_dev) {
    auto *be = reinterpret_cast<Backend *>(h);
    auto *w = reinterpret_cast<const Weight *>(wh);
    if (!w) {
        set_error("mul_mat_block_dots: null weight");
        return SAM3B200_STATUS_FAILED;
    }
    const int st = run_mul_mat(be, w, x, w->K, M, nullptr, nullptr, 0, dst_dev);
    if (st != SAM3B200_STATUS_SUCCESS) return st;
    return sam3b200_backend_synchronize(h);
}

extern "C" int sam3b200_mul_mat_dq16(sam3b200_backend *h, const sam3b200_weight *wh, const float *x, int64_t ldx,
                                     int64_t M, const float *bias, float *dst, int64_t ldd) {
    auto *be = reinterpret_cast<Backend *>(h);
    auto *w = const_cast<Weight *>(reinterpret_cast<const Weight *>(wh));
    if (!be || !w || !x || !dst) {
        set_error("mul_mat_dq16: null argument");
        return SAM3B200_STATUS_FAILED;
    }
    if (reinterpret_cast<uintptr_t>(bias) & 15) {
        set_error("mul_mat_dq16: bias must be 16-byte aligned");
        return SAM3B200_STATUS_FAILED;
    }
    if (w->type != SAM3B200_TYPE_Q8_0 && w->type != SAM3B200_TYPE_Q4_0) {
        set_error("mul_mat_dq16: weight type %d is not supported (Q8_0 and Q4_0 only)", w->type);
        return SAM3B200_STATUS_FAILED;
    }
    if (M <= 0 || M > (1 << 24) || ldx < w->K || ldd < w->N || w->K % 32 != 0) {
        set_error("mul_mat_dq16: bad shape M=%lld ldx=%lld ldd=%lld for K=%d N=%d", (long long)M, (long long)ldx,
                  (long long)ldd, w->K, w->N);
        return SAM3B200_STATUS_FAILED;
    }
    cudaSetDevice(be->device);
    if (!w->w16) {  // first use: the fp16 copy of the weight, kept with it until sam3b200_weight_free
        void *p = nullptr;
        if (!cuda_ok(cudaMalloc(&p, static_cast<size_t>(w->N) * w->K * 2), "cudaMalloc(fp16 weight)"))
            return SAM3B200_STATUS_ALLOC_FAILED;
        if (!cuda_ok(dequant_weight_f16(QMatrix{w->codes, w->quads, w->N, w->K, w->ld, weight_nib(w->type)}, p,
                                        be->stream),
                     "dequant weight")) {
            cudaFree(p);
            return SAM3B200_STATUS_FAILED;
        }
        w->w16 = p;
    }
    const int Mi = static_cast<int>(M);
    const int lda = (Mi + MMQ_ROW_ALIGN - 1) / MMQ_ROW_ALIGN * MMQ_ROW_ALIGN;
    const size_t code_bytes = (static_cast<size_t>(Mi) * w->K + 255) / 256 * 256;
    if (!be->ensure_scratch(code_bytes + static_cast<size_t>(Mi) * w->K * 2, act_quad_bytes(w->K, lda)))
        return SAM3B200_STATUS_ALLOC_FAILED;
    void *a16 = static_cast<char *>(be->act_codes) + code_bytes;
    MmqArgs a;
    a.a = QMatrix{be->act_codes, be->act_quads, Mi, w->K, lda};
    a.b = QMatrix{w->codes, w->quads, w->N, w->K, w->ld, weight_nib(w->type)};
    a.bias = bias;
    a.y = dst;
    a.ldy = ldd;
    a.dump = nullptr;
    a.err = be->err;
    be->count(3);
    if (!cuda_ok(quantize_rows_q8(x, ldx, Mi, w->K, be->act_codes, be->act_quads, lda, be->stream),
                 "quantize activations") ||
        !cuda_ok(dequant_act_f16(be->act_codes, be->act_quads, Mi, w->K, lda, a16, be->stream), "dequant activations"))
        return SAM3B200_STATUS_FAILED;
    be->prof_mark(0);
    const cudaError_t e = mmq_dq16(a, a16, w->w16, MMQ_OUT_F32, be->num_sms, be->stream);
    be->prof_mark(0);
    return cuda_ok(e, "mul_mat_dq16 launch") ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
}
