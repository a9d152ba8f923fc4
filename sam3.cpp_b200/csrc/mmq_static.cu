// mmq_static.cu -- sam3b200_mul_mat_noalloc: the quantised MUL_MAT for
// callers that cannot allocate device memory.
//
// sam3b200_mul_mat quantises the activations into scratch buffers that the
// backend allocates (and grows) with cudaMalloc on demand.  Some callers
// cannot let that happen while they compute: a host framework that plans
// every device byte up front (ggml's graph allocator hands a backend its
// buffers and expects graph_compute to allocate nothing), or a latency-bound
// loop that cannot absorb cudaMalloc's implicit device synchronisation and
// its failure path.  This entry point computes the same result with its
// scratch in a fixed array compiled into the library instead.
//
// The array lives in device memory of every GPU that loads the library, for
// the life of the process, and is shared by all calls on that device: two
// calls that overlap on the GPU (different streams or backends on the same
// device) race on it and must be serialised by the caller.  Its device
// address is looked up once per device, on the first call there; a
// cudaDeviceReset after that first call is not supported (the module is
// reloaded and the cached address would be stale).
#include "../../include/sam3_b200.h"
#include "backend_impl.h"
#include "mmq.cuh"

#include <mutex>

namespace b200 {

// 48 MiB: enough for every MUL_MAT of the SAM3 ViT-32 at 5184 tokens
// (largest: mlp.lin2, K = 4736: 24.6 MB of codes + 1.6 MB of scale records).
constexpr size_t NOALLOC_SCRATCH_BYTES = size_t(48) << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int MAX_DEVICES = 64;
std::mutex g_addr_mutex;
void *g_addr[MAX_DEVICES] = {nullptr};

// Device address of the scratch array on `device`, resolved once per device
// with that device current (the array's host-side name is only a stand-in).
void *scratch_address(int device) {
    if (device < 0 || device >= MAX_DEVICES) return nullptr;
    std::lock_guard<std::mutex> lock(g_addr_mutex);
    if (!g_addr[device]) {
        void *p = nullptr;
        if (!cuda_ok(cudaSetDevice(device), "cudaSetDevice") ||
            !cuda_ok(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(no-alloc scratch)"))
            return nullptr;
        g_addr[device] = p;
    }
    return g_addr[device];
}

}  // namespace
}  // namespace b200

using namespace b200;

extern "C" int sam3b200_mul_mat_noalloc(sam3b200_backend *h, const sam3b200_weight *wh, const float *x, int64_t ldx,
                                        int64_t M, const float *bias, float *dst, int64_t ldd) {
    auto *be = reinterpret_cast<Backend *>(h);
    auto *w = reinterpret_cast<const Weight *>(wh);
    if (reinterpret_cast<uintptr_t>(bias) & 15) {  // the tensor-core epilogue reads the bias as float4
        set_error("mul_mat_noalloc: bias must be 16-byte aligned");
        return SAM3B200_STATUS_FAILED;
    }
    if (!be || !w || !x || !dst) {
        set_error("mul_mat_noalloc: null argument");
        return SAM3B200_STATUS_FAILED;
    }
    if (w->dense || w->mins) {
        set_error("mul_mat_noalloc: weight type %d is not supported (Q8_0 and Q4_0 only)", w->type);
        return SAM3B200_STATUS_FAILED;
    }
    if (M <= 0 || M > (1 << 24) || ldx < w->K || ldd < w->N) {
        set_error("mul_mat_noalloc: bad shape M=%lld ldx=%lld ldd=%lld for K=%d N=%d", (long long)M, (long long)ldx,
                  (long long)ldd, w->K, w->N);
        return SAM3B200_STATUS_FAILED;
    }
    const int Mi = static_cast<int>(M);
    const int lda = (Mi + MMQ_ROW_ALIGN - 1) / MMQ_ROW_ALIGN * MMQ_ROW_ALIGN;
    const size_t codes_bytes = (static_cast<size_t>(Mi) * w->K + 255) / 256 * 256;
    const size_t quad_bytes = act_quad_bytes(w->K, lda);
    if (codes_bytes + quad_bytes > NOALLOC_SCRATCH_BYTES) {
        set_error("mul_mat_noalloc: M=%d x K=%d needs %zu bytes of scratch, more than the fixed %zu-byte array "
                  "(use sam3b200_mul_mat, or split M)",
                  Mi, w->K, codes_bytes + quad_bytes, NOALLOC_SCRATCH_BYTES);
        return SAM3B200_STATUS_FAILED;
    }
    unsigned char *base = static_cast<unsigned char *>(scratch_address(be->device));
    if (!base) return SAM3B200_STATUS_FAILED;
    if (!cuda_ok(cudaSetDevice(be->device), "cudaSetDevice")) return SAM3B200_STATUS_FAILED;
    void *codes = base;
    void *quads = base + codes_bytes;
    // Nothing in the scratch has to start at zero: every code and scale of
    // rows [0, M) is rewritten below (the quantiser also zeroes the record
    // slots past a row's last block, which the scale MMA reads), and padding
    // rows [M, lda) only feed output rows that are never stored.
    if (!cuda_ok(quantize_rows_q8(x, ldx, Mi, w->K, codes, quads, lda, be->stream), "quantize activations"))
        return SAM3B200_STATUS_FAILED;
    MmqArgs a;
    a.a = QMatrix{codes, quads, Mi, w->K, lda};
    a.b = QMatrix{w->codes, w->quads, w->N, w->K, w->ld, weight_nib(w->type)};
    a.bias = bias;
    a.y = dst;
    a.ldy = ldd;
    a.dump = nullptr;
    a.err = be->err;
    be->count(2);
    // the same kernel choice as sam3b200_mul_mat (Q4_1 is refused above)
    int impl = be->mmq_impl;
    if (impl == SAM3B200_MMQ_AUTO) impl = Mi < 64 ? SAM3B200_MMQ_SIMT : SAM3B200_MMQ_TC;
    const cudaError_t e = impl == SAM3B200_MMQ_SIMT
                              ? mmq_simt(a, MMQ_OUT_F32, be->stream)
                              : mmq_tc(a, MMQ_OUT_F32, be->num_sms, be->stream, be->mmq_cvt, be->mmq_bn);
    if (!cuda_ok(e, "mul_mat_noalloc launch")) return SAM3B200_STATUS_FAILED;
    return SAM3B200_STATUS_SUCCESS;
}
