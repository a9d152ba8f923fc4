// diag.cu -- failure-path diagnostics of the backend.
//
// Every mbarrier wait in the tensor-core pipelines is bounded: when a phase
// never completes, the waiting thread gives up, ORs a code into the
// backend's device error word and the kernel ends; the host then reads the
// word in sam3b200_backend_synchronize, which returns SAM3B200_STATUS_FAILED,
// and the CUDA context stays usable.  sam3b200_debug_wait_timeout exercises
// exactly that path on a barrier that nothing ever arrives on, with a short
// limit, so the failure path can be tested without breaking a real kernel.
#include "../../include/sam3_b200.h"
#include "backend_impl.h"
#include "ptx.cuh"

namespace b200 {
namespace {

constexpr int ERR_DIAG_WAIT = 1 << 24;

__global__ void wait_timeout_kernel(int *err, uint64_t limit_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    // nothing arrives on the barrier: the bounded wait runs out, records the code and returns
    if (threadIdx.x == 0) mbar_wait_ns(&bar, 0, err, ERR_DIAG_WAIT, limit_ns);
}

}  // namespace
}  // namespace b200

using namespace b200;

extern "C" int sam3b200_debug_wait_timeout(sam3b200_backend *h, uint64_t limit_ns) {
    auto *be = reinterpret_cast<Backend *>(h);
    if (!be) {
        set_error("debug_wait_timeout: null backend");
        return SAM3B200_STATUS_FAILED;
    }
    if (limit_ns == 0 || limit_ns > 1000000000ull) {
        set_error("debug_wait_timeout: limit must be in (0, 1 s], got %llu ns", (unsigned long long)limit_ns);
        return SAM3B200_STATUS_FAILED;
    }
    if (!cuda_ok(cudaSetDevice(be->device), "cudaSetDevice")) return SAM3B200_STATUS_FAILED;
    be->count(1);
    wait_timeout_kernel<<<1, 32, 0, be->stream>>>(be->err, limit_ns);
    return cuda_ok(cudaGetLastError(), "debug_wait_timeout launch") ? SAM3B200_STATUS_SUCCESS : SAM3B200_STATUS_FAILED;
}
