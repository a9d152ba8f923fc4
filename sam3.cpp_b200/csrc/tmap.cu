// tmap.cu -- see tmap.h.
#include "tmap.h"

#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <mutex>

namespace b200 {

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

bool make_tmap(CUtensorMap *map, CUtensorMapDataType dt, const void *base, int rank, const uint64_t *dims,
               const uint64_t *strides, const uint32_t *box, CUtensorMapSwizzle sw) {
    auto fn = encode_fn();
    if (!fn || rank < 1 || rank > 3) return false;
    cuuint64_t d[3], st[2];
    cuuint32_t bx[3], es[3] = {1, 1, 1};
    for (int i = 0; i < rank; ++i) {
        d[i] = dims[i];
        bx[i] = box[i];
    }
    for (int i = 0; i < rank - 1; ++i) st[i] = strides[i];
    return fn(map, dt, rank, const_cast<void *>(base), d, st, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace b200
