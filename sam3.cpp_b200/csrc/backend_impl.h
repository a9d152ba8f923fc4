// backend_impl.h -- the objects behind the opaque handles of sam3_b200.h.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include <vector>

namespace b200 {

struct Backend {
    int device = 0;
    int num_sms = 0;
    cudaStream_t stream = nullptr;
    int *err = nullptr;  // device error word written by bounded pipeline waits
    int mmq_impl = 0;    // SAM3B200_MMQ_*
    int mmq_cvt = 0;     // MMQ epilogue int->float conversion (tuning: env SAM3B200_MMQ_CVT=0|1)
    int mmq_bn = 0;      // MMQ tile width: 0 = by K (tuning: env SAM3B200_MMQ_BN=64|128)
    int mmq_arith = 1;   // SAM3B200_ARITH_*: the encoder runners' linear-layer arithmetic (env SAM3B200_ARITH)
    char name[320] = {0};
    // scratch for the quantised activations of the current MUL_MAT
    void *act_codes = nullptr;
    size_t act_codes_bytes = 0;
    void *act_quads = nullptr;
    size_t act_quads_bytes = 0;

    bool ensure_scratch(size_t need_codes, size_t need_quads);

    // launch accounting and optional per-kernel-class event timing
    // (sam3b200_backend_profile_*): class 0 = quantised MUL_MAT
    long long launches = 0;
    int profiling = 0;
    std::vector<cudaEvent_t> prof_events[4];  // begin/end pairs per class
    size_t prof_used[4] = {0, 0, 0, 0};
    void count(int n = 1) { launches += n; }
    void prof_mark(int cls);
};

// A 2-D weight in the tensor-core layout (see mmq.cuh).
struct Weight {
    int type = 0;  // ggml_type of the uploaded blocks
    int K = 0;     // ne0
    int N = 0;     // ne1
    int ld = 0;    // scale-quad rows per block (N rounded up to 128)
    void *codes = nullptr;
    void *quads = nullptr;
    void *mins = nullptr;   // Q4_1: block minima as fp16 records [K/32][ld][8] (slot b % 8)
    void *dense = nullptr;  // F16 / F32 weights: fp16 [N][K] for the fp16 tensor-core GEMM
    void *w16 = nullptr;    // Q8_0 / Q4_0: the blocks dequantised to fp16 [N][K], made by the first mul_mat_dq16
};

void set_error(const char *fmt, ...);
bool cuda_ok(cudaError_t e, const char *what);

int run_mul_mat(Backend *be, const Weight *w, const float *x, int64_t ldx, int64_t M, const float *bias, float *dst,
                int64_t ldd, int32_t *dump);

// sam_dec.cu: a decoder mask's logits [S][S] resized to out_w x out_h (bilinear) and binarised at 0 -> 255 / 0
cudaError_t launch_mask_resize(const float *src, int S, int out_w, int out_h, uint8_t *dst, cudaStream_t s);
// mem_prompt.cu: the positional row (MD floats) shared by an object pointer's prompt tokens
void obj_ptr_pos_row(int D, int MD, int rel, const float *w, const float *b, float *out);

}  // namespace b200
