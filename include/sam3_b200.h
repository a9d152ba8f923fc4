/*
 * sam3_b200.h -- C ABI of the B200 (sm_100a) backend for sam3.cpp.
 *
 * The entry points mirror the ggml backend calls sam3.cpp makes on its hot
 * path (the ggml headers themselves live in the reference's empty ggml
 * submodule, so the ABI is stated here with plain pointers and sizes):
 *
 *   backend lifetime   ggml_backend_metal_init / ggml_backend_cpu_init
 *                      (sam3.cpp:3279-3287), ggml_backend_free (:3359-3362)
 *   device buffers     ggml_backend_alloc_ctx_tensors / ggml_backend_alloc_buffer
 *                      / ggml_backend_buffer_free (:3320, :3325)
 *   tensor data        ggml_backend_tensor_set / _get (:3156, :6119, :10930),
 *                      synchronous like ggml's
 *   weights            the per-tensor upload loop of sam3_load_tensors
 *                      (:3155-3185) for 2-D Q8_0 / Q4_0 weights
 *   compute            GGML_OP_MUL_MAT nodes of the ViT blocks
 *                      (:3742, :3783, :3796, :3799), with the bias ggml_add
 *                      that follows each of them (:3743, :3784, :3797, :3800)
 *   completion         ggml_backend_graph_compute's status (:1023-1028)
 *
 * Status codes are the values of ggml's enum ggml_status.  No call throws;
 * failures return a status or NULL and leave a message for
 * sam3b200_last_error() (sam3.cpp's own convention, CLAUDE.md "no
 * exceptions").
 */
#ifndef SAM3_B200_H
#define SAM3_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* enum ggml_status */
#define SAM3B200_STATUS_ALLOC_FAILED (-2)
#define SAM3B200_STATUS_FAILED       (-1)
#define SAM3B200_STATUS_SUCCESS      (0)
#define SAM3B200_STATUS_ABORTED      (1)

/* enum ggml_type values used by sam3.cpp weight files (sam3.cpp:3246-3255) */
#define SAM3B200_TYPE_F32  0
#define SAM3B200_TYPE_F16  1
#define SAM3B200_TYPE_Q4_0 2
#define SAM3B200_TYPE_Q4_1 3
#define SAM3B200_TYPE_Q8_0 8

/* MUL_MAT implementation selector (sam3b200_set_mmq_impl). */
#define SAM3B200_MMQ_AUTO 0 /* tensor-core kernel; SIMT for tiny M */
#define SAM3B200_MMQ_TC   1 /* tcgen05 kernel, tile 128 x 128 */
#define SAM3B200_MMQ_SIMT 2 /* one thread per output */

typedef struct sam3b200_backend sam3b200_backend;
typedef struct sam3b200_weight  sam3b200_weight;

/* Replaces ggml_backend_metal_init()/ggml_backend_cpu_init() at
 * sam3.cpp:3279-3287: one backend per (process, device).  Returns NULL if
 * the device is missing or is not sm_100. */
sam3b200_backend *sam3b200_backend_init(int device);
/* ggml_backend_free (sam3.cpp:3359-3362) */
void sam3b200_backend_free(sam3b200_backend *be);
/* ggml_backend_name */
const char *sam3b200_backend_name(const sam3b200_backend *be);
/* Waits for all work queued on the backend; returns FAILED if a kernel
 * reported an error (including a bounded pipeline wait that timed out). */
int sam3b200_backend_synchronize(sam3b200_backend *be);
/* The backend's CUDA stream (cudaStream_t), for callers that time or order
 * work against it. */
void *sam3b200_backend_stream(sam3b200_backend *be);
/* Last error message of the calling thread ("" if none). */
const char *sam3b200_last_error(void);

/* ggml_backend_alloc_buffer / ggml_backend_buffer_free (sam3.cpp:3320) */
void *sam3b200_buffer_alloc(sam3b200_backend *be, size_t size);
void sam3b200_buffer_free(sam3b200_backend *be, void *ptr);

/* ggml_backend_tensor_set / ggml_backend_tensor_get: synchronous copies
 * between host memory and device memory at ptr + offset (sam3.cpp:3156,
 * 6119, 10930). */
int sam3b200_tensor_set(sam3b200_backend *be, void *dev, const void *host, size_t offset, size_t size);
int sam3b200_tensor_get(sam3b200_backend *be, const void *dev, void *host, size_t offset, size_t size);

/* Upload one 2-D weight tensor in ggml layout: ne0 = K (contiguous, a
 * multiple of 32) by ne1 = N rows of `type` (Q8_0 or Q4_0), as
 * sam3_load_tensors does with ggml_backend_tensor_set (sam3.cpp:3155-3185).
 * The backend keeps the weight in its tensor-core layout.  NULL on error. */
sam3b200_weight *sam3b200_weight_upload(sam3b200_backend *be, int type, const void *host_blocks, int64_t ne0,
                                        int64_t ne1);
void sam3b200_weight_free(sam3b200_backend *be, sam3b200_weight *w);

/* GGML_OP_MUL_MAT (+ the bias ggml_add that follows it in every ViT GEMM):
 *   dst[m][n] = sum_k w[n][k] * x[m][k]  (+ bias[n])
 * with x quantised to Q8_0 the way ggml-cpu does, and the per-32-block
 * int32 dots scaled by the two fp16 block scales (ggml vec_dot semantics).
 * x: device f32, M rows of K floats, row stride ldx; bias: device f32 [N]
 * or NULL; dst: device f32, M rows, row stride ldd.  Asynchronous on the
 * backend stream, like a node inside ggml_backend_graph_compute. */
int sam3b200_mul_mat(sam3b200_backend *be, const sam3b200_weight *w, const float *x, int64_t ldx, int64_t M,
                     const float *bias, float *dst, int64_t ldd);

/* Parity hook: the int32 block dots the MUL_MAT path forms, for every
 * (m, n, b): dst[(m*N + n)*(K/32) + b].  Same kernel as sam3b200_mul_mat
 * with the fp32 epilogue replaced by a dump.  Synchronous. */
int sam3b200_mul_mat_block_dots(sam3b200_backend *be, const sam3b200_weight *w, const float *x, int64_t M,
                                int32_t *dst_dev);

/* Select the MUL_MAT kernel (SAM3B200_MMQ_*); returns the previous one. */
int sam3b200_set_mmq_impl(sam3b200_backend *be, int impl);

#ifdef __cplusplus
}
#endif
#endif /* SAM3_B200_H */
