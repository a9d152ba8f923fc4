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
/* Failure-path diagnostic, no counterpart in the reference (its test hooks
 * exercise stages, sam3.cpp:6218-6998): queues a one-thread kernel that waits
 * with the pipelines' bounded mbarrier wait, limited to limit_ns (at most
 * 1 s), on a barrier that nothing arrives on.  The wait runs out, the kernel
 * records an error code and returns; the next sam3b200_backend_synchronize
 * returns FAILED and the backend remains usable. */
int sam3b200_debug_wait_timeout(sam3b200_backend *be, uint64_t limit_ns);
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
/* ggml_backend_tensor_memset / ggml_backend_buffer_clear: bytes [offset, offset + size) of device
 * memory at ptr set to `value`, synchronously. */
int sam3b200_tensor_memset(sam3b200_backend *be, void *dev, int value, size_t offset, size_t size);
/* ggml_backend_dev_get_memory / ggml_backend_dev_count: free and total bytes of a GPU, GPUs visible. */
int sam3b200_device_memory(int device, size_t *free_bytes, size_t *total_bytes);
int sam3b200_device_count(int *count);

/* Upload one 2-D weight tensor in ggml layout: ne0 = K (contiguous, a
 * multiple of 32) by ne1 = N rows of `type` (Q8_0 or Q4_0), as
 * sam3_load_tensors does with ggml_backend_tensor_set (sam3.cpp:3155-3185).
 * The blocks may be in host memory or in device memory of this backend's GPU
 * (a weight already in a device buffer).  The backend keeps the weight in its
 * tensor-core layout.  NULL on error. */
sam3b200_weight *sam3b200_weight_upload(sam3b200_backend *be, int type, const void *host_blocks, int64_t ne0,
                                        int64_t ne1);
void sam3b200_weight_free(sam3b200_backend *be, sam3b200_weight *w);

/* GGML_OP_MUL_MAT (+ the bias ggml_add that follows it in every ViT GEMM):
 *   dst[m][n] = sum_k w[n][k] * x[m][k]  (+ bias[n])
 * with x quantised to Q8_0 the way ggml-cpu does, and the per-32-block
 * int32 dots scaled by the two fp16 block scales (ggml vec_dot semantics).
 * x: device f32, M rows of K floats, row stride ldx; bias: device f32 [N]
 * or NULL, 16-byte aligned (refused otherwise); dst: device f32, M rows,
 * row stride ldd.  Asynchronous on the backend stream, like a node inside
 * ggml_backend_graph_compute. */
int sam3b200_mul_mat(sam3b200_backend *be, const sam3b200_weight *w, const float *x, int64_t ldx, int64_t M,
                     const float *bias, float *dst, int64_t ldd);

/* Parity hook: the int32 block dots the MUL_MAT path forms, for every
 * (m, n, b): dst[(m*N + n)*(K/32) + b].  Same kernel as sam3b200_mul_mat
 * with the fp32 epilogue replaced by a dump.  Synchronous. */
int sam3b200_mul_mat_block_dots(sam3b200_backend *be, const sam3b200_weight *w, const float *x, int64_t M,
                                int32_t *dst_dev);

/* Kernel launches the backend has issued so far (encoder and MUL_MAT). */
long long sam3b200_backend_launch_count(const sam3b200_backend *be);

/* Per-kernel-class timing, the analogue of the reference's timed sub-graph
 * profiling helper (sam3.cpp:5041-5094): while enabled, CUDA events are
 * recorded on the backend stream around every launch of class 0 (the
 * quantised MUL_MAT) and class 1 (the tracker memory attention's attention
 * kernels); profile_read syncs and returns their summed time and count.
 * Enabling resets the record. */
int sam3b200_backend_profile(sam3b200_backend *be, int enable);
int sam3b200_backend_profile_read(sam3b200_backend *be, int cls, double *total_ms, int *n);

/* MUL_MAT that allocates nothing.  No counterpart in the reference: it is
 * for callers that cannot let the library call cudaMalloc while they
 * compute -- a framework that plans all device memory up front (as ggml's
 * graph allocator does for a backend's graph_compute) or a latency-bound
 * loop that cannot take cudaMalloc's implicit synchronisation.  Same
 * arguments and result as sam3b200_mul_mat for Q8_0 and Q4_0 weights only
 * (Q4_1, F16 and F32 weights are refused with an error); the quantised
 * activations go to a fixed 48 MiB array compiled into the library
 * (resident on every GPU that loads it, until the process exits) instead of
 * backend scratch.  Shapes whose scratch (M*K bytes of codes, rounded up to
 * 256, + ceil(K/256) * roundup(M,128) * 16 bytes of scale records) exceeds
 * 48 MiB are rejected with an error message.  The kernel choice
 * follows sam3b200_set_mmq_impl as for sam3b200_mul_mat.  The first call on
 * a device looks up the array's device address; make that first call before
 * any stream capture, and do not cudaDeviceReset the device after it.  All
 * calls on a device share the array: calls that overlap on the GPU race and
 * must be serialised by the caller.  Asynchronous on the backend stream. */
int sam3b200_mul_mat_noalloc(sam3b200_backend *be, const sam3b200_weight *w, const float *x, int64_t ldx, int64_t M,
                             const float *bias, float *dst, int64_t ldd);

/* Select the MUL_MAT kernel (SAM3B200_MMQ_*); returns the previous one. */
int sam3b200_set_mmq_impl(sam3b200_backend *be, int impl);

/* Arithmetic of the quantised linear layers inside the model-level encoder
 * runners (sam3b200_vit_*: the ViT blocks of sam3_vit_block_forward,
 * sam3.cpp:3742,3783,3796,3799).  Both quantise the activations to Q8_0 with
 * ggml-cpu's rule (the same codes and scales):
 *   SAM3B200_ARITH_EXACT: int8 tcgen05 block dots (bit-exact with ggml's
 *     int32 block dots) folded block by block in fp32 on the CUDA cores;
 *   SAM3B200_ARITH_DQ16 (default): activation codes and weight blocks
 *     dequantised to fp16 (fp16(q * d), one rounding of the exact product)
 *     and multiplied on the fp16 tensor cores with fp32 accumulation over
 *     all of K -- the same sum up to rounding (~3e-4 normwise), without the
 *     per-block fold; the weights are held a second time as fp16.
 * Op-level sam3b200_mul_mat is always EXACT.  Returns the previous value;
 * other values are ignored.  Environment: SAM3B200_ARITH=0|1 at init. */
#define SAM3B200_ARITH_EXACT 0
#define SAM3B200_ARITH_DQ16  1
int sam3b200_set_arith(sam3b200_backend *be, int arith);

/* GGML_OP_MUL_MAT (sam3.cpp:3742,3783,3796,3799) in the DQ16 arithmetic of
 * sam3b200_set_arith: x quantised to Q8_0 (ggml-cpu's rule), codes and
 * weight blocks dequantised to fp16, fp16 tensor-core GEMM with fp32
 * accumulation, + bias.  Same arguments as sam3b200_mul_mat; Q8_0 and Q4_0
 * weights only (others are refused with an error).  The first call with a
 * weight makes its fp16 copy (N*K*2 bytes, freed with the weight); scratch
 * is the backend's, as for sam3b200_mul_mat.  Asynchronous on the backend
 * stream. */
int sam3b200_mul_mat_dq16(sam3b200_backend *be, const sam3b200_weight *w, const float *x, int64_t ldx, int64_t M,
                          const float *bias, float *dst, int64_t ldd);

/* GGML_OP_FLASH_ATTN_EXT as the ViT blocks use it (sam3.cpp:3778: no mask,
 * max_bias 0, logit softcap 0): dst = softmax(q k^T * scale) v per (head,
 * batch).  q, k, v: device f32 ggml tensors [D, N, heads, batch], contiguous
 * (memory [batch][heads][N][D]); dst: device f32 [D, heads, N, batch]
 * (memory [batch][N][heads][D]), the layout ggml_flash_attn_ext returns.
 * D == 64 with N a multiple of 8 runs on the tensor cores (bf16 q, k, v,
 * fp32 softmax and accumulation: within 1e-2 of the f32 reference); the other
 * head dimensions of sam3b200_flash_attn_ext_view run in fp32.  Asynchronous
 * on the backend stream. */
int sam3b200_flash_attn_ext(sam3b200_backend *be, const float *q, const float *k, const float *v, int64_t D,
                            int64_t N, int64_t heads, int64_t batch, float scale, float *dst);

/* GGML_OP_FLASH_ATTN_EXT in the general form sam3.cpp builds (max_bias 0,
 * softcap 0): q [D, NQ, heads, batch], k and v [D, NKV, heads, batch] given by
 * their ggml strides in ELEMENTS, nb[0..2] = (nb1, nb2, nb3) / sizeof(float)
 * (token, head, batch; the D elements of one token are contiguous) -- so the
 * permuted V view of sam3.cpp:3767 is passed as it is; mask_f16: NULL or the
 * F16 mask [NKV, >= NQ] with row stride mask_nb1 elements, added to every
 * head's scores (the text encoder's causal mask, sam3.cpp:3934-3951); a -inf
 * entry removes the key, a row with every key removed yields zeros.  dst: f32
 * [D, heads, NQ, batch] contiguous.  D in {16, 32, 48, 56, 64, 72, 96, 112,
 * 128, 256}.  Contiguous unmasked self-attention with D == 64 and NQ a
 * multiple of 8 (q, k, v 8-byte and dst 16-byte aligned) takes the
 * tensor-core path; every other form runs in fp32 on the CUDA cores.
 * Asynchronous on the backend stream. */
int sam3b200_flash_attn_ext_view(sam3b200_backend *be, const float *q, const float *k, const float *v,
                                 const void *mask_f16, int64_t mask_nb1, int64_t D, int64_t NQ, int64_t NKV,
                                 int64_t heads, int64_t batch, const int64_t q_nb[3], const int64_t k_nb[3],
                                 const int64_t v_nb[3], float scale, float *dst);

/* GGML_OP_CONV_TRANSPOSE_2D as ggml_conv_transpose_2d_p0 builds it
 * (sam3.cpp:3884,3887,3898 neck; :10654,10673 mask decoder): no padding, any
 * stride.  w: device ggml F16 kernel [KW, KH, OC, IC] (memory
 * [ic][oc][ky][kx]); x: device f32 [IW, IH, IC, 1] (memory [ic][iy][ix]);
 * dst: device f32 [OW, OH, OC, 1], OW = (IW-1)*stride + KW, OH likewise.
 * x is rounded to fp16 as ggml's CPU path does; products are summed in fp32
 * on the tensor cores.  Asynchronous on the backend stream (allocates its
 * scratch from the stream-ordered pool). */
int sam3b200_conv_transpose_2d(sam3b200_backend *be, const void *w_f16, const float *x, int64_t iw, int64_t ih,
                               int64_t ic, int64_t oc, int64_t kw, int64_t kh, int stride, float *dst);

/* GGML_OP_CONV_2D: ggml_conv_2d(kernel, input, s0, s1, p0, p1, d0, d1) and its
 * _sk_p0 / _s1_ph forms (sam3.cpp:3819 patch embedding, :3889-3921 neck,
 * :4474 Hiera patch embedding, :11541 memory-encoder downsampling).
 * w: device ggml F16 kernel [KW, KH, IC, OC] (memory [oc][ic][ky][kx]);
 * x: device f32 [IW, IH, IC, 1]; dst: device f32 [OW, OH, OC, 1] with
 * OW = (IW + 2*p0 - d0*(KW-1) - 1)/s0 + 1 (OH likewise).  im2col in fp16 as
 * ggml's CPU path, fp32 accumulation on the tensor cores.  Asynchronous. */
int sam3b200_conv_2d(sam3b200_backend *be, const void *w_f16, const float *x, int64_t iw, int64_t ih, int64_t ic,
                     int64_t oc, int64_t kw, int64_t kh, int s0, int s1, int p0, int p1, int d0, int d1, float *dst);

/* GGML_OP_GET_ROWS (ggml_get_rows: the text encoder's token-embedding
 * lookup, sam3.cpp:3927-4068): dst[i][:] = row idx[i] of src, dequantised to
 * f32 by ggml's rules (F32, F16, Q4_0, Q4_1, Q8_0).  src: device rows of
 * ncols elements in the ggml block format of `type`; idx: device int32 [n];
 * dst: device f32 [n][ncols].  An index outside [0, nrows) yields a zero row
 * and makes the next sam3b200_backend_synchronize fail.  Asynchronous. */
int sam3b200_get_rows(sam3b200_backend *be, int type, const void *src, int64_t ncols, int64_t nrows,
                      const int32_t *idx, int64_t n, float *dst);

/* ---- Graph level: the backend's supports_op and graph_compute -------------
 * ggml_backend_graph_compute (sam3.cpp:1023-1028) hands a backend the nodes
 * of one graph in execution order; ggml's scheduler first asks the backend's
 * supports_op which nodes it may take.  sam3b200_tensor is a ggml graph node
 * flattened to plain C: the fields of struct ggml_tensor a backend reads to
 * execute a node (type, ne, nb in bytes, op, op_params, flags, src, data,
 * extra).  A ggml shim copies each node into one of these; enum ggml_op
 * differs between ggml versions, so ops have this ABI's own codes. */
#define SAM3B200_TYPE_I32 26 /* enum ggml_type GGML_TYPE_I32: GET_ROWS indices */

#define SAM3B200_OP_NONE              0 /* leaf: data already on the device */
#define SAM3B200_OP_VIEW              1 /* VIEW / RESHAPE / PERMUTE / TRANSPOSE: data aliases src[0], nothing runs */
#define SAM3B200_OP_MUL_MAT           2 /* ggml_mul_mat(src0 = weight, src1 = x); src0 either an uploaded weight
                                           (extra) or an F32 / F16 tensor of the graph (the IM2COL result of
                                           ggml_conv_2d), src1 then F32 or F16 */
#define SAM3B200_OP_ADD               3 /* ggml_add, src1 broadcast (ggml_can_repeat); fused into the MUL_MAT before it when it is that MUL_MAT's bias */
#define SAM3B200_OP_FLASH_ATTN_EXT    4 /* ggml_flash_attn_ext(q, k, v, mask), op_params[0..2] = scale, max_bias, softcap */
#define SAM3B200_OP_CONV_TRANSPOSE_2D 5 /* ggml_conv_transpose_2d_p0(kernel, x), op_params[0] = stride */
#define SAM3B200_OP_CONV_2D           6 /* ggml_conv_2d_direct(kernel, x), op_params = s0, s1, p0, p1, d0, d1 */
#define SAM3B200_OP_GET_ROWS          7 /* ggml_get_rows(rows, I32 indices) */
#define SAM3B200_OP_CONT              8 /* ggml_cont / ggml_cpy / ggml_cont_Nd / ggml_cast: element i of src0 -> element i of
                                           dst, each in its own order; F32 <-> F16 converts (round to nearest even) */
#define SAM3B200_OP_MUL               9 /* ggml_mul, src1 broadcast */
#define SAM3B200_OP_SCALE            10 /* ggml_scale, op_params[0] = s */
#define SAM3B200_OP_UNARY            11 /* op_params[0] = SAM3B200_UNARY_* */
#define SAM3B200_OP_NORM             12 /* ggml_norm over ne0 (double sums), op_params[0] = eps */
#define SAM3B200_OP_SOFT_MAX         13 /* ggml_soft_max_ext(a, mask, scale, max_bias 0) over ne0; mask F16 / F32 or none */
#define SAM3B200_OP_WIN_PART         14 /* ggml_win_part(a, w): op_params = npx, npy, w (sam3.cpp:3734) */
#define SAM3B200_OP_WIN_UNPART       15 /* ggml_win_unpart(a, W, H, w): op_params[0] = w (sam3.cpp:3788) */
#define SAM3B200_OP_SUB              16 /* ggml_sub, src1 broadcast (RoPE, sam3.cpp:3704) */
#define SAM3B200_OP_REPEAT           17 /* ggml_repeat(src0, shape of the result): element i = src0[i mod src0.ne] (sam3.cpp:3825) */
#define SAM3B200_OP_CONCAT           18 /* ggml_concat(src0, src1, dim): op_params[0] = dim (sam3.cpp:3708) */
#define SAM3B200_OP_IM2COL           19 /* ggml_im2col(kernel, x, ...): op_params = s0, s1, p0, p1, d0, d1, is_2D; result
                                           [IC*KH*KW, OW, OH, N] F32 or F16 (ggml_conv_2d, sam3.cpp:3819) */
#define SAM3B200_OP_POOL_2D          20 /* ggml_pool_2d: op_params = op (0 max, 1 avg), k0, k1, s0, s1, p0, p1 (sam3.cpp:3918) */
#define SAM3B200_OP_PAD              21 /* ggml_pad / ggml_pad_ext: op_params = lp0, rp0, lp1, rp1, lp2, rp2, lp3, rp3, zeros
                                           (sam3.cpp:4210) */
#define SAM3B200_OP_UPSCALE          22 /* ggml_upscale nearest: op_params[0] = mode 0; factors = result ne / src ne (sam3.cpp:4586) */
#define SAM3B200_OP_CONV_2D_DW       23 /* ggml_conv_2d_dw_direct(kernel [KW, KH, 1, C], x [W, H, C, N]): op_params = s0, s1,
                                           p0, p1, d0, d1 (sam3.cpp:9089) */
#define SAM3B200_OP_GROUP_NORM       24 /* ggml_group_norm over ne0 x ne1 x (ne2 / groups): op_params[0] = groups,
                                           op_params[1] = eps (sam3.cpp:8923) */

#define SAM3B200_UNARY_RELU     1
#define SAM3B200_UNARY_SIGMOID  2
#define SAM3B200_UNARY_GELU_ERF 3 /* ggml_gelu_erf */
#define SAM3B200_UNARY_GELU     4 /* ggml_gelu as the CPU backend evaluates it (fp16 table of the tanh form) */

#define SAM3B200_TENSOR_FLAG_OUTPUT 2 /* GGML_TENSOR_FLAG_OUTPUT: the caller reads this node */

typedef struct sam3b200_tensor {
    int32_t type;          /* ggml_type value (SAM3B200_TYPE_*) */
    int32_t op;            /* SAM3B200_OP_* */
    int64_t ne[4];         /* elements per dimension, ne[0] innermost */
    size_t nb[4];          /* strides in bytes, as ggml's nb */
    int32_t op_params[16]; /* ggml op_params words (floats by their bits) */
    int32_t flags;         /* SAM3B200_TENSOR_FLAG_* */
    const struct sam3b200_tensor *src[4];
    void *data;            /* device address */
    void *extra;           /* MUL_MAT src0: the sam3b200_weight from sam3b200_weight_upload */
} sam3b200_tensor;

/* ggml_backend supports_op: 1 if this backend executes `node` as it stands
 * (op, types, shapes and strides), 0 if not -- there is no CPU fallback, so a
 * node reported 0 must go to another backend.  Pure host code: needs no
 * device and launches nothing. */
int sam3b200_supports_op(const sam3b200_tensor *node);

/* ggml_backend graph_compute: run nodes[0..n_nodes) in order on the backend
 * stream and wait for them, returning the ggml_status.  Every node is checked
 * first (sam3b200_supports_op, then the graph rules: a MUL_MAT's weight is an
 * uploaded handle of matching shape; data aligned -- 16 bytes for MUL_MAT,
 * FLASH_ATTN_EXT, the convolutions and GET_ROWS, one element for the
 * elementwise ops and NORM); if any node is rejected nothing is launched and
 * the message names the node.  An ADD of a packed [N] vector right after the
 * MUL_MAT it reads, when nothing else reads that MUL_MAT and it is not
 * flagged OUTPUT, runs inside the MUL_MAT as its bias (same result bits as
 * the unfused pair).  The checks come before the backend is touched, so a
 * NULL backend reports a rejected graph's own error first. */
int sam3b200_graph_compute(sam3b200_backend *be, sam3b200_tensor *const *nodes, int n_nodes);

/* ---- SAM2 Hiera image encoder (config 1: Hiera trunk + FPN neck) ----------
 * The graph sam2_build_hiera_graph + sam2_build_fpn_neck_graph build
 * (sam3.cpp:4467-4583), per-block metadata as sam2_precompute_hiera_metadata
 * (sam3.cpp:1680-1740).  Weights by their weight-file names
 * (sam3.cpp:1800-1851): "hiera.patch_embed.{weight,bias}", "hiera.pos_embed",
 * "hiera.pos_embed_window", "hiera.blocks.<i>.{norm1,norm2}.{weight,bias}",
 * "...attn.qkv.{weight,bias}", "...attn.proj.{weight,bias}",
 * "...mlp.fc1/fc2.{weight,bias}", "...proj.{weight,bias}" (stage
 * transitions), "fpn.convs.<j>.{weight,bias}".  Linear weights Q8_0/Q4_0,
 * convolution and norm tensors F32/F16. */
typedef struct {
    int32_t img;                     /* input side, 1024 */
    int32_t embed;                   /* hiera_embed_dim */
    int32_t heads;                   /* hiera_num_heads */
    int32_t stages[4];
    int32_t q_pool;
    int32_t window_spec[4];
    int32_t n_global;
    int32_t global_idx[8];
    int32_t bkg_h, bkg_w;            /* hiera.pos_embed grid */
    int32_t neck_dim;                /* 256 */
    int32_t fpn_top_down_n;
    int32_t fpn_top_down_levels[4];
    int32_t scalp;
} sam3b200_hiera_hparams;

typedef struct sam3b200_hiera sam3b200_hiera;

sam3b200_hiera *sam3b200_hiera_create(sam3b200_backend *be, const sam3b200_hiera_hparams *hp);
void sam3b200_hiera_free(sam3b200_hiera *h);
int sam3b200_hiera_set_tensor(sam3b200_hiera *h, const char *name, int type, const void *data, const int64_t ne[4]);
/* Number of tensors still missing; their names, newline-separated, into buf. */
int sam3b200_hiera_missing(sam3b200_hiera *h, char *buf, int cap);
/* Block i's metadata: dim_in, dim_out, heads, window size (0 = global), Q stride. */
int sam3b200_hiera_block_info(sam3b200_hiera *h, int i, int32_t info[5]);
/* Stage runners (device pointers, asynchronous): patch embedding + positional
 * embedding, image f32 CHW [3][img][img] -> x [S*S][embed] (S = img/4); one
 * block, x [H*W][dim_in] -> out [H'*W'][dim_out] (H' = H/2 at a Q-stride
 * block; out may equal x otherwise). */
int sam3b200_hiera_run_prefix(sam3b200_hiera *h, const float *img_chw_dev, float *x_dev);
int sam3b200_hiera_run_block(sam3b200_hiera *h, int i, const float *x_dev, int H, int W, float *out_dev);
/* Whole encoder from a preprocessed image (sam3b200_preprocess_sam2 output). */
int sam3b200_hiera_encode_device(sam3b200_hiera *h, const float *img_chw_dev);
/* Outputs: i = 0..3 FPN levels [neck_dim, W, H, 1] (levels >= 4 - scalp fail),
 * i = 4..7 stage outputs [dim, W, H, 1]; token-major device f32. */
int sam3b200_hiera_output(sam3b200_hiera *h, int i, const float **dev, int64_t ne[4]);

/* ---- SAM prompt encoder + mask decoder (PVS, sam3_segment_pvs) -----------
 * The graph of sam3.cpp:10765-11115 (decoder sam3_build_sam_dec_graph
 * :10548-10763) on the B200.  Inputs are the encoder's three finest maps in
 * token-major device f32: image features [H*H][256] (neck / FPN level 2),
 * feat_s0 [(4H)^2][256] and feat_s1 [(2H)^2][256] (levels 0 and 1).  Weights
 * by their weight-file names (sam3.cpp:1854-1968): "sam_pe.*", "sam_dec.*",
 * "no_mem_embed". */
typedef struct {
    int32_t feat_size;        /* H: 64 for SAM2 at 1024, 72 for SAM3 at 1008 */
    int32_t embed;            /* 256 */
    int32_t depth;            /* two-way blocks, 2 */
    int32_t heads;            /* 8 */
    int32_t mlp_dim;          /* 2048 */
    int32_t n_multimask;      /* 3: four mask tokens */
    int32_t pred_obj_scores;  /* 1: object-score token and head */
    int32_t max_points;       /* prompt token capacity including the padding token (<= 64) */
} sam3b200_sam_dec_hparams;

typedef struct sam3b200_sam_dec sam3b200_sam_dec;

sam3b200_sam_dec *sam3b200_sam_dec_create(sam3b200_backend *be, const sam3b200_sam_dec_hparams *hp);
void sam3b200_sam_dec_free(sam3b200_sam_dec *d);
int sam3b200_sam_dec_set_tensor(sam3b200_sam_dec *d, const char *name, int type, const void *data,
                                const int64_t ne[4]);
int sam3b200_sam_dec_missing(sam3b200_sam_dec *d, char *buf, int cap);
/* One PVS decode: prompts in original-image pixels (coords x, y pairs; labels
 * 1 positive, 0 negative, 2 / 3 box corners, in the reference's order: box
 * corners, positive, negative; the padding token is appended here),
 * orig_w x orig_h the original image, img_size the encoder input side.
 * Synchronous (reads back the IoU and object scores). */
int sam3b200_sam_dec_run(sam3b200_sam_dec *d, const float *img_feats_dev, const float *feat_s0_dev,
                         const float *feat_s1_dev, const float *coords, const int32_t *labels, int n_prompts,
                         int orig_w, int orig_h, int img_size);
/* The decode of a propagated video frame (sam3_propagate_single,
 * sam3.cpp:11312-11347): the memory-conditioned features [H*H][256] (the
 * memory attention's output) without no_mem_embed, no user prompt -- the
 * single not_a_point padding token -- and the same high-resolution maps.
 * Synchronous like sam3b200_sam_dec_run. */
int sam3b200_sam_dec_run_tracking(sam3b200_sam_dec *d, const float *cond_feats_dev, const float *feat_s0_dev,
                                  const float *feat_s1_dev);
/* Output token of mask m (0 .. n_multimask) of the last run, device [256]:
 * the decoder's mask_tokens output (token 0 is the SAM output token). */
int sam3b200_sam_dec_mask_token(sam3b200_sam_dec *d, int m, const float **dev);
/* Results of the last run: mask logits [n_multimask + 1][(4H)^2] (device),
 * IoU predictions, object-score logit, SAM output token [256] (device). */
int sam3b200_sam_dec_outputs(sam3b200_sam_dec *d, const float **masks_dev, float iou[4], float *obj_logit,
                             const float **sam_token_dev);
/* Mask m resized to out_w x out_h (bilinear, sam3.cpp:9617-9643) and
 * binarised at logit 0 (:11071-11075): dst_dev uint8 [out_h][out_w], 255 / 0. */
int sam3b200_sam_dec_mask(sam3b200_sam_dec *d, int m, int out_w, int out_h, uint8_t *dst_dev);

/* ---- SAM3 text encoder (the PCS path's text side) ------------------------
 * The graph sam3_build_text_encoder_graph builds (sam3.cpp:4039-4066; block
 * :3958-4032; causal mask :3934-3951): token embedding rows + positional
 * embedding, `layers` pre-LN blocks (16-head causal attention, GELU-erf MLP),
 * final LayerNorm, resizer to out_dim.  Weights by name (sam3.cpp:2628-2654):
 * "text.token_embed.weight", "text.pos_embed", "text.ln_final.*",
 * "text.resizer.*", "text.blocks.<i>.{attn.in_proj,attn.out_proj,ln_1,ln_2,
 * mlp.fc1,mlp.fc2}.{weight,bias}". */
typedef struct {
    int32_t width;    /* 1024 */
    int32_t heads;    /* 16 (head dim 64) */
    int32_t layers;   /* 24 */
    int32_t ctx_len;  /* 32 */
    int32_t vocab;    /* 49408 */
    int32_t out_dim;  /* 256 */
} sam3b200_text_hparams;

typedef struct sam3b200_text sam3b200_text;

sam3b200_text *sam3b200_text_create(sam3b200_backend *be, const sam3b200_text_hparams *hp);
void sam3b200_text_free(sam3b200_text *t);
int sam3b200_text_set_tensor(sam3b200_text *t, const char *name, int type, const void *data, const int64_t ne[4]);
int sam3b200_text_missing(sam3b200_text *t, char *buf, int cap);
/* Encode n_ids (<= ctx_len) host token ids, padded with id 0 to ctx_len as
 * the reference does.  Asynchronous after the id upload. */
int sam3b200_text_encode(sam3b200_text *t, const int32_t *ids, int n_ids);
/* Text features: device f32 [out_dim, ctx_len] (memory [ctx_len][out_dim]). */
int sam3b200_text_output(sam3b200_text *t, const float **dev, int64_t ne[2]);

/* ---- Memory attention of the video tracker -------------------------------
 * The graph sam3_build_mem_attn_graph builds (sam3.cpp:9228-9341) with the
 * inputs sam3_propagate_single prepares (:11175-11310): current-frame tokens
 * conditioned on the memory bank through `layers` blocks of single-head
 * self-attention (RoPE on q and k), cross-attention to the memories (keys
 * from prompt + prompt_pos, values from prompt, both projected mem_dim ->
 * d_model; RoPE on q and on the first M_total - n_obj_ptr_tokens keys only),
 * ReLU feed-forward, then LayerNorm.  Weights by name (sam3.cpp:2008-2042):
 * "mem_attn.norm.{weight,bias}", "mem_attn.layers.<i>.{sa,ca}.{q,k,v,out}_proj
 * .{weight,bias}", ".linear1", ".linear2", ".norm1".."norm3". */
typedef struct {
    int32_t d_model;         /* 256 (neck_dim; the single head's width) */
    int32_t mem_dim;         /* 64 (mem_out_dim) */
    int32_t layers;          /* 4 */
    int32_t ffn_dim;         /* 2048 */
    int32_t max_tokens;      /* capacity: current-frame tokens N (H*H) */
    int32_t max_mem_tokens;  /* capacity: memory tokens M_total (spatial + object-pointer) */
} sam3b200_mem_attn_hparams;

typedef struct sam3b200_mem_attn sam3b200_mem_attn;

sam3b200_mem_attn *sam3b200_mem_attn_create(sam3b200_backend *be, const sam3b200_mem_attn_hparams *hp);
void sam3b200_mem_attn_free(sam3b200_mem_attn *m);
int sam3b200_mem_attn_set_tensor(sam3b200_mem_attn *m, const char *name, int type, const void *data,
                                 const int64_t ne[4]);
int sam3b200_mem_attn_missing(sam3b200_mem_attn *m, char *buf, int cap);
/* Host inputs (the tensors sam3_propagate_single sets), ggml layouts:
 * curr, src_pos [d_model, N]; prompt, prompt_pos [mem_dim, M_total];
 * rope_q [2, d_model/2, N]; rope_k [2, d_model/2, M_total - n_obj_ptr_tokens]
 * or NULL (no rotation of the keys).  Asynchronous after the uploads. */
int sam3b200_mem_attn_run(sam3b200_mem_attn *m, const float *curr, const float *src_pos, const float *prompt,
                          const float *prompt_pos, const float *rope_q, const float *rope_k, int n_tokens,
                          int n_mem_tokens, int n_obj_ptr_tokens);
/* The same with every input already in device memory. */
int sam3b200_mem_attn_run_device(sam3b200_mem_attn *m, const float *curr, const float *src_pos,
                                 const float *prompt, const float *prompt_pos, const float *rope_q,
                                 const float *rope_k, int n_tokens, int n_mem_tokens, int n_obj_ptr_tokens);
/* Conditioned tokens: device f32 [d_model, N] of the last run. */
int sam3b200_mem_attn_output(sam3b200_mem_attn *m, const float **dev);

/* Host-side preparation of the memory attention's inputs for one propagated
 * frame, as sam3_propagate_single does it before it builds its graph
 * (sam3.cpp:11175-11233).  No device work.
 *
 * sam3_select_memory_frames (sam3.cpp:9427-9451): the memory-bank slots that
 * take part -- all of them when there are at most max_slots, else the first,
 * the newest and evenly spaced ones between -- sorted, written to out[cap];
 * returns the count or -1. */
int sam3b200_select_memory_frames(int bank_size, int max_slots, int32_t *out, int cap);

typedef struct {
    int32_t d_model;      /* D: 256 (the object-pointer width) */
    int32_t mem_dim;      /* MD: 64 (memory feature width, prompt row width) */
    int32_t num_maskmem;  /* 7: rows of the temporal code table */
    int32_t max_obj_ptrs; /* 16: pointers taken from the pointer bank */
} sam3b200_mem_prompt_hparams;

/* sam3_build_prompt_and_pos (sam3.cpp:9126-9217) with the temporal positions
 * of sam3_propagate_single: prompt and prompt_pos rows of MD floats --
 * n_slots * slot_tokens spatial memory tokens (features as given; positional
 * code = the slot's spatial code + mem_enc.tpos_enc row num_maskmem - t - 1,
 * t = 0 for a conditioning slot and n_slots - s otherwise, no temporal code
 * for t >= num_maskmem), then D / MD tokens per object pointer for the first
 * min(n_ptrs, max_obj_ptrs) pointers (positional code: the 1-D sine code of
 * max(1, |cur_frame - ptr_frames[p]|) / 15 through obj_ptr_tpos_proj,
 * weight [D, MD] in ggml layout + bias [MD]).  The slots are the selected
 * ones, in the order of sam3b200_select_memory_frames.  NULL tpos_enc /
 * tpos_proj_w / tpos_proj_b act as zeros (a model without them).  Returns the
 * prompt token count M_total and the pointer-token count, or -1 (too many
 * tokens for cap_tokens, null inputs). */
int64_t sam3b200_build_mem_prompt(const sam3b200_mem_prompt_hparams *hp, int n_slots, int slot_tokens,
                                  const float *const *slot_feats, const float *const *slot_pes,
                                  const int32_t *slot_is_cond, int n_ptrs, const float *const *obj_ptrs,
                                  const int32_t *ptr_frames, int cur_frame, const float *tpos_enc,
                                  const float *tpos_proj_w, const float *tpos_proj_b, float *prompt,
                                  float *prompt_pos, int64_t cap_tokens, int32_t *n_ptr_tokens);

/* sam3_extract_obj_ptr_cpu (sam3.cpp:9347-9420): the object pointer of a
 * decoded frame -- the SAM output token (sam3b200_sam_dec_outputs) through
 * obj_ptr_proj (three d_model x d_model layers, ReLU after the first two;
 * w[j] f32 [out][in], b[j] f32 [out]), or no_obj_ptr when the object-score
 * logit is <= 0.  blend != 0 is the SAM2 / EdgeTAM fixed_no_obj_ptr rule:
 * l * mlp + (1 - l) * no_obj_ptr with l = [obj_score > 0].  Host code. */
int sam3b200_extract_obj_ptr(int d_model, int blend, const float *sam_token, float obj_score,
                             const float *const *w, const float *const *b, const float *no_obj_ptr, float *out);

/* sam3_sinusoidal_pe_2d (sam3.cpp:3601-3637): the 2-D sine code of an H x W
 * map, out [H][W][d_model] (channels [0, d/2) from y, [d/2, d) from x). */
int sam3b200_sinusoidal_pe_2d(int H, int W, int d_model, float *out);

/* The memory of one tracked object in one stream (sam3_tracker's mem_banks /
 * ptr_banks, sam3.cpp:951-990), host side.  add_slot stores the features the
 * memory encoder produced for a frame ([H*H][MD], sam3b200_mem_enc_output
 * copied back) with the H x H sine code, keeping at most num_maskmem slots by
 * dropping the oldest non-conditioning slot (else slot 1) as
 * sam3_encode_memory does (:11700-11711); add_ptr keeps the newest
 * max_obj_ptrs object pointers (sam3_store_obj_ptr, :11716-11734); prompt
 * selects the slots and builds the memory attention's prompt for cur_frame
 * as sam3_propagate_single does (sam3b200_select_memory_frames +
 * sam3b200_build_mem_prompt).  state reports the slot frames / flags and the
 * pointer frames; returns the slot count. */
typedef struct sam3b200_mem_bank sam3b200_mem_bank;
sam3b200_mem_bank *sam3b200_mem_bank_create(const sam3b200_mem_prompt_hparams *hp, int feat_size);
void sam3b200_mem_bank_free(sam3b200_mem_bank *b);
int sam3b200_mem_bank_add_slot(sam3b200_mem_bank *b, const float *feats, int frame, int is_cond);
int sam3b200_mem_bank_add_ptr(sam3b200_mem_bank *b, const float *ptr, int frame);
int sam3b200_mem_bank_state(const sam3b200_mem_bank *b, int32_t *slot_frames, int32_t *slot_cond, int slot_cap,
                            int32_t *ptr_frames, int ptr_cap, int32_t *n_ptrs);
int64_t sam3b200_mem_bank_prompt(const sam3b200_mem_bank *b, int cur_frame, const float *tpos_enc,
                                 const float *tpos_proj_w, const float *tpos_proj_b, float *prompt,
                                 float *prompt_pos, int64_t cap_tokens, int32_t *n_ptr_tokens);

/* sam3_compute_axial_cis (sam3.cpp:3559-3590): the 2-D RoPE table of an
 * end_x x end_y map, out [N][dim/2][2] (cos, sin; x frequencies then y). */
int sam3b200_axial_cis(int dim, int end_x, int end_y, float theta, float scale_pos, float *out);
/* The memory attention's rope_q ([H*H][d_model/2][2]) and rope_k (rope_q once
 * per slot the bank's prompt selects, cap_k_tokens rows of room) as
 * sam3_propagate_single builds them (:11240-11275); returns the rope_k row
 * count (0 when the bank is empty) or -1. */
int64_t sam3b200_mem_bank_rope(const sam3b200_mem_bank *b, float *rope_q, float *rope_k, int64_t cap_k_tokens);

/* ---- Memory encoder of the video tracker ----------------------------------
 * sam3_encode_memory (sam3.cpp:11510-11615) up to the stored [mem_dim, H, H]
 * memory features: mask logits resized to img (bilinear), sigmoid * scale +
 * bias, resized to 16H; mask downsampler (4 x conv 3x3 s2 + LayerNorm2d +
 * GELU, conv 1x1); + conv 1x1 of the frame's pixel features; 2 CXBlock
 * fusers (sam3_cxblock_forward, :9066-9108); conv 1x1 to mem_dim; plus
 * no_obj_embed_spatial when the object score is <= 0.  Weights by name
 * (sam3.cpp:1972-2005): "mem_enc.ds.{0,3,6,9,12}.*" (convolutions),
 * "mem_enc.ds.{1,4,7,10}.*" (LayerNorm2d), "mem_enc.pix_feat_proj.*",
 * "mem_enc.fuser.<i>.{dwconv,norm,pwconv1,pwconv2}.*", ".gamma",
 * "mem_enc.out_proj.*", optional "no_obj_embed_spatial"; "mem_enc.tpos_enc"
 * is accepted and left to the host prompt builder. */
typedef struct {
    int32_t feat;          /* H: 64 (SAM2 at 1024), 72 (SAM3 at 1008) */
    int32_t img;           /* the effective image size (HIGH_RES): 1024 / 1008 */
    int32_t d_model;       /* 256 */
    int32_t mem_dim;       /* 64 */
    int32_t fuser_layers;  /* 2 */
    int32_t fuser_dim;     /* 1024 */
    float sigmoid_scale;   /* sigmoid_scale_x100 / 100 (20.0) */
    float sigmoid_bias;    /* sigmoid_bias_x100 / 100 (-10.0) */
    int32_t max_mask;      /* capacity: mask_w * mask_h of the logits */
} sam3b200_mem_enc_hparams;

typedef struct sam3b200_mem_enc sam3b200_mem_enc;

sam3b200_mem_enc *sam3b200_mem_enc_create(sam3b200_backend *be, const sam3b200_mem_enc_hparams *hp);
void sam3b200_mem_enc_free(sam3b200_mem_enc *m);
int sam3b200_mem_enc_set_tensor(sam3b200_mem_enc *m, const char *name, int type, const void *data,
                                const int64_t ne[4]);
int sam3b200_mem_enc_missing(sam3b200_mem_enc *m, char *buf, int cap);
/* Host inputs: mask logits [mask_h][mask_w] (the decoder's low-resolution
 * mask), pixel features [d_model, H, H] (memory [H*H][d_model], the tracker
 * neck's level-2 map).  Asynchronous after the uploads. */
int sam3b200_mem_enc_run(sam3b200_mem_enc *m, const float *mask_logits, int mask_w, int mask_h,
                         const float *pix_feat, float obj_score);
/* The same with both inputs in device memory. */
int sam3b200_mem_enc_run_device(sam3b200_mem_enc *m, const float *mask_logits, int mask_w, int mask_h,
                                const float *pix_feat, float obj_score);
/* Memory features: device f32 [mem_dim, H, H] (memory [H*H][mem_dim]). */
int sam3b200_mem_enc_output(sam3b200_mem_enc *m, const float **dev);

/* ---- Video tracker frame loop (visual-only models) ------------------------
 * sam3_create_visual_tracker / sam3_tracker_add_instance /
 * sam3_propagate_frame (sam3.cpp:12017-12262) on the device, over the
 * runners above (all four created on `be`): per frame the Hiera encode, then
 * per tracked instance the memory prompt from its device-resident bank, the
 * memory attention, the decoder on the conditioned features, the kept mask,
 * the memory encoder (-> a new bank slot) and the object pointer (-> the
 * pointer bank).  Weights by name (sam3.cpp:2046-2060):
 * "obj_ptr_proj.layers.{0,1,2}.{weight,bias}", "no_obj_ptr",
 * "obj_ptr_tpos_proj.{weight,bias}" (optional), "mem_enc.tpos_enc"
 * (optional); F32 or F16.  The host post-processing of sam3_propagate_frame
 * (hole filling, sprinkle removal, overlap resolution) is not part of it. */
typedef struct {
    int32_t feat;             /* H: 64 (SAM2 at 1024) */
    int32_t img;              /* encoder input side: 1024 */
    int32_t d_model;          /* 256 */
    int32_t mem_dim;          /* 64 */
    int32_t num_maskmem;      /* 7: memory slots per instance */
    int32_t max_obj_ptrs;     /* 16 */
    int32_t multimask_in_sam; /* 1 (SAM2): a propagated frame keeps the best of masks 1..3 by IoU */
    int32_t multimask_token_for_obj_ptr; /* 1: its pointer comes from that mask's token */
    int32_t fixed_no_obj_ptr; /* 1 (SAM2): pointer = [obj > 0] * mlp + [obj <= 0] * no_obj_ptr */
    int32_t max_instances;    /* capacity */
    int32_t max_keep_alive;   /* an instance unseen for more frames is dropped (sam3_update_tracker) */
} sam3b200_tracker_hparams;

typedef struct sam3b200_tracker sam3b200_tracker;

sam3b200_tracker *sam3b200_tracker_create(sam3b200_backend *be, const sam3b200_tracker_hparams *hp,
                                          sam3b200_hiera *enc, sam3b200_sam_dec *dec, sam3b200_mem_attn *attn,
                                          sam3b200_mem_enc *menc);
void sam3b200_tracker_free(sam3b200_tracker *t);
int sam3b200_tracker_set_tensor(sam3b200_tracker *t, const char *name, int type, const void *data,
                                const int64_t ne[4]);
/* sam3_encode_image of the next frame (a SAM2-preprocessed frame in device memory). */
int sam3b200_tracker_encode(sam3b200_tracker *t, const float *img_chw_dev);
/* The same from a host RGB frame (uint8 [h][w][3]): upload, SAM2 preprocessing
 * (sam2_preprocess_image), encode -- the image half of sam3_propagate_frame. */
int sam3b200_tracker_encode_image(sam3b200_tracker *t, const uint8_t *rgb, int w, int h);
/* sam3_tracker_reset (sam3.cpp:12090-12110): no instances, frame index 0. */
void sam3b200_tracker_reset(sam3b200_tracker *t);
/* sam3_tracker_add_instance on the encoded frame: PVS decode of the prompts
 * (sam3b200_sam_dec_run's conventions; mask 0), the mask at orig_w x orig_h
 * as +-6 logits on the 4H grid -> a conditioning memory slot, and the SAM
 * token's object pointer.  Returns the instance id (>= 1) or -1. */
int sam3b200_tracker_add_instance(sam3b200_tracker *t, const float *coords, const int32_t *labels, int n_prompts,
                                  int orig_w, int orig_h);
/* sam3_propagate_frame after its encode: every instance propagated and
 * remembered, then the frame index advances.  Synchronous. */
int sam3b200_tracker_propagate(sam3b200_tracker *t);
int sam3b200_tracker_frame_index(const sam3b200_tracker *t);
/* ids of the tracked instances (count returned) */
int sam3b200_tracker_instances(const sam3b200_tracker *t, int32_t *ids, int cap);
/* An instance's last result: kept mask logits [(4H)^2] and its output token
 * [d_model] (device), predicted IoU, object-score logit, last frame seen. */
int sam3b200_tracker_instance(sam3b200_tracker *t, int id, const float **mask_logits_dev, const float **token_dev,
                              float *iou, float *obj_score, int32_t *last_seen);
/* That mask at out_w x out_h (bilinear, binarised at 0): dst_dev uint8 255 / 0. */
int sam3b200_tracker_mask(sam3b200_tracker *t, int id, int out_w, int out_h, uint8_t *dst_dev);
/* An instance's memory: slot frames / conditioning flags / device features
 * [H*H][mem_dim] (slot count returned), pointer frames / device pointers
 * [d_model] (*n_ptrs). */
int sam3b200_tracker_bank(sam3b200_tracker *t, int id, int32_t *slot_frames, int32_t *slot_cond,
                          const float **slot_feats_dev, int slot_cap, int32_t *ptr_frames, const float **ptrs_dev,
                          int ptr_cap, int32_t *n_ptrs);
/* The memory attention inputs the last propagated instance used: prompt and
 * prompt_pos, device [M_total][mem_dim]. */
int sam3b200_tracker_prompt(sam3b200_tracker *t, const float **prompt_dev, const float **prompt_pos_dev);

/* ---- Fusion encoder of the SAM3 detector (the PCS path) --------------------
 * The graph sam3_build_fenc_graph builds (sam3.cpp:8146-8165; layer
 * :8033-8139): `layers` pre-LN blocks over the detector's image tokens --
 * self-attention with the positional code on q and k, cross-attention to the
 * prompt tokens under their padding bias, ReLU FFN.  Weights by name
 * (sam3.cpp:2655-2682): "fenc.layers.<i>.{sa,ca}.in_proj_{weight,bias}",
 * ".{sa,ca}.out_proj.*", ".linear1.*", ".linear2.*", ".norm1".."norm3". */
typedef struct {
    int32_t d_model;     /* 256 */
    int32_t heads;       /* 8 (fenc_heads) */
    int32_t layers;      /* 6 (fenc_layers) */
    int32_t ffn_dim;     /* 2048 (fenc_ffn_dim) */
    int32_t max_tokens;  /* capacity: image tokens (72 * 72) */
    int32_t max_prompt;  /* capacity: prompt tokens (text ctx_len 32 + geometry tokens) */
} sam3b200_fenc_hparams;

typedef struct sam3b200_fenc sam3b200_fenc;

sam3b200_fenc *sam3b200_fenc_create(sam3b200_backend *be, const sam3b200_fenc_hparams *hp);
void sam3b200_fenc_free(sam3b200_fenc *f);
int sam3b200_fenc_set_tensor(sam3b200_fenc *f, const char *name, int type, const void *data, const int64_t ne[4]);
int sam3b200_fenc_missing(sam3b200_fenc *f, char *buf, int cap);
/* Host inputs: image_feats, pos [d_model, n_tokens] (the detector neck's
 * level-2 map and its sine code), prompt [d_model, n_prompt], prompt_bias
 * [n_prompt] (0 valid, -1e9 padding; NULL = no mask). */
int sam3b200_fenc_run(sam3b200_fenc *f, const float *image_feats, const float *prompt, const float *pos,
                      const float *prompt_bias, int n_tokens, int n_prompt);
int sam3b200_fenc_run_device(sam3b200_fenc *f, const float *image_feats, const float *prompt, const float *pos,
                             const float *prompt_bias, int n_tokens, int n_prompt);
/* Conditioned image tokens: device f32 [d_model, n_tokens]. */
int sam3b200_fenc_output(sam3b200_fenc *f, const float **dev);

/* ---- DETR decoder of the SAM3 detector (the PCS path) ---------------------
 * The graph sam3_build_ddec_graph builds (sam3.cpp:8749-8888): presence token
 * + num_queries object queries refined through `layers` post-norm layers
 * (self-attention, text cross-attention under the padding bias, image
 * cross-attention under the box-relative bias of sam3_compute_box_rpb, ReLU
 * FFN) with per-layer query positions from the boxes' sine code and box
 * refinement; then the dot-product scores against the pooled text
 * (sam3_dot_product_scoring, :8640-8739) and the presence logit.  Weights by
 * name (sam3.cpp:2684-2789): "ddec.*" and "scoring.*". */
typedef struct {
    int32_t d_model;      /* 256 */
    int32_t heads;        /* 8 (ddec_heads) */
    int32_t layers;       /* 6 (ddec_layers) */
    int32_t ffn_dim;      /* 2048 (ddec_ffn_dim; also the scoring prompt MLP) */
    int32_t num_queries;  /* 200 (ddec_num_queries) */
    int32_t feat;         /* 72: the side of the image-token grid */
    int32_t max_prompt;   /* capacity: text (+ geometry) tokens */
} sam3b200_ddec_hparams;

typedef struct sam3b200_ddec sam3b200_ddec;

sam3b200_ddec *sam3b200_ddec_create(sam3b200_backend *be, const sam3b200_ddec_hparams *hp);
void sam3b200_ddec_free(sam3b200_ddec *d);
int sam3b200_ddec_set_tensor(sam3b200_ddec *d, const char *name, int type, const void *data, const int64_t ne[4]);
int sam3b200_ddec_missing(sam3b200_ddec *d, char *buf, int cap);
/* Host inputs: enc_feats, enc_pos [d_model, feat*feat] (the fusion encoder's
 * output and the image positional code), text [d_model, n_text], text_bias
 * [n_text] (0 / -1e9; NULL = no mask), text_valid [n_text] (n_text/n_valid
 * for valid tokens, 0 for padding; NULL = plain mean). */
int sam3b200_ddec_run(sam3b200_ddec *d, const float *enc_feats, const float *enc_pos, const float *text,
                      const float *text_bias, const float *text_valid, int n_text);
int sam3b200_ddec_run_device(sam3b200_ddec *d, const float *enc_feats, const float *enc_pos, const float *text,
                             const float *text_bias, const float *text_valid, int n_text);
/* Device outputs of the last run: queries [d_model, 1 + num_queries]
 * (presence, then the normed object queries: the segmentation head's input),
 * boxes [4, num_queries] (cx, cy, w, h in [0, 1]), class scores
 * [num_queries], presence logit [1].  Any pointer may be NULL. */
int sam3b200_ddec_outputs(sam3b200_ddec *d, const float **queries, const float **boxes, const float **scores,
                          const float **presence);

/* ---- Segmentation head of the SAM3 detector (the PCS path) ----------------
 * The graph sam3_build_seg_head_graph builds (sam3.cpp:8975-9058): the
 * fusion-encoder tokens cross-attend to the prompt, replace the lowest FPN
 * level, and the pixel decoder (sam3_pixel_decoder, :8899-8960: nearest 2x
 * upsample + add, conv 3x3, GroupNorm(8), ReLU, twice) brings them to 4*feat;
 * a 1x1 instance head and the 3-layer mask-embedding MLP of the queries give
 * the mask logits.  Weights by name (sam3.cpp:2845-2880): "seg.*". */
typedef struct {
    int32_t d_model;      /* 256 */
    int32_t heads;        /* 8 */
    int32_t feat;         /* 72: the fusion-encoder grid; the masks are 4 * feat square */
    int32_t max_queries;  /* capacity: queries per run (200) */
    int32_t max_prompt;   /* capacity: prompt tokens */
} sam3b200_seg_hparams;

typedef struct sam3b200_seg sam3b200_seg;

sam3b200_seg *sam3b200_seg_create(sam3b200_backend *be, const sam3b200_seg_hparams *hp);
void sam3b200_seg_free(sam3b200_seg *h);
int sam3b200_seg_set_tensor(sam3b200_seg *h, const char *name, int type, const void *data, const int64_t ne[4]);
int sam3b200_seg_missing(sam3b200_seg *h, char *buf, int cap);
/* Host inputs: enc [d_model, feat^2] (fusion encoder output), fpn0
 * [d_model, (4 feat)^2] and fpn1 [d_model, (2 feat)^2] (the detector neck's
 * finest levels), queries [d_model, n_queries] (the decoder's object
 * queries), text [d_model, n_text], text_bias [n_text] or NULL. */
int sam3b200_seg_run(sam3b200_seg *h, const float *enc, const float *fpn0, const float *fpn1, const float *queries,
                     int n_queries, const float *text, const float *text_bias, int n_text);
int sam3b200_seg_run_device(sam3b200_seg *h, const float *enc, const float *fpn0, const float *fpn1,
                            const float *queries, int n_queries, const float *text, const float *text_bias,
                            int n_text);
/* Mask logits: device f32 [(4 feat)^2, n_queries] (memory [n_queries][pixels]). */
int sam3b200_seg_output(sam3b200_seg *h, const float **dev);

/* ---- Geometry (exemplar-prompt) encoder of the SAM3 detector --------------
 * The transformer of sam3_build_geom_enc_graph (sam3.cpp:7677-7800) over the
 * geometry tokens the host prepares (box embeddings + CLS after the final
 * projection and norm, sam3_precompute_geom_input): `layers` pre-LN layers
 * of self-attention (no position), cross-attention to the image (keys from
 * features + positional code, values from features), ReLU FFN, then
 * geom.encode_norm.  Weights by name (sam3.cpp:2821-2842):
 * "geom.layers.<i>.*", "geom.encode_norm.*"; the other "geom.*" tensors feed
 * the host-side token preparation. */
typedef struct {
    int32_t d_model;           /* 256 */
    int32_t heads;             /* 8 */
    int32_t layers;            /* 3 (geom_layers) */
    int32_t ffn_dim;           /* 2048 */
    int32_t max_tokens;        /* capacity: exemplar boxes + 1 */
    int32_t max_image_tokens;  /* capacity: image tokens (72 * 72) */
} sam3b200_geom_hparams;

typedef struct sam3b200_geom sam3b200_geom;

sam3b200_geom *sam3b200_geom_create(sam3b200_backend *be, const sam3b200_geom_hparams *hp);
void sam3b200_geom_free(sam3b200_geom *g);
int sam3b200_geom_set_tensor(sam3b200_geom *g, const char *name, int type, const void *data, const int64_t ne[4]);
int sam3b200_geom_missing(sam3b200_geom *g, char *buf, int cap);
/* Host inputs: tokens [d_model, n_tokens], img_feats and img_pe
 * [d_model, n_image]. */
int sam3b200_geom_run(sam3b200_geom *g, const float *tokens, int n_tokens, const float *img_feats,
                      const float *img_pe, int n_image);
int sam3b200_geom_run_device(sam3b200_geom *g, const float *tokens, int n_tokens, const float *img_feats,
                             const float *img_pe, int n_image);
/* Encoded geometry tokens: device f32 [d_model, n_tokens]. */
int sam3b200_geom_output(sam3b200_geom *g, const float **dev);

/* ---- SAM3 visual encoder (sam3_encode_image for a visual-only model) ----
 *
 * Hyper-parameters of the ViT + tracker neck, the fields sam3_hparams holds
 * for the encoder (sam3.cpp:74-98): img_size 1008, patch 14, embed 1024,
 * depth 32, heads 16 (head_dim must be 64), mlp 4736, window 24, global
 * blocks {7, 15, 23, 31}, pos_embed grid 24 (img/patch/3, sam3.cpp:2533),
 * neck_dim 256; wtype is the ggml type of the four linear weights of every
 * block (Q8_0 or Q4_0; sam3.cpp:2476-2499 picks it per tensor). */
typedef struct {
    int img, patch, embed, depth, heads, mlp, window;
    int n_global;
    int global_idx[4];
    int pos_grid, neck_dim, wtype;
} sam3b200_vit_hparams;

typedef struct sam3b200_vit sam3b200_vit;

/* Allocate an encoder and its activation buffers on the backend's device
 * (the model + state pair of sam3_load_model / sam3_create_state,
 * sam3.cpp:3204-3348, 3380-3415, restricted to the visual encoder). */
sam3b200_vit *sam3b200_vit_create(sam3b200_backend *be, const sam3b200_vit_hparams *hp);
void sam3b200_vit_free(sam3b200_vit *vit);

/* One weight tensor by its weight-file name and ggml shape (ne[0..3]),
 * the per-tensor step of sam3_load_tensors (sam3.cpp:3095-3198): names
 * "vit.patch_embed.proj.weight", "vit.pos_embed", "vit.ln_pre.{weight,bias}",
 * "vit.blocks.<i>.{norm1,norm2}.{weight,bias}", "...attn.qkv.{weight,bias}",
 * "...attn.proj.{weight,bias}", "...mlp.lin1.{weight,bias}",
 * "...mlp.lin2.{weight,bias}", "...attn.freqs_cis", "neck.trk.<s>.*"
 * (sam3.cpp:2529-2600).  Linear weights are Q8_0/Q4_0, the rest F32/F16. */
int sam3b200_vit_set_tensor(sam3b200_vit *vit, const char *name, int type, const void *data, const int64_t ne[4]);

/* Number of encoder tensors not yet set; their names, newline-separated,
 * into buf (may be NULL). */
int sam3b200_vit_missing(sam3b200_vit *vit, char *buf, int cap);

/* sam3_encode_image (sam3.cpp:6028-6149): uint8 RGB HWC host image of any
 * size (resized like sam3_resize_bilinear when it is not img x img), then
 * preprocessing, ViT and tracker neck; the four neck maps are copied to
 * out_host[i] (f32 [neck_dim, W, H], W = H = 4G, 2G, G, G/2 for G =
 * img/patch; NULL entries are skipped).  Synchronous. */
int sam3b200_encode_image(sam3b200_vit *vit, const uint8_t *rgb, int w, int h, float *const out_host[4]);

/* Same with the image already in device memory; asynchronous on the
 * backend stream; results stay in the encoder's buffers
 * (sam3b200_vit_output). */
int sam3b200_encode_image_device(sam3b200_vit *vit, const uint8_t *rgb_dev, int w, int h);

/* sam3_encode_image for n images at once (a batch of sam3.cpp:6028-6149
 * calls; the reference has no batched form): each image is preprocessed and
 * embedded, then the ViT blocks run once over the n images' tokens stacked
 * image-major -- every MUL_MAT, attention and LayerNorm launch covers all n,
 * which fills the 148 SMs in whole waves -- and each image gets its neck.
 * Results per image are bit-identical to n single encodes.  DQ16 arithmetic
 * (sam3b200_set_arith); under EXACT the images are encoded one by one.  The
 * first call with a larger n than before grows the block-loop buffers (~0.11
 * GB per extra 1008^2 image) and synchronises.  rgb[i]: n uint8 RGB HWC host
 * images of w x h; out_host[4 i + j]: image i's neck map j (as for
 * sam3b200_encode_image; NULL entries skipped).  Synchronous. */
int sam3b200_encode_images(sam3b200_vit *vit, int n, const uint8_t *const *rgb, int w, int h,
                           float *const *out_host);

/* Same with the images in device memory; asynchronous on the backend
 * stream.  Afterwards sam3b200_vit_output(0..3) holds the last image's neck
 * maps and sam3b200_vit_output(-1) the first image's ViT output (the n
 * outputs follow it, image-major). */
int sam3b200_encode_images_device(sam3b200_vit *vit, int n, const uint8_t *const *rgb_dev, int w, int h);

/* Device pointer and ggml shape of output i (0..3 = neck_trk_i, -1 = the
 * ViT output [embed, G, G]) of the last encode. */
int sam3b200_vit_output(sam3b200_vit *vit, int i, const float **dev, int64_t ne[4]);
/* The detector neck's level i (0..3) of the last encode, same layout: a full
 * (not visual-only) SAM3 model runs both necks of sam3_build_neck_graph
 * (sam3.cpp:3867-3925) on the ViT output, "neck.det.<s>.*" weights beside
 * "neck.trk.<s>.*"; fails when no neck.det tensor was set. */
int sam3b200_vit_output_det(sam3b200_vit *vit, int i, const float **dev, int64_t ne[4]);

/* sam3_preprocess_image (sam3.cpp:3490-3518, with sam3_resize_bilinear
 * :3445-3485 when w x h != img x img): device uint8 RGB HWC -> device f32
 * CHW [img, img, 3] normalised (p/255 - 0.5)/0.5.  Asynchronous. */
int sam3b200_preprocess(sam3b200_backend *be, const uint8_t *rgb_dev, int w, int h, int img, float *out_dev);

/* sam2_preprocess_image (sam3.cpp:3522-3548, same resize): the SAM2 / Hiera
 * input, normalised (p/255 - mean[c]) / std[c] with the ImageNet mean
 * (0.485, 0.456, 0.406) and std (0.229, 0.224, 0.225).  Asynchronous. */
int sam3b200_preprocess_sam2(sam3b200_backend *be, const uint8_t *rgb_dev, int w, int h, int img, float *out_dev);

/* Stage runners on caller-provided device tensors, the analogue of the
 * reference's stage test hooks (sam3.h sam3_vit_prefix_stage /
 * sam3_vit_block_stage): prefix image f32 CHW -> x [embed, G, G]; one
 * block in place on x; neck from x into the encoder's outputs. */
int sam3b200_vit_run_prefix(sam3b200_vit *vit, const float *img_chw_dev, float *x_dev);
int sam3b200_vit_run_block(sam3b200_vit *vit, int idx, float *x_dev);
int sam3b200_vit_run_neck(sam3b200_vit *vit, const float *x_dev);

/* ---- Weight files (sam3_load_model / sam3_load_tensors) -------------------
 * The format sam3.cpp reads (sam3.cpp:3095-3198, 3204-3330): magic "sam3"
 * (version 3) or "sam2" (version 1), ftype, tensor count, the int32
 * hyper-parameter words of sam3_load_hparams / sam2_load_hparams
 * (:1481-1525, :1568-1630), then per tensor n_dims, name length, ggml type,
 * ne[0..n_dims), the name, zero padding to a 32-byte file offset and the data.
 * Opening scans the records (no tensor data is read and no GPU is used). */
typedef struct sam3b200_file sam3b200_file;

sam3b200_file *sam3b200_file_open(const char *path);
void sam3b200_file_close(sam3b200_file *f);
int sam3b200_file_info(const sam3b200_file *f, uint32_t *magic, int32_t *version, int32_t *ftype,
                       int32_t *n_tensors);
/* Copies up to cap hyper-parameter words; returns how many the file holds. */
int sam3b200_file_hparams(const sam3b200_file *f, int32_t *words, int cap);
/* Record i: name, ggml type, ne[4] (1-padded), data offset and size in bytes. */
int sam3b200_file_tensor(const sam3b200_file *f, int i, char *name, int name_cap, int32_t *type, int64_t ne[4],
                         int64_t *offset, int64_t *bytes);
/* Runner hyper-parameters derived from the file (SAM3: ViT + text; SAM2: Hiera). */
int sam3b200_file_vit_hparams(const sam3b200_file *f, sam3b200_vit_hparams *out);
int sam3b200_file_text_hparams(const sam3b200_file *f, sam3b200_text_hparams *out);
int sam3b200_file_hiera_hparams(const sam3b200_file *f, sam3b200_hiera_hparams *out);

/* The runners a file's tensors go to, by name prefix: "vit."/"neck.trk."/
 * "neck.det." -> vit, "hiera."/"fpn." -> hiera, "text." -> text, "sam_pe."/"sam_dec."/
 * "no_mem_embed" -> sam_dec, "mem_attn." -> mem_attn, "mem_enc."/
 * "no_obj_embed_spatial" -> mem_enc, "fenc." -> fenc, "ddec."/"scoring." ->
 * ddec, "seg." -> seg, "geom.layers."/"geom.encode_norm." -> geom.  A NULL
 * runner leaves its tensors skipped. */
typedef struct {
    sam3b200_vit *vit;
    sam3b200_hiera *hiera;
    sam3b200_text *text;
    sam3b200_sam_dec *sam_dec;
    sam3b200_mem_attn *mem_attn;
    sam3b200_mem_enc *mem_enc;
    sam3b200_fenc *fenc;
    sam3b200_ddec *ddec;
    sam3b200_seg *seg;
    sam3b200_geom *geom;
} sam3b200_model_parts;

/* Stream every tensor to its runner through two pinned staging buffers (a
 * reader thread overlaps the file reads with the device copies).  Fails on
 * the first tensor a runner rejects; counts loaded and skipped tensors. */
int sam3b200_file_load(sam3b200_file *f, sam3b200_backend *be, const sam3b200_model_parts *parts,
                       int64_t *n_loaded, int64_t *n_skipped);
/* Names of the tensors the last load skipped, newline-separated; returns the count. */
int sam3b200_file_skipped(const sam3b200_file *f, char *buf, int cap);

#ifdef __cplusplus
}
#endif
#endif /* SAM3_B200_H */
