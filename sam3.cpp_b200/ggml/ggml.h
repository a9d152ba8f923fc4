/* ggml.h -- the subset of ggml's public C API that sam3.cpp's graph code and
 * a ggml backend use, written here so the B200 backend (ggml-b200.cpp) builds
 * and runs without the ggml fork sam3.cpp pins (an un-vendored submodule).
 *
 * Names, field names, the ggml_type codes and the ggml_status codes are
 * ggml's.  The ggml_op / ggml_unary_op numbering is this header's own: the
 * backend translates ops by name (a switch over GGML_OP_*), so it compiles
 * unchanged against the fork's ggml.h, whose numbering is whatever that
 * commit has.  struct ggml_tensor has ggml's member names and order.
 *
 * The functions declared here that build graphs only record shapes, strides
 * and sources (ggml-mini.cpp); every computation runs in a backend. */
#pragma once

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GGML_MAX_DIMS 4
#define GGML_MAX_PARAMS 2048
#define GGML_MAX_SRC 10
#define GGML_MAX_NAME 64
#define GGML_MAX_OP_PARAMS 64
#define GGML_DEFAULT_GRAPH_SIZE 2048
#define GGML_MEM_ALIGN 16

typedef uint16_t ggml_fp16_t;

enum ggml_status {
    GGML_STATUS_ALLOC_FAILED = -2,
    GGML_STATUS_FAILED = -1,
    GGML_STATUS_SUCCESS = 0,
    GGML_STATUS_ABORTED = 1,
};

enum ggml_type {
    GGML_TYPE_F32 = 0,
    GGML_TYPE_F16 = 1,
    GGML_TYPE_Q4_0 = 2,
    GGML_TYPE_Q4_1 = 3,
    GGML_TYPE_Q5_0 = 6,
    GGML_TYPE_Q5_1 = 7,
    GGML_TYPE_Q8_0 = 8,
    GGML_TYPE_Q8_1 = 9,
    GGML_TYPE_I8 = 24,
    GGML_TYPE_I16 = 25,
    GGML_TYPE_I32 = 26,
    GGML_TYPE_I64 = 27,
    GGML_TYPE_F64 = 28,
    GGML_TYPE_BF16 = 30,
    GGML_TYPE_COUNT = 40,
};

enum ggml_op {
    GGML_OP_NONE = 0,
    GGML_OP_DUP,
    GGML_OP_ADD,
    GGML_OP_SUB,
    GGML_OP_MUL,
    GGML_OP_DIV,
    GGML_OP_LOG,
    GGML_OP_SIN,
    GGML_OP_COS,
    GGML_OP_REPEAT,
    GGML_OP_CONCAT,
    GGML_OP_NORM,
    GGML_OP_GROUP_NORM,
    GGML_OP_MUL_MAT,
    GGML_OP_SCALE,
    GGML_OP_CPY,
    GGML_OP_CONT,
    GGML_OP_RESHAPE,
    GGML_OP_VIEW,
    GGML_OP_PERMUTE,
    GGML_OP_TRANSPOSE,
    GGML_OP_GET_ROWS,
    GGML_OP_SOFT_MAX,
    GGML_OP_CLAMP,
    GGML_OP_CONV_TRANSPOSE_2D,
    GGML_OP_IM2COL,
    GGML_OP_CONV_2D,
    GGML_OP_CONV_2D_DW,
    GGML_OP_POOL_1D,
    GGML_OP_POOL_2D,
    GGML_OP_UPSCALE,
    GGML_OP_PAD,
    GGML_OP_WIN_PART,
    GGML_OP_WIN_UNPART,
    GGML_OP_FLASH_ATTN_EXT,
    GGML_OP_UNARY,
    GGML_OP_COUNT,
};

enum ggml_unary_op {
    GGML_UNARY_OP_ABS,
    GGML_UNARY_OP_SGN,
    GGML_UNARY_OP_NEG,
    GGML_UNARY_OP_TANH,
    GGML_UNARY_OP_RELU,
    GGML_UNARY_OP_SIGMOID,
    GGML_UNARY_OP_GELU,
    GGML_UNARY_OP_GELU_ERF,
    GGML_UNARY_OP_SILU,
    GGML_UNARY_OP_COUNT,
};

enum ggml_op_pool { GGML_OP_POOL_MAX, GGML_OP_POOL_AVG, GGML_OP_POOL_COUNT };

enum ggml_scale_mode { GGML_SCALE_MODE_NEAREST = 0, GGML_SCALE_MODE_BILINEAR = 1 };

enum ggml_prec { GGML_PREC_DEFAULT = 0, GGML_PREC_F32 = 10 };

enum ggml_tensor_flag {
    GGML_TENSOR_FLAG_INPUT = 1,
    GGML_TENSOR_FLAG_OUTPUT = 2,
    GGML_TENSOR_FLAG_PARAM = 4,
    GGML_TENSOR_FLAG_LOSS = 8,
};

struct ggml_backend_buffer;

struct ggml_tensor {
    enum ggml_type type;
    struct ggml_backend_buffer *buffer;
    int64_t ne[GGML_MAX_DIMS];
    size_t nb[GGML_MAX_DIMS];
    enum ggml_op op;
    int32_t op_params[GGML_MAX_OP_PARAMS / sizeof(int32_t)];
    int32_t flags;
    struct ggml_tensor *src[GGML_MAX_SRC];
    struct ggml_tensor *view_src;
    size_t view_offs;
    void *data;
    char name[GGML_MAX_NAME];
    void *extra;
    char padding[8];
};

struct ggml_context;
struct ggml_cgraph;

struct ggml_init_params {
    size_t mem_size;   /* bytes of tensor metadata (and data, unless no_alloc) the context may hold */
    void *mem_buffer;  /* ignored: the context allocates its own */
    bool no_alloc;     /* tensors get no data; a backend buffer provides it */
};

/* type traits */
size_t ggml_type_size(enum ggml_type type);
int64_t ggml_blck_size(enum ggml_type type);
const char *ggml_type_name(enum ggml_type type);
bool ggml_is_quantized(enum ggml_type type);
size_t ggml_row_size(enum ggml_type type, int64_t ne);
const char *ggml_op_name(enum ggml_op op);
const char *ggml_status_to_string(enum ggml_status status);
float ggml_fp16_to_fp32(ggml_fp16_t h);
ggml_fp16_t ggml_fp32_to_fp16(float f);
void ggml_fp16_to_fp32_row(const ggml_fp16_t *x, float *y, int64_t n);
void ggml_fp32_to_fp16_row(const float *x, ggml_fp16_t *y, int64_t n);

/* tensor queries */
int64_t ggml_nelements(const struct ggml_tensor *t);
int64_t ggml_nrows(const struct ggml_tensor *t);
size_t ggml_nbytes(const struct ggml_tensor *t);
int ggml_n_dims(const struct ggml_tensor *t);
bool ggml_is_contiguous(const struct ggml_tensor *t);
bool ggml_is_empty(const struct ggml_tensor *t);
enum ggml_unary_op ggml_get_unary_op(const struct ggml_tensor *t);
const char *ggml_get_name(const struct ggml_tensor *t);
struct ggml_tensor *ggml_set_name(struct ggml_tensor *t, const char *name);
void ggml_set_input(struct ggml_tensor *t);
void ggml_set_output(struct ggml_tensor *t);
void *ggml_get_data(const struct ggml_tensor *t);

/* contexts */
size_t ggml_tensor_overhead(void);
size_t ggml_graph_overhead(void);
size_t ggml_graph_overhead_custom(size_t size, bool grads);
struct ggml_context *ggml_init(struct ggml_init_params params);
void ggml_free(struct ggml_context *ctx);
struct ggml_tensor *ggml_get_tensor(struct ggml_context *ctx, const char *name);
struct ggml_tensor *ggml_get_first_tensor(const struct ggml_context *ctx);
struct ggml_tensor *ggml_get_next_tensor(const struct ggml_context *ctx, struct ggml_tensor *t);

struct ggml_tensor *ggml_new_tensor(struct ggml_context *ctx, enum ggml_type type, int n_dims, const int64_t *ne);
struct ggml_tensor *ggml_new_tensor_1d(struct ggml_context *ctx, enum ggml_type type, int64_t ne0);
struct ggml_tensor *ggml_new_tensor_2d(struct ggml_context *ctx, enum ggml_type type, int64_t ne0, int64_t ne1);
struct ggml_tensor *ggml_new_tensor_3d(struct ggml_context *ctx, enum ggml_type type, int64_t ne0, int64_t ne1,
                                       int64_t ne2);
struct ggml_tensor *ggml_new_tensor_4d(struct ggml_context *ctx, enum ggml_type type, int64_t ne0, int64_t ne1,
                                       int64_t ne2, int64_t ne3);
struct ggml_tensor *ggml_dup_tensor(struct ggml_context *ctx, const struct ggml_tensor *src);
struct ggml_tensor *ggml_view_tensor(struct ggml_context *ctx, struct ggml_tensor *src);

/* graph builders (shapes only) */
struct ggml_tensor *ggml_add(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b);
struct ggml_tensor *ggml_add_inplace(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b);
struct ggml_tensor *ggml_sub(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b);
struct ggml_tensor *ggml_mul(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b);
struct ggml_tensor *ggml_mul_inplace(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b);
struct ggml_tensor *ggml_scale(struct ggml_context *ctx, struct ggml_tensor *a, float s);
struct ggml_tensor *ggml_repeat(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b);
struct ggml_tensor *ggml_concat(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b, int dim);
struct ggml_tensor *ggml_norm(struct ggml_context *ctx, struct ggml_tensor *a, float eps);
struct ggml_tensor *ggml_group_norm(struct ggml_context *ctx, struct ggml_tensor *a, int n_groups, float eps);
struct ggml_tensor *ggml_mul_mat(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b);
struct ggml_tensor *ggml_relu(struct ggml_context *ctx, struct ggml_tensor *a);
struct ggml_tensor *ggml_sigmoid(struct ggml_context *ctx, struct ggml_tensor *a);
struct ggml_tensor *ggml_gelu(struct ggml_context *ctx, struct ggml_tensor *a);
struct ggml_tensor *ggml_gelu_erf(struct ggml_context *ctx, struct ggml_tensor *a);
struct ggml_tensor *ggml_soft_max_ext(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *mask,
                                      float scale, float max_bias);
struct ggml_tensor *ggml_cont(struct ggml_context *ctx, struct ggml_tensor *a);
struct ggml_tensor *ggml_cpy(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b);
struct ggml_tensor *ggml_cast(struct ggml_context *ctx, struct ggml_tensor *a, enum ggml_type type);
struct ggml_tensor *ggml_reshape_1d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0);
struct ggml_tensor *ggml_reshape_2d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, int64_t ne1);
struct ggml_tensor *ggml_reshape_3d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, int64_t ne1,
                                    int64_t ne2);
struct ggml_tensor *ggml_reshape_4d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, int64_t ne1,
                                    int64_t ne2, int64_t ne3);
struct ggml_tensor *ggml_view_1d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, size_t offset);
struct ggml_tensor *ggml_view_2d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, int64_t ne1,
                                 size_t nb1, size_t offset);
struct ggml_tensor *ggml_view_3d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, int64_t ne1,
                                 int64_t ne2, size_t nb1, size_t nb2, size_t offset);
struct ggml_tensor *ggml_view_4d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, int64_t ne1,
                                 int64_t ne2, int64_t ne3, size_t nb1, size_t nb2, size_t nb3, size_t offset);
struct ggml_tensor *ggml_permute(struct ggml_context *ctx, struct ggml_tensor *a, int axis0, int axis1, int axis2,
                                 int axis3);
struct ggml_tensor *ggml_transpose(struct ggml_context *ctx, struct ggml_tensor *a);
struct ggml_tensor *ggml_get_rows(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b);
struct ggml_tensor *ggml_win_part(struct ggml_context *ctx, struct ggml_tensor *a, int w);
struct ggml_tensor *ggml_win_unpart(struct ggml_context *ctx, struct ggml_tensor *a, int w0, int h0, int w);
struct ggml_tensor *ggml_flash_attn_ext(struct ggml_context *ctx, struct ggml_tensor *q, struct ggml_tensor *k,
                                        struct ggml_tensor *v, struct ggml_tensor *mask, float scale,
                                        float max_bias, float logit_softcap);
struct ggml_tensor *ggml_im2col(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b, int s0,
                                int s1, int p0, int p1, int d0, int d1, bool is_2D, enum ggml_type dst_type);
struct ggml_tensor *ggml_conv_2d(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b, int s0,
                                 int s1, int p0, int p1, int d0, int d1);
struct ggml_tensor *ggml_conv_2d_sk_p0(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b);
struct ggml_tensor *ggml_conv_2d_s1_ph(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b);
struct ggml_tensor *ggml_conv_2d_direct(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b,
                                        int s0, int s1, int p0, int p1, int d0, int d1);
struct ggml_tensor *ggml_conv_2d_dw_direct(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b,
                                           int s0, int s1, int p0, int p1, int d0, int d1);
struct ggml_tensor *ggml_conv_transpose_2d_p0(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b,
                                              int stride);
struct ggml_tensor *ggml_pool_2d(struct ggml_context *ctx, struct ggml_tensor *a, enum ggml_op_pool op, int k0,
                                 int k1, int s0, int s1, float p0, float p1);
struct ggml_tensor *ggml_pad(struct ggml_context *ctx, struct ggml_tensor *a, int p0, int p1, int p2, int p3);
struct ggml_tensor *ggml_pad_ext(struct ggml_context *ctx, struct ggml_tensor *a, int lp0, int rp0, int lp1, int rp1,
                                 int lp2, int rp2, int lp3, int rp3);
struct ggml_tensor *ggml_upscale(struct ggml_context *ctx, struct ggml_tensor *a, int scale_factor,
                                 enum ggml_scale_mode mode);

/* graphs */
struct ggml_cgraph *ggml_new_graph(struct ggml_context *ctx);
struct ggml_cgraph *ggml_new_graph_custom(struct ggml_context *ctx, size_t size, bool grads);
void ggml_build_forward_expand(struct ggml_cgraph *cgraph, struct ggml_tensor *tensor);
int ggml_graph_n_nodes(struct ggml_cgraph *cgraph);
struct ggml_tensor *ggml_graph_node(struct ggml_cgraph *cgraph, int i); /* i < 0 counts from the end */
struct ggml_tensor *ggml_graph_get_tensor(const struct ggml_cgraph *cgraph, const char *name);

#ifdef __cplusplus
}
#endif
