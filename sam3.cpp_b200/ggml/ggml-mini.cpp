// ggml-mini.cpp -- the parts of ggml's core that a caller of a ggml backend
// goes through, restated for building and running graphs on the B200 backend
// without the ggml fork: contexts that hold tensor metadata, graph builders
// that record shapes, strides, op parameters and sources (the shape rules of
// ggml.c for each op), the forward graph order, the backend / buffer dispatch
// of ggml-backend.c and a graph allocator.  Nothing here computes a tensor:
// every op runs in a backend.  A build inside the fork links the fork's
// libggml-base instead of this file.
//
// C++14, no exceptions across the C API: a broken precondition (the cases
// where ggml.c asserts) prints the reason and aborts, as GGML_ASSERT does.
#include "ggml-alloc.h"
#include "ggml-backend-impl.h"
#include "ggml.h"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <string>
#include <unordered_set>
#include <vector>

#define MINI_ASSERT(x)                                                                  \
    do {                                                                                \
        if (!(x)) {                                                                     \
            std::fprintf(stderr, "%s:%d: GGML_ASSERT(%s) failed\n", __FILE__, __LINE__, #x); \
            std::abort();                                                               \
        }                                                                               \
    } while (0)

struct ggml_cgraph {
    size_t size = 0;
    std::vector<ggml_tensor *> nodes;
    std::vector<ggml_tensor *> leafs;
    std::unordered_set<const ggml_tensor *> visited;
};

struct ggml_context {
    size_t mem_size = 0;
    size_t used = 0;
    bool no_alloc = false;
    std::deque<ggml_tensor> tensors;  // stable addresses, creation order
    std::deque<std::vector<char>> host_data;
    std::deque<ggml_cgraph> graphs;
};

namespace {

struct TypeInfo {
    const char *name;
    int64_t blck;
    size_t size;
    bool quantized;
};

TypeInfo type_info(ggml_type t) {
    switch (t) {
        case GGML_TYPE_F32: return {"f32", 1, 4, false};
        case GGML_TYPE_F16: return {"f16", 1, 2, false};
        case GGML_TYPE_BF16: return {"bf16", 1, 2, false};
        case GGML_TYPE_Q4_0: return {"q4_0", 32, 18, true};
        case GGML_TYPE_Q4_1: return {"q4_1", 32, 20, true};
        case GGML_TYPE_Q5_0: return {"q5_0", 32, 22, true};
        case GGML_TYPE_Q5_1: return {"q5_1", 32, 24, true};
        case GGML_TYPE_Q8_0: return {"q8_0", 32, 34, true};
        case GGML_TYPE_Q8_1: return {"q8_1", 32, 36, true};
        case GGML_TYPE_I8: return {"i8", 1, 1, false};
        case GGML_TYPE_I16: return {"i16", 1, 2, false};
        case GGML_TYPE_I32: return {"i32", 1, 4, false};
        case GGML_TYPE_I64: return {"i64", 1, 8, false};
        case GGML_TYPE_F64: return {"f64", 1, 8, false};
        default: return {"unknown", 1, 0, false};
    }
}

ggml_tensor *new_tensor_impl(ggml_context *ctx, ggml_type type, int n_dims, const int64_t *ne, ggml_tensor *view_src,
                             size_t view_offs) {
    MINI_ASSERT(n_dims >= 1 && n_dims <= GGML_MAX_DIMS);
    const TypeInfo ti = type_info(type);
    MINI_ASSERT(ti.size != 0);
    if (view_src && view_src->view_src) {  // a view of a view points at the base tensor
        view_offs += view_src->view_offs;
        view_src = view_src->view_src;
    }
    ctx->used += ggml_tensor_overhead();
    MINI_ASSERT(ctx->used <= ctx->mem_size);  // the context was sized for fewer tensors
    ctx->tensors.emplace_back();
    ggml_tensor *t = &ctx->tensors.back();
    std::memset(t, 0, sizeof *t);
    t->type = type;
    for (int i = 0; i < GGML_MAX_DIMS; ++i) t->ne[i] = i < n_dims ? ne[i] : 1;
    t->nb[0] = ti.size;
    t->nb[1] = ti.size * static_cast<size_t>(t->ne[0] / ti.blck);
    for (int i = 2; i < GGML_MAX_DIMS; ++i) t->nb[i] = t->nb[i - 1] * static_cast<size_t>(t->ne[i - 1]);
    t->view_src = view_src;
    t->view_offs = view_offs;
    if (view_src) {
        t->buffer = view_src->buffer;
        if (view_src->data) t->data = static_cast<char *>(view_src->data) + view_offs;
    } else if (!ctx->no_alloc) {
        ctx->host_data.emplace_back(ggml_nbytes(t));
        t->data = ctx->host_data.back().data();
    }
    return t;
}

ggml_tensor *new_tensor(ggml_context *ctx, ggml_type type, int64_t ne0, int64_t ne1 = 1, int64_t ne2 = 1,
                        int64_t ne3 = 1) {
    const int64_t ne[4] = {ne0, ne1, ne2, ne3};
    return new_tensor_impl(ctx, type, 4, ne, nullptr, 0);
}

void set_param_f32(ggml_tensor *t, int i, float v) { std::memcpy(&t->op_params[i], &v, sizeof v); }

bool can_repeat(const ggml_tensor *t0, const ggml_tensor *t1) {  // t0 repeats into t1
    for (int i = 0; i < GGML_MAX_DIMS; ++i)
        if (t0->ne[i] == 0 || t1->ne[i] % t0->ne[i] != 0) return false;
    return true;
}

ggml_tensor *binary(ggml_context *ctx, ggml_op op, ggml_tensor *a, ggml_tensor *b, bool inplace) {
    MINI_ASSERT(can_repeat(b, a));
    ggml_tensor *r = inplace ? ggml_view_tensor(ctx, a) : ggml_dup_tensor(ctx, a);
    r->op = op;
    r->src[0] = a;
    r->src[1] = b;
    return r;
}

ggml_tensor *unary(ggml_context *ctx, ggml_tensor *a, ggml_unary_op u) {
    ggml_tensor *r = ggml_dup_tensor(ctx, a);
    r->op = GGML_OP_UNARY;
    r->op_params[0] = u;
    r->src[0] = a;
    return r;
}

int64_t conv_out_size(int64_t ins, int64_t ks, int s, int p, int d) { return (ins + 2 * p - d * (ks - 1) - 1) / s + 1; }

ggml_tensor *view_impl(ggml_context *ctx, ggml_tensor *a, int n_dims, const int64_t *ne, size_t offset) {
    ggml_tensor *r = new_tensor_impl(ctx, a->type, n_dims, ne, a, offset);
    r->op = GGML_OP_VIEW;
    r->src[0] = a;
    std::memcpy(r->op_params, &offset, sizeof offset);
    return r;
}

ggml_tensor *reshape_impl(ggml_context *ctx, ggml_tensor *a, int n_dims, const int64_t *ne) {
    MINI_ASSERT(ggml_is_contiguous(a));
    int64_t n = 1;
    for (int i = 0; i < n_dims; ++i) n *= ne[i];
    MINI_ASSERT(n == ggml_nelements(a));
    ggml_tensor *r = new_tensor_impl(ctx, a->type, n_dims, ne, a, 0);
    r->op = GGML_OP_RESHAPE;
    r->src[0] = a;
    return r;
}

void visit(ggml_cgraph *g, ggml_tensor *t) {
    if (!g->visited.insert(t).second) return;
    for (int i = 0; i < GGML_MAX_SRC; ++i)
        if (t->src[i]) visit(g, t->src[i]);
    if (t->op == GGML_OP_NONE && !(t->flags & GGML_TENSOR_FLAG_PARAM)) {
        g->leafs.push_back(t);
    } else {
        MINI_ASSERT(g->nodes.size() < g->size);  // the graph was created for fewer nodes
        g->nodes.push_back(t);
    }
}

// fp16 <-> fp32, IEEE binary16 with round to nearest even
uint16_t f32_to_f16_bits(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t absx = x & 0x7fffffffu;
    if (absx >= 0x7f800000u) return static_cast<uint16_t>(sign | (absx > 0x7f800000u ? 0x7e00u : 0x7c00u));
    if (absx >= 0x477ff000u) return static_cast<uint16_t>(sign | 0x7c00u);  // rounds to >= 65520: infinity
    if (absx < 0x38800000u) {                                               // below the smallest normal half
        if (absx < 0x33000000u) return static_cast<uint16_t>(sign);         // below half the smallest subnormal
        const uint32_t e = absx >> 23, m = (absx & 0x7fffffu) | 0x800000u;
        const uint32_t shift = 126 - e;  // value = m * 2^(e - 150); in units of 2^-24: m >> (126 - e)
        uint32_t h = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1u))) ++h;
        return static_cast<uint16_t>(sign | h);
    }
    uint32_t h = ((absx >> 13) - (112u << 10));
    const uint32_t rem = absx & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
    return static_cast<uint16_t>(sign | h);
}

float f16_bits_to_f32(uint16_t h) {
    const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu, x;
    if (e == 0) {
        if (m == 0) {
            x = sign;
        } else {  // subnormal: normalise
            int s = -1;
            do {
                ++s;
                m <<= 1;
            } while (!(m & 0x400u));
            x = sign | ((112u - s) << 23) | ((m & 0x3ffu) << 13);
        }
    } else if (e == 31) {
        x = sign | 0x7f800000u | (m << 13);
    } else {
        x = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    std::memcpy(&f, &x, 4);
    return f;
}

}  // namespace

extern "C" {

// ---- type traits --------------------------------------------------------------------------------

size_t ggml_type_size(enum ggml_type type) { return type_info(type).size; }
int64_t ggml_blck_size(enum ggml_type type) { return type_info(type).blck; }
const char *ggml_type_name(enum ggml_type type) { return type_info(type).name; }
bool ggml_is_quantized(enum ggml_type type) { return type_info(type).quantized; }
size_t ggml_row_size(enum ggml_type type, int64_t ne) {
    const TypeInfo ti = type_info(type);
    return ti.size * static_cast<size_t>(ne / ti.blck);
}

const char *ggml_op_name(enum ggml_op op) {
    static const char *names[GGML_OP_COUNT] = {
        "NONE", "DUP", "ADD", "SUB", "MUL", "DIV", "LOG", "SIN", "COS", "REPEAT", "CONCAT", "NORM", "GROUP_NORM",
        "MUL_MAT", "SCALE", "CPY", "CONT", "RESHAPE", "VIEW", "PERMUTE", "TRANSPOSE", "GET_ROWS", "SOFT_MAX",
        "CLAMP", "CONV_TRANSPOSE_2D", "IM2COL", "CONV_2D", "CONV_2D_DW", "POOL_1D", "POOL_2D", "UPSCALE", "PAD",
        "WIN_PART", "WIN_UNPART", "FLASH_ATTN_EXT", "UNARY"};
    return op >= 0 && op < GGML_OP_COUNT ? names[op] : "?";
}

const char *ggml_status_to_string(enum ggml_status status) {
    switch (status) {
        case GGML_STATUS_ALLOC_FAILED: return "GGML status: error (failed to allocate memory)";
        case GGML_STATUS_FAILED: return "GGML status: error (operation failed)";
        case GGML_STATUS_SUCCESS: return "GGML status: success";
        case GGML_STATUS_ABORTED: return "GGML status: warning (operation aborted)";
    }
    return "GGML status: unknown";
}

float ggml_fp16_to_fp32(ggml_fp16_t h) { return f16_bits_to_f32(h); }
ggml_fp16_t ggml_fp32_to_fp16(float f) { return f32_to_f16_bits(f); }
void ggml_fp16_to_fp32_row(const ggml_fp16_t *x, float *y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = f16_bits_to_f32(x[i]);
}
void ggml_fp32_to_fp16_row(const float *x, ggml_fp16_t *y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = f32_to_f16_bits(x[i]);
}

// ---- tensor queries -----------------------------------------------------------------------------

int64_t ggml_nelements(const struct ggml_tensor *t) { return t->ne[0] * t->ne[1] * t->ne[2] * t->ne[3]; }
int64_t ggml_nrows(const struct ggml_tensor *t) { return t->ne[1] * t->ne[2] * t->ne[3]; }

size_t ggml_nbytes(const struct ggml_tensor *t) {
    for (int i = 0; i < GGML_MAX_DIMS; ++i)
        if (t->ne[i] <= 0) return 0;
    const int64_t blck = ggml_blck_size(t->type);
    size_t n;
    if (blck == 1) {
        n = ggml_type_size(t->type);
        for (int i = 0; i < GGML_MAX_DIMS; ++i) n += static_cast<size_t>(t->ne[i] - 1) * t->nb[i];
    } else {
        n = static_cast<size_t>(t->ne[0]) * t->nb[0] / static_cast<size_t>(blck);
        for (int i = 1; i < GGML_MAX_DIMS; ++i) n += static_cast<size_t>(t->ne[i] - 1) * t->nb[i];
    }
    return n;
}

int ggml_n_dims(const struct ggml_tensor *t) {
    for (int i = GGML_MAX_DIMS - 1; i >= 1; --i)
        if (t->ne[i] > 1) return i + 1;
    return 1;
}

bool ggml_is_contiguous(const struct ggml_tensor *t) {
    size_t next = ggml_type_size(t->type);
    if (t->ne[0] != ggml_blck_size(t->type) && t->nb[0] != next) return false;
    next *= static_cast<size_t>(t->ne[0] / ggml_blck_size(t->type));
    for (int i = 1; i < GGML_MAX_DIMS; ++i) {
        if (t->ne[i] != 1) {
            if (t->nb[i] != next) return false;
            next *= static_cast<size_t>(t->ne[i]);
        }
    }
    return true;
}

bool ggml_is_empty(const struct ggml_tensor *t) {
    for (int i = 0; i < GGML_MAX_DIMS; ++i)
        if (t->ne[i] == 0) return true;
    return false;
}

enum ggml_unary_op ggml_get_unary_op(const struct ggml_tensor *t) {
    MINI_ASSERT(t->op == GGML_OP_UNARY);
    return static_cast<ggml_unary_op>(t->op_params[0]);
}

const char *ggml_get_name(const struct ggml_tensor *t) { return t->name; }

struct ggml_tensor *ggml_set_name(struct ggml_tensor *t, const char *name) {
    std::snprintf(t->name, sizeof t->name, "%s", name);
    return t;
}

void ggml_set_input(struct ggml_tensor *t) { t->flags |= GGML_TENSOR_FLAG_INPUT; }
void ggml_set_output(struct ggml_tensor *t) { t->flags |= GGML_TENSOR_FLAG_OUTPUT; }
void *ggml_get_data(const struct ggml_tensor *t) { return t->data; }

// ---- contexts -----------------------------------------------------------------------------------

size_t ggml_tensor_overhead(void) { return sizeof(ggml_tensor) + 32; }
size_t ggml_graph_overhead_custom(size_t size, bool) { return 64 + size * 3 * sizeof(void *); }
size_t ggml_graph_overhead(void) { return ggml_graph_overhead_custom(GGML_DEFAULT_GRAPH_SIZE, false); }

struct ggml_context *ggml_init(struct ggml_init_params params) {
    auto *ctx = new ggml_context();
    ctx->mem_size = params.mem_size;
    ctx->no_alloc = params.no_alloc;
    return ctx;
}

void ggml_free(struct ggml_context *ctx) { delete ctx; }

struct ggml_tensor *ggml_get_tensor(struct ggml_context *ctx, const char *name) {
    for (auto &t : ctx->tensors)
        if (std::strcmp(t.name, name) == 0) return &t;
    return nullptr;
}

struct ggml_tensor *ggml_get_first_tensor(const struct ggml_context *ctx) {
    return ctx->tensors.empty() ? nullptr : const_cast<ggml_tensor *>(&ctx->tensors.front());
}

struct ggml_tensor *ggml_get_next_tensor(const struct ggml_context *ctx, struct ggml_tensor *t) {
    for (size_t i = 0; i + 1 < ctx->tensors.size(); ++i)
        if (&ctx->tensors[i] == t) return const_cast<ggml_tensor *>(&ctx->tensors[i + 1]);
    return nullptr;
}

struct ggml_tensor *ggml_new_tensor(struct ggml_context *ctx, enum ggml_type type, int n_dims, const int64_t *ne) {
    return new_tensor_impl(ctx, type, n_dims, ne, nullptr, 0);
}
struct ggml_tensor *ggml_new_tensor_1d(struct ggml_context *ctx, enum ggml_type type, int64_t ne0) {
    return new_tensor(ctx, type, ne0);
}
struct ggml_tensor *ggml_new_tensor_2d(struct ggml_context *ctx, enum ggml_type type, int64_t ne0, int64_t ne1) {
    return new_tensor(ctx, type, ne0, ne1);
}
struct ggml_tensor *ggml_new_tensor_3d(struct ggml_context *ctx, enum ggml_type type, int64_t ne0, int64_t ne1,
                                       int64_t ne2) {
    return new_tensor(ctx, type, ne0, ne1, ne2);
}
struct ggml_tensor *ggml_new_tensor_4d(struct ggml_context *ctx, enum ggml_type type, int64_t ne0, int64_t ne1,
                                       int64_t ne2, int64_t ne3) {
    return new_tensor(ctx, type, ne0, ne1, ne2, ne3);
}
struct ggml_tensor *ggml_dup_tensor(struct ggml_context *ctx, const struct ggml_tensor *src) {
    return new_tensor_impl(ctx, src->type, GGML_MAX_DIMS, src->ne, nullptr, 0);
}
struct ggml_tensor *ggml_view_tensor(struct ggml_context *ctx, struct ggml_tensor *src) {
    ggml_tensor *r = new_tensor_impl(ctx, src->type, GGML_MAX_DIMS, src->ne, src, 0);
    std::memcpy(r->nb, src->nb, sizeof r->nb);
    return r;
}

// ---- graph builders -----------------------------------------------------------------------------

struct ggml_tensor *ggml_add(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b) {
    return binary(ctx, GGML_OP_ADD, a, b, false);
}
struct ggml_tensor *ggml_add_inplace(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b) {
    return binary(ctx, GGML_OP_ADD, a, b, true);
}
struct ggml_tensor *ggml_sub(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b) {
    return binary(ctx, GGML_OP_SUB, a, b, false);
}
struct ggml_tensor *ggml_mul(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b) {
    return binary(ctx, GGML_OP_MUL, a, b, false);
}
struct ggml_tensor *ggml_mul_inplace(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b) {
    return binary(ctx, GGML_OP_MUL, a, b, true);
}

struct ggml_tensor *ggml_scale(struct ggml_context *ctx, struct ggml_tensor *a, float s) {
    ggml_tensor *r = ggml_dup_tensor(ctx, a);
    r->op = GGML_OP_SCALE;
    set_param_f32(r, 0, s);
    set_param_f32(r, 1, 0.0f);
    r->src[0] = a;
    return r;
}

struct ggml_tensor *ggml_repeat(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b) {
    MINI_ASSERT(can_repeat(a, b));
    ggml_tensor *r = new_tensor_impl(ctx, a->type, GGML_MAX_DIMS, b->ne, nullptr, 0);
    r->op = GGML_OP_REPEAT;
    r->src[0] = a;
    return r;
}

struct ggml_tensor *ggml_concat(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b, int dim) {
    MINI_ASSERT(dim >= 0 && dim < GGML_MAX_DIMS && a->type == b->type);
    int64_t ne[GGML_MAX_DIMS];
    for (int d = 0; d < GGML_MAX_DIMS; ++d) {
        if (d == dim) {
            ne[d] = a->ne[d] + b->ne[d];
        } else {
            MINI_ASSERT(a->ne[d] == b->ne[d]);
            ne[d] = a->ne[d];
        }
    }
    ggml_tensor *r = new_tensor_impl(ctx, a->type, GGML_MAX_DIMS, ne, nullptr, 0);
    r->op = GGML_OP_CONCAT;
    r->op_params[0] = dim;
    r->src[0] = a;
    r->src[1] = b;
    return r;
}

struct ggml_tensor *ggml_norm(struct ggml_context *ctx, struct ggml_tensor *a, float eps) {
    ggml_tensor *r = ggml_dup_tensor(ctx, a);
    r->op = GGML_OP_NORM;
    set_param_f32(r, 0, eps);
    r->src[0] = a;
    return r;
}

struct ggml_tensor *ggml_group_norm(struct ggml_context *ctx, struct ggml_tensor *a, int n_groups, float eps) {
    ggml_tensor *r = ggml_dup_tensor(ctx, a);
    r->op = GGML_OP_GROUP_NORM;
    r->op_params[0] = n_groups;
    set_param_f32(r, 1, eps);
    r->src[0] = a;
    return r;
}

struct ggml_tensor *ggml_mul_mat(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b) {
    MINI_ASSERT(a->ne[0] == b->ne[0] && b->ne[2] % a->ne[2] == 0 && b->ne[3] % a->ne[3] == 0);
    ggml_tensor *r = new_tensor(ctx, GGML_TYPE_F32, a->ne[1], b->ne[1], b->ne[2], b->ne[3]);
    r->op = GGML_OP_MUL_MAT;
    r->src[0] = a;
    r->src[1] = b;
    return r;
}

struct ggml_tensor *ggml_relu(struct ggml_context *ctx, struct ggml_tensor *a) {
    return unary(ctx, a, GGML_UNARY_OP_RELU);
}
struct ggml_tensor *ggml_sigmoid(struct ggml_context *ctx, struct ggml_tensor *a) {
    return unary(ctx, a, GGML_UNARY_OP_SIGMOID);
}
struct ggml_tensor *ggml_gelu(struct ggml_context *ctx, struct ggml_tensor *a) {
    return unary(ctx, a, GGML_UNARY_OP_GELU);
}
struct ggml_tensor *ggml_gelu_erf(struct ggml_context *ctx, struct ggml_tensor *a) {
    return unary(ctx, a, GGML_UNARY_OP_GELU_ERF);
}

struct ggml_tensor *ggml_soft_max_ext(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *mask,
                                      float scale, float max_bias) {
    ggml_tensor *r = ggml_dup_tensor(ctx, a);
    r->op = GGML_OP_SOFT_MAX;
    set_param_f32(r, 0, scale);
    set_param_f32(r, 1, max_bias);
    r->src[0] = a;
    r->src[1] = mask;
    return r;
}

struct ggml_tensor *ggml_cont(struct ggml_context *ctx, struct ggml_tensor *a) {
    ggml_tensor *r = ggml_dup_tensor(ctx, a);
    r->op = GGML_OP_CONT;
    r->src[0] = a;
    return r;
}

struct ggml_tensor *ggml_cpy(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b) {
    MINI_ASSERT(ggml_nelements(a) == ggml_nelements(b));
    ggml_tensor *r = ggml_view_tensor(ctx, b);
    r->op = GGML_OP_CPY;
    r->src[0] = a;
    r->src[1] = b;
    return r;
}

struct ggml_tensor *ggml_cast(struct ggml_context *ctx, struct ggml_tensor *a, enum ggml_type type) {
    ggml_tensor *r = new_tensor_impl(ctx, type, GGML_MAX_DIMS, a->ne, nullptr, 0);
    r->op = GGML_OP_CPY;
    r->src[0] = a;
    r->src[1] = r;
    return r;
}

struct ggml_tensor *ggml_reshape_1d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0) {
    const int64_t ne[1] = {ne0};
    return reshape_impl(ctx, a, 1, ne);
}
struct ggml_tensor *ggml_reshape_2d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, int64_t ne1) {
    const int64_t ne[2] = {ne0, ne1};
    return reshape_impl(ctx, a, 2, ne);
}
struct ggml_tensor *ggml_reshape_3d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, int64_t ne1,
                                    int64_t ne2) {
    const int64_t ne[3] = {ne0, ne1, ne2};
    return reshape_impl(ctx, a, 3, ne);
}
struct ggml_tensor *ggml_reshape_4d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, int64_t ne1,
                                    int64_t ne2, int64_t ne3) {
    const int64_t ne[4] = {ne0, ne1, ne2, ne3};
    return reshape_impl(ctx, a, 4, ne);
}

struct ggml_tensor *ggml_view_1d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, size_t offset) {
    const int64_t ne[1] = {ne0};
    return view_impl(ctx, a, 1, ne, offset);
}
struct ggml_tensor *ggml_view_2d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, int64_t ne1,
                                 size_t nb1, size_t offset) {
    const int64_t ne[2] = {ne0, ne1};
    ggml_tensor *r = view_impl(ctx, a, 2, ne, offset);
    r->nb[1] = nb1;
    r->nb[2] = r->nb[1] * static_cast<size_t>(ne1);
    r->nb[3] = r->nb[2];
    return r;
}
struct ggml_tensor *ggml_view_3d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, int64_t ne1,
                                 int64_t ne2, size_t nb1, size_t nb2, size_t offset) {
    const int64_t ne[3] = {ne0, ne1, ne2};
    ggml_tensor *r = view_impl(ctx, a, 3, ne, offset);
    r->nb[1] = nb1;
    r->nb[2] = nb2;
    r->nb[3] = r->nb[2] * static_cast<size_t>(ne2);
    return r;
}
struct ggml_tensor *ggml_view_4d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, int64_t ne1,
                                 int64_t ne2, int64_t ne3, size_t nb1, size_t nb2, size_t nb3, size_t offset) {
    const int64_t ne[4] = {ne0, ne1, ne2, ne3};
    ggml_tensor *r = view_impl(ctx, a, 4, ne, offset);
    r->nb[1] = nb1;
    r->nb[2] = nb2;
    r->nb[3] = nb3;
    return r;
}

struct ggml_tensor *ggml_permute(struct ggml_context *ctx, struct ggml_tensor *a, int axis0, int axis1, int axis2,
                                 int axis3) {
    const int ax[4] = {axis0, axis1, axis2, axis3};
    for (int i = 0; i < 4; ++i) MINI_ASSERT(ax[i] >= 0 && ax[i] < 4);
    MINI_ASSERT(axis0 != axis1 && axis0 != axis2 && axis0 != axis3 && axis1 != axis2 && axis1 != axis3 &&
                axis2 != axis3);
    ggml_tensor *r = ggml_view_tensor(ctx, a);
    for (int i = 0; i < 4; ++i) {
        r->ne[ax[i]] = a->ne[i];
        r->nb[ax[i]] = a->nb[i];
    }
    r->op = GGML_OP_PERMUTE;
    r->src[0] = a;
    for (int i = 0; i < 4; ++i) r->op_params[i] = ax[i];
    return r;
}

struct ggml_tensor *ggml_transpose(struct ggml_context *ctx, struct ggml_tensor *a) {
    ggml_tensor *r = ggml_view_tensor(ctx, a);
    r->ne[0] = a->ne[1];
    r->ne[1] = a->ne[0];
    r->nb[0] = a->nb[1];
    r->nb[1] = a->nb[0];
    r->op = GGML_OP_TRANSPOSE;
    r->src[0] = a;
    return r;
}

struct ggml_tensor *ggml_get_rows(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b) {
    MINI_ASSERT(a->ne[2] == b->ne[1] && b->type == GGML_TYPE_I32);
    ggml_tensor *r = new_tensor(ctx, GGML_TYPE_F32, a->ne[0], b->ne[0], b->ne[1], b->ne[2]);
    r->op = GGML_OP_GET_ROWS;
    r->src[0] = a;
    r->src[1] = b;
    return r;
}

struct ggml_tensor *ggml_win_part(struct ggml_context *ctx, struct ggml_tensor *a, int w) {
    MINI_ASSERT(a->ne[3] == 1 && a->type == GGML_TYPE_F32);
    const int px = (w - a->ne[1] % w) % w, py = (w - a->ne[2] % w) % w;
    const int npx = (px + a->ne[1]) / w, npy = (py + a->ne[2]) / w;
    ggml_tensor *r = new_tensor(ctx, GGML_TYPE_F32, a->ne[0], w, w, npx * npy);
    r->op = GGML_OP_WIN_PART;
    r->op_params[0] = npx;
    r->op_params[1] = npy;
    r->op_params[2] = w;
    r->src[0] = a;
    return r;
}

struct ggml_tensor *ggml_win_unpart(struct ggml_context *ctx, struct ggml_tensor *a, int w0, int h0, int w) {
    MINI_ASSERT(a->type == GGML_TYPE_F32);
    ggml_tensor *r = new_tensor(ctx, GGML_TYPE_F32, a->ne[0], w0, h0, 1);
    r->op = GGML_OP_WIN_UNPART;
    r->op_params[0] = w;
    r->src[0] = a;
    return r;
}

struct ggml_tensor *ggml_flash_attn_ext(struct ggml_context *ctx, struct ggml_tensor *q, struct ggml_tensor *k,
                                        struct ggml_tensor *v, struct ggml_tensor *mask, float scale,
                                        float max_bias, float logit_softcap) {
    MINI_ASSERT(k->ne[0] == q->ne[0] && k->ne[1] == v->ne[1] && q->ne[2] % k->ne[2] == 0);
    ggml_tensor *r = new_tensor(ctx, GGML_TYPE_F32, v->ne[0], q->ne[2], q->ne[1], q->ne[3]);
    r->op = GGML_OP_FLASH_ATTN_EXT;
    set_param_f32(r, 0, scale);
    set_param_f32(r, 1, max_bias);
    set_param_f32(r, 2, logit_softcap);
    r->src[0] = q;
    r->src[1] = k;
    r->src[2] = v;
    r->src[3] = mask;
    return r;
}

struct ggml_tensor *ggml_im2col(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b, int s0,
                                int s1, int p0, int p1, int d0, int d1, bool is_2D, enum ggml_type dst_type) {
    if (is_2D) MINI_ASSERT(a->ne[2] == b->ne[2]);
    const int64_t OH = is_2D ? conv_out_size(b->ne[1], a->ne[1], s1, p1, d1) : 0;
    const int64_t OW = conv_out_size(b->ne[0], a->ne[0], s0, p0, d0);
    MINI_ASSERT((!is_2D || OH > 0) && OW > 0);
    ggml_tensor *r = new_tensor(ctx, dst_type, is_2D ? a->ne[2] * a->ne[1] * a->ne[0] : a->ne[1] * a->ne[0], OW,
                                is_2D ? OH : b->ne[2], is_2D ? b->ne[3] : 1);
    const int32_t p[7] = {s0, s1, p0, p1, d0, d1, is_2D ? 1 : 0};
    std::memcpy(r->op_params, p, sizeof p);
    r->op = GGML_OP_IM2COL;
    r->src[0] = a;
    r->src[1] = b;
    return r;
}

// ggml_conv_2d: the im2col form -- columns [IC*KH*KW, OW, OH, N] of the kernel's type, a MUL_MAT of the
// columns with the kernel as [IC*KH*KW, OC], then [OW, OH, N, OC] permuted to [OW, OH, OC, N]
struct ggml_tensor *ggml_conv_2d(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b, int s0,
                                 int s1, int p0, int p1, int d0, int d1) {
    ggml_tensor *col = ggml_im2col(ctx, a, b, s0, s1, p0, p1, d0, d1, true, a->type);
    ggml_tensor *r = ggml_mul_mat(ctx, ggml_reshape_2d(ctx, col, col->ne[0], col->ne[3] * col->ne[2] * col->ne[1]),
                                  ggml_reshape_2d(ctx, a, a->ne[0] * a->ne[1] * a->ne[2], a->ne[3]));
    r = ggml_reshape_4d(ctx, r, col->ne[1], col->ne[2], col->ne[3], a->ne[3]);
    return ggml_cont(ctx, ggml_permute(ctx, r, 0, 1, 3, 2));
}

struct ggml_tensor *ggml_conv_2d_sk_p0(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b) {
    return ggml_conv_2d(ctx, a, b, static_cast<int>(a->ne[0]), static_cast<int>(a->ne[1]), 0, 0, 1, 1);
}

struct ggml_tensor *ggml_conv_2d_s1_ph(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b) {
    return ggml_conv_2d(ctx, a, b, 1, 1, static_cast<int>(a->ne[0] / 2), static_cast<int>(a->ne[1] / 2), 1, 1);
}

struct ggml_tensor *ggml_conv_2d_direct(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b,
                                        int s0, int s1, int p0, int p1, int d0, int d1) {
    MINI_ASSERT(a->ne[2] == b->ne[2]);
    ggml_tensor *r = new_tensor(ctx, GGML_TYPE_F32, conv_out_size(b->ne[0], a->ne[0], s0, p0, d0),
                                conv_out_size(b->ne[1], a->ne[1], s1, p1, d1), a->ne[3], b->ne[3]);
    const int32_t p[6] = {s0, s1, p0, p1, d0, d1};
    std::memcpy(r->op_params, p, sizeof p);
    r->op = GGML_OP_CONV_2D;
    r->src[0] = a;
    r->src[1] = b;
    return r;
}

struct ggml_tensor *ggml_conv_2d_dw_direct(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b,
                                           int s0, int s1, int p0, int p1, int d0, int d1) {
    MINI_ASSERT(a->ne[2] == 1 && a->ne[3] == b->ne[2]);
    ggml_tensor *r = new_tensor(ctx, b->type, conv_out_size(b->ne[0], a->ne[0], s0, p0, d0),
                                conv_out_size(b->ne[1], a->ne[1], s1, p1, d1), b->ne[2], b->ne[3]);
    // an input whose channels are innermost in memory (CWHN) gives a result laid out the same way
    if (b->nb[2] == ggml_type_size(b->type) && b->nb[0] == b->ne[2] * b->nb[2]) {
        const size_t ts = ggml_type_size(r->type);
        r->nb[0] = static_cast<size_t>(r->ne[2]) * ts;
        r->nb[1] = static_cast<size_t>(r->ne[0]) * r->nb[0];
        r->nb[2] = ts;
    }
    const int32_t p[6] = {s0, s1, p0, p1, d0, d1};
    std::memcpy(r->op_params, p, sizeof p);
    r->op = GGML_OP_CONV_2D_DW;
    r->src[0] = a;
    r->src[1] = b;
    return r;
}

struct ggml_tensor *ggml_conv_transpose_2d_p0(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b,
                                              int stride) {
    MINI_ASSERT(a->ne[3] == b->ne[2]);
    ggml_tensor *r = new_tensor(ctx, GGML_TYPE_F32, (b->ne[0] - 1) * stride + a->ne[0],
                                (b->ne[1] - 1) * stride + a->ne[1], a->ne[2], b->ne[3]);
    r->op_params[0] = stride;
    r->op = GGML_OP_CONV_TRANSPOSE_2D;
    r->src[0] = a;
    r->src[1] = b;
    return r;
}

struct ggml_tensor *ggml_pool_2d(struct ggml_context *ctx, struct ggml_tensor *a, enum ggml_op_pool op, int k0,
                                 int k1, int s0, int s1, float p0, float p1) {
    const int64_t ow = static_cast<int64_t>((a->ne[0] + 2 * p0 - k0) / s0 + 1);
    const int64_t oh = static_cast<int64_t>((a->ne[1] + 2 * p1 - k1) / s1 + 1);
    ggml_tensor *r = new_tensor(ctx, GGML_TYPE_F32, ow, oh, a->ne[2], a->ne[3]);
    const int32_t p[7] = {op, k0, k1, s0, s1, static_cast<int32_t>(p0), static_cast<int32_t>(p1)};
    std::memcpy(r->op_params, p, sizeof p);
    r->op = GGML_OP_POOL_2D;
    r->src[0] = a;
    return r;
}

struct ggml_tensor *ggml_pad_ext(struct ggml_context *ctx, struct ggml_tensor *a, int lp0, int rp0, int lp1, int rp1,
                                 int lp2, int rp2, int lp3, int rp3) {
    ggml_tensor *r = new_tensor(ctx, a->type, a->ne[0] + lp0 + rp0, a->ne[1] + lp1 + rp1, a->ne[2] + lp2 + rp2,
                                a->ne[3] + lp3 + rp3);
    const int32_t p[8] = {lp0, rp0, lp1, rp1, lp2, rp2, lp3, rp3};
    std::memcpy(r->op_params, p, sizeof p);
    r->op = GGML_OP_PAD;
    r->src[0] = a;
    return r;
}

struct ggml_tensor *ggml_pad(struct ggml_context *ctx, struct ggml_tensor *a, int p0, int p1, int p2, int p3) {
    return ggml_pad_ext(ctx, a, 0, p0, 0, p1, 0, p2, 0, p3);
}

struct ggml_tensor *ggml_upscale(struct ggml_context *ctx, struct ggml_tensor *a, int scale_factor,
                                 enum ggml_scale_mode mode) {
    MINI_ASSERT(scale_factor > 0);
    ggml_tensor *r = new_tensor(ctx, a->type, a->ne[0] * scale_factor, a->ne[1] * scale_factor, a->ne[2], a->ne[3]);
    r->op_params[0] = mode;
    r->op = GGML_OP_UPSCALE;
    r->src[0] = a;
    return r;
}

// ---- graphs -------------------------------------------------------------------------------------

struct ggml_cgraph *ggml_new_graph_custom(struct ggml_context *ctx, size_t size, bool) {
    ctx->used += ggml_graph_overhead_custom(size, false);
    MINI_ASSERT(ctx->used <= ctx->mem_size);
    ctx->graphs.emplace_back();
    ctx->graphs.back().size = size;
    return &ctx->graphs.back();
}

struct ggml_cgraph *ggml_new_graph(struct ggml_context *ctx) {
    return ggml_new_graph_custom(ctx, GGML_DEFAULT_GRAPH_SIZE, false);
}

void ggml_build_forward_expand(struct ggml_cgraph *cgraph, struct ggml_tensor *tensor) { visit(cgraph, tensor); }

int ggml_graph_n_nodes(struct ggml_cgraph *cgraph) { return static_cast<int>(cgraph->nodes.size()); }

struct ggml_tensor *ggml_graph_node(struct ggml_cgraph *cgraph, int i) {
    const int n = static_cast<int>(cgraph->nodes.size());
    if (i < 0) i += n;
    MINI_ASSERT(i >= 0 && i < n);
    return cgraph->nodes[static_cast<size_t>(i)];
}

struct ggml_tensor *ggml_graph_get_tensor(const struct ggml_cgraph *cgraph, const char *name) {
    for (auto *t : cgraph->leafs)
        if (std::strcmp(t->name, name) == 0) return t;
    for (auto *t : cgraph->nodes)
        if (std::strcmp(t->name, name) == 0) return t;
    return nullptr;
}

// ---- backend dispatch ---------------------------------------------------------------------------

const char *ggml_backend_buft_name(ggml_backend_buffer_type_t buft) { return buft->iface.get_name(buft); }

ggml_backend_buffer_t ggml_backend_buft_alloc_buffer(ggml_backend_buffer_type_t buft, size_t size) {
    return buft->iface.alloc_buffer(buft, size);
}

size_t ggml_backend_buft_get_alignment(ggml_backend_buffer_type_t buft) { return buft->iface.get_alignment(buft); }

size_t ggml_backend_buft_get_alloc_size(ggml_backend_buffer_type_t buft, const struct ggml_tensor *tensor) {
    return buft->iface.get_alloc_size ? buft->iface.get_alloc_size(buft, tensor) : ggml_nbytes(tensor);
}

bool ggml_backend_buft_is_host(ggml_backend_buffer_type_t buft) {
    return buft->iface.is_host ? buft->iface.is_host(buft) : false;
}

ggml_backend_dev_t ggml_backend_buft_get_device(ggml_backend_buffer_type_t buft) { return buft->device; }

ggml_backend_buffer_t ggml_backend_buffer_init(ggml_backend_buffer_type_t buft, struct ggml_backend_buffer_i iface,
                                               void *context, size_t size) {
    auto *b = new ggml_backend_buffer();
    b->iface = iface;
    b->buft = buft;
    b->context = context;
    b->size = size;
    b->usage = GGML_BACKEND_BUFFER_USAGE_ANY;
    return b;
}

void ggml_backend_buffer_free(ggml_backend_buffer_t buffer) {
    if (!buffer) return;
    if (buffer->iface.free_buffer) buffer->iface.free_buffer(buffer);
    delete buffer;
}

void *ggml_backend_buffer_get_base(ggml_backend_buffer_t buffer) { return buffer->iface.get_base(buffer); }
size_t ggml_backend_buffer_get_size(ggml_backend_buffer_t buffer) { return buffer->size; }

enum ggml_status ggml_backend_buffer_init_tensor(ggml_backend_buffer_t buffer, struct ggml_tensor *tensor) {
    return buffer->iface.init_tensor ? buffer->iface.init_tensor(buffer, tensor) : GGML_STATUS_SUCCESS;
}

void ggml_backend_buffer_clear(ggml_backend_buffer_t buffer, uint8_t value) {
    if (buffer->size) buffer->iface.clear(buffer, value);
}

void ggml_backend_buffer_set_usage(ggml_backend_buffer_t buffer, enum ggml_backend_buffer_usage usage) {
    buffer->usage = usage;
}

enum ggml_backend_buffer_usage ggml_backend_buffer_get_usage(ggml_backend_buffer_t buffer) { return buffer->usage; }
ggml_backend_buffer_type_t ggml_backend_buffer_get_type(ggml_backend_buffer_t buffer) { return buffer->buft; }

const char *ggml_backend_name(ggml_backend_t backend) { return backend ? backend->iface.get_name(backend) : "NULL"; }

void ggml_backend_free(ggml_backend_t backend) {
    if (backend) backend->iface.free(backend);
}

ggml_backend_buffer_type_t ggml_backend_get_default_buffer_type(ggml_backend_t backend) {
    return backend->device->iface.get_buffer_type(backend->device);
}

ggml_backend_buffer_t ggml_backend_alloc_buffer(ggml_backend_t backend, size_t size) {
    return ggml_backend_buft_alloc_buffer(ggml_backend_get_default_buffer_type(backend), size);
}

void ggml_backend_synchronize(ggml_backend_t backend) {
    if (backend->iface.synchronize) backend->iface.synchronize(backend);
}

enum ggml_status ggml_backend_graph_compute(ggml_backend_t backend, struct ggml_cgraph *cgraph) {
    const ggml_status st = backend->iface.graph_compute(backend, cgraph);
    ggml_backend_synchronize(backend);
    return st;
}

ggml_backend_dev_t ggml_backend_get_device(ggml_backend_t backend) { return backend->device; }

bool ggml_backend_dev_supports_op(ggml_backend_dev_t device, const struct ggml_tensor *op) {
    return device->iface.supports_op(device, op);
}

bool ggml_backend_supports_op(ggml_backend_t backend, const struct ggml_tensor *op) {
    return ggml_backend_dev_supports_op(backend->device, op);
}

static ggml_backend_buffer_t buffer_of(const ggml_tensor *t) { return t->view_src ? t->view_src->buffer : t->buffer; }

void ggml_backend_tensor_set(struct ggml_tensor *tensor, const void *data, size_t offset, size_t size) {
    ggml_backend_buffer_t buf = buffer_of(tensor);
    if (size == 0) return;
    MINI_ASSERT(buf != nullptr && tensor->data != nullptr);
    MINI_ASSERT(offset + size <= ggml_nbytes(tensor));
    buf->iface.set_tensor(buf, tensor, data, offset, size);
}

void ggml_backend_tensor_get(const struct ggml_tensor *tensor, void *data, size_t offset, size_t size) {
    ggml_backend_buffer_t buf = buffer_of(tensor);
    if (size == 0) return;
    MINI_ASSERT(buf != nullptr && tensor->data != nullptr);
    MINI_ASSERT(offset + size <= ggml_nbytes(tensor));
    buf->iface.get_tensor(buf, tensor, data, offset, size);
}

void ggml_backend_tensor_memset(struct ggml_tensor *tensor, uint8_t value, size_t offset, size_t size) {
    ggml_backend_buffer_t buf = buffer_of(tensor);
    if (size == 0) return;
    MINI_ASSERT(buf != nullptr && tensor->data != nullptr && buf->iface.memset_tensor != nullptr);
    MINI_ASSERT(offset + size <= ggml_nbytes(tensor));
    buf->iface.memset_tensor(buf, tensor, value, offset, size);
}

static size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// views take their data from their (already placed) source
static void init_view(ggml_tensor *t) {
    t->buffer = t->view_src->buffer;
    t->data = static_cast<char *>(t->view_src->data) + t->view_offs;
    ggml_backend_buffer_init_tensor(t->buffer, t);
}

ggml_backend_buffer_t ggml_backend_alloc_ctx_tensors_from_buft(struct ggml_context *ctx,
                                                               ggml_backend_buffer_type_t buft) {
    const size_t align = ggml_backend_buft_get_alignment(buft);
    size_t total = 0;
    for (auto &t : ctx->tensors)
        if (!t.data && !t.view_src) total += align_up(ggml_backend_buft_get_alloc_size(buft, &t), align);
    if (total == 0) return nullptr;
    ggml_backend_buffer_t buf = ggml_backend_buft_alloc_buffer(buft, total);
    if (!buf) return nullptr;
    char *base = static_cast<char *>(ggml_backend_buffer_get_base(buf));
    size_t off = 0;
    for (auto &t : ctx->tensors) {
        if (t.data || t.view_src) continue;
        t.data = base + off;
        t.buffer = buf;
        ggml_backend_buffer_init_tensor(buf, &t);
        off += align_up(ggml_backend_buft_get_alloc_size(buft, &t), align);
    }
    for (auto &t : ctx->tensors)
        if (t.view_src && !t.data && t.view_src->data) init_view(&t);
    return buf;
}

ggml_backend_buffer_t ggml_backend_alloc_ctx_tensors(struct ggml_context *ctx, ggml_backend_t backend) {
    return ggml_backend_alloc_ctx_tensors_from_buft(ctx, ggml_backend_get_default_buffer_type(backend));
}

// ---- allocators ---------------------------------------------------------------------------------

struct ggml_tallocr ggml_tallocr_new(ggml_backend_buffer_t buffer) {
    ggml_tallocr t;
    t.buffer = buffer;
    t.base = ggml_backend_buffer_get_base(buffer);
    t.alignment = ggml_backend_buft_get_alignment(buffer->buft);
    t.offset = align_up(reinterpret_cast<uintptr_t>(t.base), t.alignment) - reinterpret_cast<uintptr_t>(t.base);
    return t;
}

enum ggml_status ggml_tallocr_alloc(struct ggml_tallocr *talloc, struct ggml_tensor *tensor) {
    const size_t size = align_up(ggml_backend_buft_get_alloc_size(talloc->buffer->buft, tensor), talloc->alignment);
    if (talloc->offset + size > ggml_backend_buffer_get_size(talloc->buffer)) {
        std::fprintf(stderr, "ggml_tallocr_alloc: not enough space in the buffer for %s (%zu bytes)\n", tensor->name,
                     size);
        return GGML_STATUS_ALLOC_FAILED;
    }
    tensor->data = static_cast<char *>(talloc->base) + talloc->offset;
    tensor->buffer = talloc->buffer;
    talloc->offset += size;
    return ggml_backend_buffer_init_tensor(talloc->buffer, tensor);
}

// One buffer for the graph's tensors without data, each at its own offset (no reuse between nodes,
// so every intermediate stays readable after the graph ran).
struct ggml_gallocr {
    ggml_backend_buffer_type_t buft = nullptr;
    ggml_backend_buffer_t buffer = nullptr;
};

ggml_gallocr_t ggml_gallocr_new(ggml_backend_buffer_type_t buft) {
    auto *g = new ggml_gallocr();
    g->buft = buft;
    return g;
}

void ggml_gallocr_free(ggml_gallocr_t galloc) {
    if (!galloc) return;
    ggml_backend_buffer_free(galloc->buffer);
    delete galloc;
}

static bool needs_place(const ggml_tensor *t, const ggml_backend_buffer_t own) {
    return !t->view_src && (!t->data || (own && t->buffer == own));
}

static size_t graph_bytes(ggml_gallocr_t g, ggml_cgraph *graph) {
    const size_t align = ggml_backend_buft_get_alignment(g->buft);
    size_t total = 0;
    for (auto *list : {&graph->leafs, &graph->nodes})
        for (auto *t : *list)
            if (needs_place(t, g->buffer)) total += align_up(ggml_backend_buft_get_alloc_size(g->buft, t), align);
    return total;
}

bool ggml_gallocr_reserve(ggml_gallocr_t galloc, struct ggml_cgraph *graph) {
    const size_t need = graph_bytes(galloc, graph);
    if (galloc->buffer && ggml_backend_buffer_get_size(galloc->buffer) >= need) return true;
    // a larger buffer: tensors placed in the old one must be placed again
    for (auto *list : {&graph->leafs, &graph->nodes})
        for (auto *t : *list)
            if (galloc->buffer && t->buffer == galloc->buffer) {
                t->data = nullptr;
                t->buffer = nullptr;
            }
    ggml_backend_buffer_free(galloc->buffer);
    galloc->buffer = ggml_backend_buft_alloc_buffer(galloc->buft, need ? need : 1);
    if (galloc->buffer) ggml_backend_buffer_set_usage(galloc->buffer, GGML_BACKEND_BUFFER_USAGE_COMPUTE);
    return galloc->buffer != nullptr;
}

bool ggml_gallocr_alloc_graph(ggml_gallocr_t galloc, struct ggml_cgraph *graph) {
    if (!ggml_gallocr_reserve(galloc, graph)) return false;
    const size_t align = ggml_backend_buft_get_alignment(galloc->buft);
    char *base = static_cast<char *>(ggml_backend_buffer_get_base(galloc->buffer));
    size_t off = 0;
    auto place = [&](ggml_tensor *t) {
        if (t->view_src) {
            if (t->view_src->data) init_view(t);
            return;
        }
        if (!needs_place(t, galloc->buffer)) return;
        t->data = base + off;
        t->buffer = galloc->buffer;
        ggml_backend_buffer_init_tensor(galloc->buffer, t);
        off += align_up(ggml_backend_buft_get_alloc_size(galloc->buft, t), align);
    };
    for (auto *t : graph->leafs) place(t);
    for (auto *t : graph->nodes) {
        for (int s = 0; s < GGML_MAX_SRC; ++s)
            if (t->src[s] && t->src[s]->view_src && !t->src[s]->data) place(t->src[s]);
        place(t);
    }
    return true;
}

size_t ggml_gallocr_get_buffer_size(ggml_gallocr_t galloc, int buffer_id) {
    return buffer_id == 0 && galloc->buffer ? ggml_backend_buffer_get_size(galloc->buffer) : 0;
}

}  // extern "C"
