// graph.cu -- the backend's supports_op and graph_compute over flattened ggml
// graph nodes (sam3b200_tensor, include/sam3_b200.h).
//
// sam3.cpp reaches every kernel through ggml_backend_graph_compute
// (sam3.cpp:1019-1030), which hands the backend the nodes of one graph in
// execution order.  This file is that executor for the ops the B200 backend
// owns: MUL_MAT (with the bias ADD that follows every linear layer fused into
// it, sam3.cpp:3742-3743), FLASH_ATTN_EXT (:3778), CONV_TRANSPOSE_2D (:3884),
// CONV_2D (:3819) and GET_ROWS (the text encoder's token rows).  Views run
// nothing (their data already aliases their source).  The whole graph is
// checked before anything is launched, so a rejected graph leaves the device
// untouched; each node then runs through the same entry point a direct caller
// uses, so results are those of the op-level entries.
#include "../../include/sam3_b200.h"
#include "backend_impl.h"

#include <cstdarg>
#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <unordered_map>

static_assert(sizeof(sam3b200_tensor) == 192, "sam3b200_tensor layout is part of the C ABI");
static_assert(offsetof(sam3b200_tensor, src) == 144, "sam3b200_tensor layout is part of the C ABI");

namespace b200 {
namespace {

using T = sam3b200_tensor;

// Bytes of one ggml block and elements per block (ggml's type traits for the
// types this backend reads).
bool type_traits(int type, size_t *block_bytes, int64_t *block_elems) {
    switch (type) {
        case SAM3B200_TYPE_F32: *block_bytes = 4; *block_elems = 1; return true;
        case SAM3B200_TYPE_F16: *block_bytes = 2; *block_elems = 1; return true;
        case SAM3B200_TYPE_I32: *block_bytes = 4; *block_elems = 1; return true;
        case SAM3B200_TYPE_Q4_0: *block_bytes = 18; *block_elems = 32; return true;
        case SAM3B200_TYPE_Q4_1: *block_bytes = 20; *block_elems = 32; return true;
        case SAM3B200_TYPE_Q8_0: *block_bytes = 34; *block_elems = 32; return true;
        default: return false;
    }
}

bool shape_ok(const T *t) {
    for (int d = 0; d < 4; ++d)
        if (t->ne[d] < 1 || t->ne[d] > (1ll << 31)) return false;
    return true;
}

bool is_empty(const T *t) {
    for (int d = 0; d < 4; ++d)
        if (t->ne[d] == 0) return true;
    return false;
}

// ggml_is_contiguous: strides are the packed ones of the type.
bool contiguous(const T *t) {
    size_t bb;
    int64_t be;
    if (!type_traits(t->type, &bb, &be) || t->ne[0] % be != 0) return false;
    size_t expect = bb;
    if (t->nb[0] != expect) return false;
    expect = bb * static_cast<size_t>(t->ne[0] / be);
    for (int d = 1; d < 4; ++d) {
        if (t->ne[d] > 1 && t->nb[d] != expect) return false;
        expect *= static_cast<size_t>(t->ne[d]);
    }
    return true;
}

// Byte stride between consecutive rows of an f32 tensor whose dims 1..3 are
// read as one run of ne1*ne2*ne3 rows (ggml_mul_mat broadcasting a 2-D weight
// over them); 0 if those dims do not flatten to one evenly strided run or the
// elements of a row are not packed.
size_t flat_row_stride(const T *t) {
    if (t->type != SAM3B200_TYPE_F32 || t->nb[0] != 4) return 0;
    size_t stride = 0, next = 0;
    for (int d = 1; d < 4; ++d) {
        if (t->ne[d] == 1) continue;
        if (stride == 0) stride = t->nb[d];
        else if (t->nb[d] != next) return 0;
        next = t->nb[d] * static_cast<size_t>(t->ne[d]);
    }
    if (stride == 0) stride = static_cast<size_t>(t->ne[0]) * 4;  // one row
    if (stride % 4 != 0 || stride < static_cast<size_t>(t->ne[0]) * 4) return 0;
    return stride;
}

int64_t rows_of(const T *t) { return t->ne[1] * t->ne[2] * t->ne[3]; }

float param_f32(const T *t, int i) {
    float f;
    std::memcpy(&f, &t->op_params[i], sizeof f);
    return f;
}

bool attn_dim_ok(int64_t D) {
    return D == 16 || D == 32 || D == 48 || D == 56 || D == 64 || D == 72 || D == 96 || D == 112 || D == 128 ||
           D == 256;
}

__attribute__((format(printf, 3, 4))) bool reject(char *why, size_t cap, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(why, cap, fmt, ap);
    va_end(ap);
    return false;
}

// The node-local rules of each op; on failure `why` says which.
bool check_node(const T *n, char *why, size_t cap) {
    if (!n) return reject(why, cap, "null node");
    const T *a = n->src[0], *b = n->src[1];
    switch (n->op) {
        case SAM3B200_OP_NONE: return true;
        case SAM3B200_OP_VIEW: return a ? true : reject(why, cap, "VIEW without a source");
        case SAM3B200_OP_MUL_MAT: {
            if (!a || !b) return reject(why, cap, "MUL_MAT needs src0 (weight) and src1 (x)");
            if (a->type != SAM3B200_TYPE_Q8_0 && a->type != SAM3B200_TYPE_Q4_0 && a->type != SAM3B200_TYPE_Q4_1 &&
                a->type != SAM3B200_TYPE_F16 && a->type != SAM3B200_TYPE_F32)
                return reject(why, cap, "MUL_MAT weight type %d (F32, F16, Q4_0, Q4_1, Q8_0)", a->type);
            if (!shape_ok(a) || a->ne[2] != 1 || a->ne[3] != 1 || !contiguous(a))
                return reject(why, cap, "MUL_MAT weight must be a contiguous 2-D tensor");
            const bool quant = a->type != SAM3B200_TYPE_F16 && a->type != SAM3B200_TYPE_F32;
            if (a->ne[0] % (quant ? 32 : 8) != 0)
                return reject(why, cap, "MUL_MAT K=%lld is not a multiple of %d", (long long)a->ne[0], quant ? 32 : 8);
            if (b->type != SAM3B200_TYPE_F32 || !shape_ok(b) || b->ne[0] != a->ne[0])
                return reject(why, cap, "MUL_MAT x must be f32 with ne0 == K=%lld", (long long)a->ne[0]);
            if (!flat_row_stride(b)) return reject(why, cap, "MUL_MAT x rows do not flatten to one strided run");
            if (n->type != SAM3B200_TYPE_F32 || n->ne[0] != a->ne[1] || n->ne[1] != b->ne[1] ||
                n->ne[2] != b->ne[2] || n->ne[3] != b->ne[3])
                return reject(why, cap, "MUL_MAT result must be f32 [N, ne1, ne2, ne3] of x");
            if (!flat_row_stride(n)) return reject(why, cap, "MUL_MAT result rows do not flatten to one strided run");
            if (rows_of(b) > (1 << 24)) return reject(why, cap, "MUL_MAT with more than 2^24 rows");
            return true;
        }
        case SAM3B200_OP_ADD: {
            if (!a || !b || a->op != SAM3B200_OP_MUL_MAT)
                return reject(why, cap, "ADD runs here only as the bias add of a MUL_MAT (src0 = the MUL_MAT)");
            if (b->type != SAM3B200_TYPE_F32 || b->ne[0] != a->ne[0] || b->ne[1] != 1 || b->ne[2] != 1 ||
                b->ne[3] != 1 || b->nb[0] != 4)
                return reject(why, cap, "ADD bias must be a packed f32 vector of the MUL_MAT's %lld outputs",
                              (long long)a->ne[0]);
            if (n->type != SAM3B200_TYPE_F32 || std::memcmp(n->ne, a->ne, sizeof n->ne) != 0 || !flat_row_stride(n))
                return reject(why, cap, "ADD result must be f32 of the MUL_MAT's shape with rows in one strided run");
            return true;
        }
        case SAM3B200_OP_FLASH_ATTN_EXT: {
            const T *v = n->src[2], *m = n->src[3];
            if (!a || !b || !v) return reject(why, cap, "FLASH_ATTN_EXT needs q, k and v");
            const int64_t D = a->ne[0], NQ = a->ne[1], NKV = b->ne[1], H = a->ne[2], B = a->ne[3];
            for (const T *t : {a, b, v})
                if (t->type != SAM3B200_TYPE_F32 || !shape_ok(t) || t->nb[0] != 4 || t->nb[1] % 4 || t->nb[2] % 4 ||
                    t->nb[3] % 4)
                    return reject(why, cap, "FLASH_ATTN_EXT q, k, v must be f32 with packed rows");
            if (b->ne[0] != D || v->ne[0] != D || v->ne[1] != NKV || b->ne[2] != H || v->ne[2] != H ||
                b->ne[3] != B || v->ne[3] != B)
                return reject(why, cap, "FLASH_ATTN_EXT k, v must be [D, NKV, heads, batch] of q's D, heads and batch");
            if (!attn_dim_ok(D))
                return reject(why, cap, "FLASH_ATTN_EXT head dim %lld (16, 32, 48, 56, 64, 72, 96, 112, 128, 256)",
                              (long long)D);
            if (NQ > (1 << 24) || NKV > (1 << 24) || H * B > 65535) return reject(why, cap, "FLASH_ATTN_EXT too large");
            if (param_f32(n, 1) != 0.f || param_f32(n, 2) != 0.f)
                return reject(why, cap, "FLASH_ATTN_EXT with max_bias or logit softcap (sam3.cpp uses neither)");
            if (m && (m->type != SAM3B200_TYPE_F16 || !shape_ok(m) || m->ne[0] != NKV || m->ne[1] < NQ ||
                      m->ne[2] != 1 || m->ne[3] != 1 || m->nb[0] != 2 || m->nb[1] % 2))
                return reject(why, cap, "FLASH_ATTN_EXT mask must be F16 [NKV, >= NQ] shared by every head");
            if (n->type != SAM3B200_TYPE_F32 || n->ne[0] != D || n->ne[1] != H || n->ne[2] != NQ || n->ne[3] != B ||
                !contiguous(n))
                return reject(why, cap, "FLASH_ATTN_EXT result must be contiguous f32 [D, heads, NQ, batch]");
            return true;
        }
        case SAM3B200_OP_CONV_TRANSPOSE_2D: {
            if (!a || !b) return reject(why, cap, "CONV_TRANSPOSE_2D needs the kernel and the input");
            const int s = n->op_params[0];
            if (a->type != SAM3B200_TYPE_F16 || !shape_ok(a) || !contiguous(a))
                return reject(why, cap, "CONV_TRANSPOSE_2D kernel must be contiguous F16 [KW, KH, OC, IC]");
            if (b->type != SAM3B200_TYPE_F32 || !shape_ok(b) || !contiguous(b) || b->ne[2] != a->ne[3] ||
                b->ne[3] != 1)
                return reject(why, cap, "CONV_TRANSPOSE_2D input must be contiguous f32 [IW, IH, IC, 1]");
            if (s <= 0) return reject(why, cap, "CONV_TRANSPOSE_2D stride %d", s);
            const int64_t ow = (b->ne[0] - 1) * s + a->ne[0], oh = (b->ne[1] - 1) * s + a->ne[1];
            if (n->type != SAM3B200_TYPE_F32 || n->ne[0] != ow || n->ne[1] != oh || n->ne[2] != a->ne[2] ||
                n->ne[3] != 1 || !contiguous(n))
                return reject(why, cap, "CONV_TRANSPOSE_2D result must be contiguous f32 [%lld, %lld, OC, 1]",
                              (long long)ow, (long long)oh);
            return true;
        }
        case SAM3B200_OP_CONV_2D: {
            if (!a || !b) return reject(why, cap, "CONV_2D needs the kernel and the input");
            const int32_t *p = n->op_params;  // s0, s1, p0, p1, d0, d1
            if (a->type != SAM3B200_TYPE_F16 || !shape_ok(a) || !contiguous(a))
                return reject(why, cap, "CONV_2D kernel must be contiguous F16 [KW, KH, IC, OC]");
            if (b->type != SAM3B200_TYPE_F32 || !shape_ok(b) || !contiguous(b) || b->ne[2] != a->ne[2] ||
                b->ne[3] != 1)
                return reject(why, cap, "CONV_2D input must be contiguous f32 [IW, IH, IC, 1]");
            if (p[0] <= 0 || p[1] <= 0 || p[2] < 0 || p[3] < 0 || p[4] <= 0 || p[5] <= 0)
                return reject(why, cap, "CONV_2D stride/padding/dilation (%d %d %d %d %d %d)", p[0], p[1], p[2],
                              p[3], p[4], p[5]);
            // span of the last kernel start; negative = the dilated kernel overhangs the padded input
            const int64_t span_w = b->ne[0] + 2 * p[2] - p[4] * (a->ne[0] - 1) - 1;
            const int64_t span_h = b->ne[1] + 2 * p[3] - p[5] * (a->ne[1] - 1) - 1;
            if (span_w < 0 || span_h < 0) return reject(why, cap, "CONV_2D kernel larger than the padded input");
            const int64_t ow = span_w / p[0] + 1, oh = span_h / p[1] + 1;
            if (n->type != SAM3B200_TYPE_F32 || n->ne[0] != ow || n->ne[1] != oh || n->ne[2] != a->ne[3] ||
                n->ne[3] != 1 || !contiguous(n))
                return reject(why, cap, "CONV_2D result must be contiguous f32 [%lld, %lld, OC, 1]", (long long)ow,
                              (long long)oh);
            return true;
        }
        case SAM3B200_OP_GET_ROWS: {
            if (!a || !b) return reject(why, cap, "GET_ROWS needs the rows and the indices");
            size_t bb;
            int64_t be;
            if (a->type == SAM3B200_TYPE_I32 || !type_traits(a->type, &bb, &be))
                return reject(why, cap, "GET_ROWS source type %d (F32, F16, Q4_0, Q4_1, Q8_0)", a->type);
            if (!shape_ok(a) || a->ne[2] != 1 || a->ne[3] != 1 || !contiguous(a))
                return reject(why, cap, "GET_ROWS source must be a contiguous 2-D tensor");
            if (b->type != SAM3B200_TYPE_I32 || !shape_ok(b) || b->ne[1] != 1 || b->ne[2] != 1 || b->ne[3] != 1 ||
                !contiguous(b))
                return reject(why, cap, "GET_ROWS indices must be a contiguous I32 vector");
            if (n->type != SAM3B200_TYPE_F32 || n->ne[0] != a->ne[0] || n->ne[1] != b->ne[0] || n->ne[2] != 1 ||
                n->ne[3] != 1 || !contiguous(n))
                return reject(why, cap, "GET_ROWS result must be contiguous f32 [ncols, n]");
            return true;
        }
        default: return reject(why, cap, "op %d is not executed by this backend", n->op);
    }
}

bool computes(const T *n) { return n->op != SAM3B200_OP_NONE && n->op != SAM3B200_OP_VIEW && !is_empty(n); }

bool aligned16(const void *p) { return p && (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace b200

using namespace b200;

extern "C" int sam3b200_supports_op(const sam3b200_tensor *node) {
    char why[256];
    if (node && is_empty(node)) return 1;  // empty nodes run nothing
    return check_node(node, why, sizeof why) ? 1 : 0;
}

extern "C" int sam3b200_graph_compute(sam3b200_backend *h, sam3b200_tensor *const *nodes, int n_nodes) {
    if (n_nodes < 0 || (n_nodes > 0 && !nodes)) {
        set_error("graph_compute: null node list");
        return SAM3B200_STATUS_FAILED;
    }
    char why[256];
    // pass 1: every node on its own, then the fusion rule of ADD
    std::unordered_map<const T *, int> uses;
    for (int i = 0; i < n_nodes; ++i) {
        const T *n = nodes[i];
        if (!n) {
            set_error("graph_compute: node %d is null", i);
            return SAM3B200_STATUS_FAILED;
        }
        for (const T *s : n->src)
            if (s) ++uses[s];
    }
    for (int i = 0; i < n_nodes; ++i) {
        const T *n = nodes[i];
        if (is_empty(n)) continue;
        if (!check_node(n, why, sizeof why)) {
            set_error("graph_compute: node %d rejected: %s", i, why);
            return SAM3B200_STATUS_FAILED;
        }
        if (n->op == SAM3B200_OP_ADD) {
            const T *mm = n->src[0];
            if (i == 0 || nodes[i - 1] != mm || (mm->flags & SAM3B200_TENSOR_FLAG_OUTPUT) || uses[mm] != 1) {
                set_error("graph_compute: node %d rejected: ADD runs only fused into the MUL_MAT just before it, "
                          "whose result nothing else reads and which is not an output",
                          i);
                return SAM3B200_STATUS_FAILED;
            }
        }
    }
    // pass 2: device data of every node that computes, and the uploaded weights
    // (a MUL_MAT fused with its ADD writes the ADD's result, never its own)
    for (int i = 0; i < n_nodes; ++i) {
        const T *n = nodes[i];
        if (!computes(n)) continue;
        const bool fused = n->op == SAM3B200_OP_MUL_MAT && i + 1 < n_nodes && nodes[i + 1]->op == SAM3B200_OP_ADD &&
                           nodes[i + 1]->src[0] == n;
        if (!fused && !aligned16(n->data)) {
            set_error("graph_compute: node %d rejected: result data is null or not 16-byte aligned", i);
            return SAM3B200_STATUS_FAILED;
        }
        for (int s = 0; s < 4; ++s) {
            const T *src = n->src[s];
            if (!src || (n->op == SAM3B200_OP_MUL_MAT && s == 0) || (n->op == SAM3B200_OP_ADD && s == 0)) continue;
            if (!aligned16(src->data)) {
                set_error("graph_compute: node %d rejected: src%d data is null or not 16-byte aligned", i, s);
                return SAM3B200_STATUS_FAILED;
            }
        }
        if (n->op == SAM3B200_OP_MUL_MAT) {
            const T *wt = n->src[0];
            const auto *w = static_cast<const Weight *>(wt->extra);
            if (!w) {
                set_error("graph_compute: node %d rejected: MUL_MAT weight has no handle from sam3b200_weight_upload "
                          "in extra",
                          i);
                return SAM3B200_STATUS_FAILED;
            }
            if (w->type != wt->type || w->K != wt->ne[0] || w->N != wt->ne[1]) {
                set_error("graph_compute: node %d rejected: MUL_MAT weight handle is type %d [%d, %d], the node says "
                          "type %d [%lld, %lld]",
                          i, w->type, w->K, w->N, wt->type, (long long)wt->ne[0], (long long)wt->ne[1]);
                return SAM3B200_STATUS_FAILED;
            }
        }
    }
    auto *be = reinterpret_cast<sam3b200_backend *>(h);
    if (!be) {
        set_error("graph_compute: null backend");
        return SAM3B200_STATUS_FAILED;
    }
    // run the nodes in order
    for (int i = 0; i < n_nodes; ++i) {
        const T *n = nodes[i];
        if (!computes(n)) continue;
        const T *a = n->src[0], *b = n->src[1];
        int st = SAM3B200_STATUS_SUCCESS;
        switch (n->op) {
            case SAM3B200_OP_MUL_MAT: {
                // the bias add right after it runs inside it, writing the ADD's result
                const T *add = i + 1 < n_nodes && nodes[i + 1]->op == SAM3B200_OP_ADD && nodes[i + 1]->src[0] == n
                                   ? nodes[i + 1]
                                   : nullptr;
                const T *out = add ? add : n;
                st = sam3b200_mul_mat(be, static_cast<const sam3b200_weight *>(a->extra),
                                      static_cast<const float *>(b->data), static_cast<int64_t>(flat_row_stride(b) / 4),
                                      rows_of(b), add ? static_cast<const float *>(add->src[1]->data) : nullptr,
                                      static_cast<float *>(out->data), static_cast<int64_t>(flat_row_stride(out) / 4));
                break;
            }
            case SAM3B200_OP_ADD: break;  // ran with its MUL_MAT
            case SAM3B200_OP_FLASH_ATTN_EXT: {
                const T *v = n->src[2], *m = n->src[3];
                const int64_t qn[3] = {static_cast<int64_t>(a->nb[1] / 4), static_cast<int64_t>(a->nb[2] / 4),
                                       static_cast<int64_t>(a->nb[3] / 4)};
                const int64_t kn[3] = {static_cast<int64_t>(b->nb[1] / 4), static_cast<int64_t>(b->nb[2] / 4),
                                       static_cast<int64_t>(b->nb[3] / 4)};
                const int64_t vn[3] = {static_cast<int64_t>(v->nb[1] / 4), static_cast<int64_t>(v->nb[2] / 4),
                                       static_cast<int64_t>(v->nb[3] / 4)};
                st = sam3b200_flash_attn_ext_view(be, static_cast<const float *>(a->data),
                                                  static_cast<const float *>(b->data),
                                                  static_cast<const float *>(v->data), m ? m->data : nullptr,
                                                  m ? static_cast<int64_t>(m->nb[1] / 2) : 0, a->ne[0], a->ne[1],
                                                  b->ne[1], a->ne[2], a->ne[3], qn, kn, vn, param_f32(n, 0),
                                                  static_cast<float *>(n->data));
                break;
            }
            case SAM3B200_OP_CONV_TRANSPOSE_2D:
                st = sam3b200_conv_transpose_2d(be, a->data, static_cast<const float *>(b->data), b->ne[0], b->ne[1],
                                                b->ne[2], a->ne[2], a->ne[0], a->ne[1], n->op_params[0],
                                                static_cast<float *>(n->data));
                break;
            case SAM3B200_OP_CONV_2D: {
                const int32_t *p = n->op_params;
                st = sam3b200_conv_2d(be, a->data, static_cast<const float *>(b->data), b->ne[0], b->ne[1], b->ne[2],
                                      a->ne[3], a->ne[0], a->ne[1], p[0], p[1], p[2], p[3], p[4], p[5],
                                      static_cast<float *>(n->data));
                break;
            }
            case SAM3B200_OP_GET_ROWS:
                st = sam3b200_get_rows(be, a->type, a->data, a->ne[0], a->ne[1], static_cast<const int32_t *>(b->data),
                                       b->ne[0], static_cast<float *>(n->data));
                break;
            default: break;
        }
        if (st != SAM3B200_STATUS_SUCCESS) {
            const std::string msg = sam3b200_last_error();
            sam3b200_backend_synchronize(be);  // let the nodes already queued finish before returning
            set_error("graph_compute: node %d failed: %s", i, msg.c_str());
            return st;
        }
    }
    return sam3b200_backend_synchronize(be);
}
