// A ggml caller of the B200 backend, built by tests/test_ggml_backend*.py against the ggml-compatible
// headers (sam3.cpp_b200/ggml) and linked with libggml_b200.so + libggml_mini.so.
//
// vit_block_graph() builds the graph of one SAM3 ViT block node for node as sam3_vit_block_forward
// builds it (sam3.cpp:3714-3805), with sam3_layer_norm (sam3.cpp:1041-1051) and the RoPE of
// sam3_apply_rope (sam3.cpp:3671-3710) as ggml ops, places the weights in a B200 buffer through
// ggml_backend_alloc_ctx_tensors + ggml_backend_tensor_set, allocates the graph with ggml_gallocr
// on the backend's default buffer type and runs it with ggml_backend_graph_compute -- the calls
// sam3.cpp makes (sam3.cpp:3320, 6101-6119, 1019-1030).
#include "ggml-alloc.h"
#include "ggml-b200.h"
#include "ggml-backend.h"
#include "ggml.h"

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>

namespace {

struct Block {
    ggml_tensor *norm1_w, *norm1_b, *norm2_w, *norm2_b;
    ggml_tensor *qkv_w, *qkv_b, *proj_w, *proj_b, *fc1_w, *fc1_b, *fc2_w, *fc2_b;
    ggml_tensor *freqs;  // [2, HD/2, tokens of one attention window]
};

ggml_tensor *layer_norm(ggml_context *ctx, ggml_tensor *x, ggml_tensor *w, ggml_tensor *b) {
    x = ggml_norm(ctx, x, 1e-5f);
    x = ggml_mul_inplace(ctx, x, w);
    return ggml_add_inplace(ctx, x, b);
}

// x [HD, N, heads*B]; freqs [2, HD/2, N] of (cos, sin) pairs
ggml_tensor *rope(ggml_context *ctx, ggml_tensor *x, ggml_tensor *freqs) {
    const int64_t hd = x->ne[0], n = x->ne[1], nhb = x->ne[2], half = hd / 2;
    ggml_tensor *pairs = ggml_reshape_4d(ctx, x, 2, half, n, nhb);
    ggml_tensor *fc = ggml_reshape_4d(ctx, freqs, 2, half, n, 1);
    ggml_tensor *c = ggml_view_4d(ctx, fc, 1, half, n, 1, fc->nb[1], fc->nb[2], fc->nb[3], 0);
    ggml_tensor *s = ggml_view_4d(ctx, fc, 1, half, n, 1, fc->nb[1], fc->nb[2], fc->nb[3], fc->nb[0]);
    ggml_tensor *re = ggml_view_4d(ctx, pairs, 1, half, n, nhb, pairs->nb[1], pairs->nb[2], pairs->nb[3], 0);
    ggml_tensor *im = ggml_view_4d(ctx, pairs, 1, half, n, nhb, pairs->nb[1], pairs->nb[2], pairs->nb[3],
                                   pairs->nb[0]);
    ggml_tensor *out_re = ggml_sub(ctx, ggml_mul(ctx, re, c), ggml_mul(ctx, im, s));
    ggml_tensor *out_im = ggml_add(ctx, ggml_mul(ctx, re, s), ggml_mul(ctx, im, c));
    ggml_tensor *out = ggml_concat(ctx, out_re, out_im, 0);
    return ggml_reshape_3d(ctx, ggml_cont(ctx, out), hd, n, nhb);
}

// x [E, W, H, 1]; window 0 = global attention
ggml_tensor *block_forward(ggml_context *ctx, ggml_tensor *x, const Block &blk, int E, int NH, int window) {
    const int HD = E / NH;
    ggml_tensor *shortcut = x;
    x = layer_norm(ctx, x, blk.norm1_w, blk.norm1_b);
    const int64_t w0 = x->ne[1], h0 = x->ne[2];
    if (window) x = ggml_win_part(ctx, x, window);
    const int64_t W = x->ne[1], H = x->ne[2], B = x->ne[3];
    {
        ggml_tensor *cur = ggml_mul_mat(ctx, blk.qkv_w, x);
        cur = ggml_add(ctx, cur, blk.qkv_b);
        cur = ggml_reshape_4d(ctx, cur, E, 3, W * H, B);
        cur = ggml_cont(ctx, ggml_permute(ctx, cur, 0, 3, 1, 2));
        ggml_tensor *Q = ggml_view_3d(ctx, cur, E, W * H, B, cur->nb[1], cur->nb[2], 0);
        ggml_tensor *K = ggml_view_3d(ctx, cur, E, W * H, B, cur->nb[1], cur->nb[2], cur->nb[3]);
        ggml_tensor *V = ggml_view_3d(ctx, cur, E, W * H, B, cur->nb[1], cur->nb[2], 2 * cur->nb[3]);
        Q = ggml_reshape_4d(ctx, Q, HD, NH, W * H, B);
        Q = ggml_cont(ctx, ggml_permute(ctx, Q, 0, 2, 1, 3));
        Q = ggml_reshape_3d(ctx, Q, HD, W * H, NH * B);
        K = ggml_reshape_4d(ctx, K, HD, NH, W * H, B);
        K = ggml_cont(ctx, ggml_permute(ctx, K, 0, 2, 1, 3));
        K = ggml_reshape_3d(ctx, K, HD, W * H, NH * B);
        V = ggml_reshape_4d(ctx, V, HD, NH, W * H, B);
        V = ggml_permute(ctx, V, 0, 2, 1, 3);
        Q = rope(ctx, Q, blk.freqs);
        K = rope(ctx, K, blk.freqs);
        Q = ggml_reshape_4d(ctx, Q, HD, W * H, NH, B);
        K = ggml_reshape_4d(ctx, K, HD, W * H, NH, B);
        ggml_tensor *attn = ggml_flash_attn_ext(ctx, Q, K, V, nullptr, 1.0f / std::sqrt(static_cast<float>(HD)),
                                                0.0f, 0.0f);
        x = ggml_reshape_4d(ctx, attn, E, W, H, B);
        x = ggml_mul_mat(ctx, blk.proj_w, x);
        x = ggml_add(ctx, x, blk.proj_b);
    }
    if (window) x = ggml_win_unpart(ctx, x, static_cast<int>(w0), static_cast<int>(h0), window);
    x = ggml_add(ctx, shortcut, x);
    shortcut = x;
    x = layer_norm(ctx, x, blk.norm2_w, blk.norm2_b);
    x = ggml_mul_mat(ctx, blk.fc1_w, x);
    x = ggml_add(ctx, x, blk.fc1_b);
    x = ggml_gelu_erf(ctx, x);
    x = ggml_mul_mat(ctx, blk.fc2_w, x);
    x = ggml_add(ctx, x, blk.fc2_b);
    return ggml_add(ctx, shortcut, x);
}

Block new_block(ggml_context *ctx, int E, int mlp, int NH, int tokens, ggml_type wtype) {
    Block b;
    b.norm1_w = ggml_new_tensor_1d(ctx, GGML_TYPE_F32, E);
    b.norm1_b = ggml_new_tensor_1d(ctx, GGML_TYPE_F32, E);
    b.norm2_w = ggml_new_tensor_1d(ctx, GGML_TYPE_F32, E);
    b.norm2_b = ggml_new_tensor_1d(ctx, GGML_TYPE_F32, E);
    b.qkv_w = ggml_new_tensor_2d(ctx, wtype, E, 3 * E);
    b.qkv_b = ggml_new_tensor_1d(ctx, GGML_TYPE_F32, 3 * E);
    b.proj_w = ggml_new_tensor_2d(ctx, wtype, E, E);
    b.proj_b = ggml_new_tensor_1d(ctx, GGML_TYPE_F32, E);
    b.fc1_w = ggml_new_tensor_2d(ctx, wtype, E, mlp);
    b.fc1_b = ggml_new_tensor_1d(ctx, GGML_TYPE_F32, mlp);
    b.fc2_w = ggml_new_tensor_2d(ctx, wtype, mlp, E);
    b.fc2_b = ggml_new_tensor_1d(ctx, GGML_TYPE_F32, E);
    b.freqs = ggml_new_tensor_3d(ctx, GGML_TYPE_F32, 2, E / NH / 2, tokens);
    return b;
}

struct Graph {
    ggml_context *wctx = nullptr, *cctx = nullptr;
    Block blk;
    ggml_tensor *x = nullptr, *out = nullptr;
    ggml_cgraph *gf = nullptr;
};

// hp = E, heads, G (the map is G x G tokens), window (0 = global), weight ggml_type, mlp
Graph build(const int32_t *hp) {
    Graph g;
    const int E = hp[0], NH = hp[1], G = hp[2], window = hp[3], mlp = hp[5];
    const ggml_type wtype = static_cast<ggml_type>(hp[4]);
    ggml_init_params wp = {ggml_tensor_overhead() * 16, nullptr, true};
    g.wctx = ggml_init(wp);
    g.blk = new_block(g.wctx, E, mlp, NH, window ? window * window : G * G, wtype);
    ggml_init_params cp = {ggml_tensor_overhead() * 512 + ggml_graph_overhead(), nullptr, true};
    g.cctx = ggml_init(cp);
    g.x = ggml_new_tensor_4d(g.cctx, GGML_TYPE_F32, E, G, G, 1);
    ggml_set_input(g.x);
    g.out = block_forward(g.cctx, g.x, g.blk, E, NH, window);
    ggml_set_output(g.out);
    g.gf = ggml_new_graph(g.cctx);
    ggml_build_forward_expand(g.gf, g.out);
    return g;
}

void release(Graph &g) {
    ggml_free(g.cctx);
    ggml_free(g.wctx);
}

}  // namespace

extern "C" {

// Host-only: the number of graph nodes and how many of them the B200 device accepts
// (ggml_backend_dev_supports_op); the first refused node's op name goes to `first_refused`.
int vit_block_graph_check(const int32_t *hp, int32_t *n_nodes, int32_t *n_supported, char *first_refused,
                          int cap) {
    Graph g = build(hp);
    ggml_backend_buffer_type_t buft = ggml_backend_b200_buffer_type(0);
    if (!buft) return -1;
    const int n = ggml_graph_n_nodes(g.gf);
    int ok = 0;
    first_refused[0] = 0;
    for (int i = 0; i < n; ++i) {
        ggml_tensor *t = ggml_graph_node(g.gf, i);
        if (ggml_backend_dev_supports_op(ggml_backend_buft_get_device(buft), t)) {
            ++ok;
        } else if (!first_refused[0]) {
            std::snprintf(first_refused, static_cast<size_t>(cap), "%s", ggml_op_name(t->op));
        }
    }
    *n_nodes = n;
    *n_supported = ok;
    release(g);
    return 0;
}

// weights: qkv, proj, fc1, fc2 blocks (ggml rows of the weight type); vecs: qkv_b, proj_b, fc1_b,
// fc2_b, norm1_w, norm1_b, norm2_w, norm2_b; freqs [tokens][HD/2][2]; x and out [G*G][E] f32.
// Returns the ggml_status of the compute (or -10 on a setup failure).
int vit_block_graph_run(int device, const int32_t *hp, const void *const *weights, const float *const *vecs,
                        const float *freqs, const float *x, float *out, int32_t *n_nodes) {
    Graph g = build(hp);
    ggml_backend_t backend = ggml_backend_b200_init(device);
    if (!backend) {
        release(g);
        return -10;
    }
    int st = -10;
    ggml_backend_buffer_t wbuf = ggml_backend_alloc_ctx_tensors(g.wctx, backend);
    ggml_gallocr_t galloc = ggml_gallocr_new(ggml_backend_get_default_buffer_type(backend));
    if (wbuf && galloc) {
        ggml_backend_buffer_set_usage(wbuf, GGML_BACKEND_BUFFER_USAGE_WEIGHTS);
        ggml_tensor *mats[4] = {g.blk.qkv_w, g.blk.proj_w, g.blk.fc1_w, g.blk.fc2_w};
        for (int i = 0; i < 4; ++i) ggml_backend_tensor_set(mats[i], weights[i], 0, ggml_nbytes(mats[i]));
        ggml_tensor *v[8] = {g.blk.qkv_b, g.blk.proj_b, g.blk.fc1_b, g.blk.fc2_b,
                             g.blk.norm1_w, g.blk.norm1_b, g.blk.norm2_w, g.blk.norm2_b};
        for (int i = 0; i < 8; ++i) ggml_backend_tensor_set(v[i], vecs[i], 0, ggml_nbytes(v[i]));
        ggml_backend_tensor_set(g.blk.freqs, freqs, 0, ggml_nbytes(g.blk.freqs));
        if (ggml_gallocr_alloc_graph(galloc, g.gf)) {
            ggml_backend_tensor_set(g.x, x, 0, ggml_nbytes(g.x));
            st = ggml_backend_graph_compute(backend, g.gf);
            if (st == GGML_STATUS_SUCCESS) ggml_backend_tensor_get(g.out, out, 0, ggml_nbytes(g.out));
        }
    }
    *n_nodes = ggml_graph_n_nodes(g.gf);
    ggml_gallocr_free(galloc);
    ggml_backend_buffer_free(wbuf);
    ggml_backend_free(backend);
    release(g);
    return st;
}

}  // extern "C"
