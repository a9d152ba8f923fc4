"""CPU checks of the graph-level entries (sam3b200_supports_op, sam3b200_graph_compute): the node
layout of the C ABI, which nodes the backend accepts, and the graph rules, all decided on the host
before any device work -- the backend half of ggml_backend_graph_compute (sam3.cpp:1019-1030)."""
import ctypes

import pytest

F32, F16, Q4_0, Q4_1, Q8_0, I32 = 0, 1, 2, 3, 8, 26
A = 1 << 20  # a fake, 16-byte aligned device address: these checks never dereference data


@pytest.fixture(scope="module")
def g(b200):
    b200.lib()
    return b200


def test_node_layout_matches_the_header(g):
    """sam3b200_tensor: 192 bytes, src at 144 (static_assert on the C side)."""
    assert ctypes.sizeof(g.GraphTensor) == 192
    assert g.GraphTensor.src.offset == 144
    assert g.GraphTensor.ne.offset == 8 and g.GraphTensor.nb.offset == 40 and g.GraphTensor.flags.offset == 136


def _mm(g, wtype=Q8_0, K=256, N=96, rows=(40,), data=None):
    w = g.graph_tensor(wtype, [K, N])
    x = g.graph_tensor(F32, [K, *rows], data=A)
    return g.graph_tensor(F32, [N, *rows], op=g.OP_MUL_MAT, src=(w, x), data=data)


def _fa(g, D=64, NQ=48, NKV=48, H=2, B=2, mask=True, params=None):
    nb = [4, 3 * H * D * 4, D * 4, NQ * 3 * H * D * 4]  # views into one [B, N, 3, H, D] qkv tensor
    q = g.graph_tensor(F32, [D, NQ, H, B], nb=nb, data=A)
    k = g.graph_tensor(F32, [D, NKV, H, B], nb=nb, data=A + H * D * 4)
    v = g.graph_tensor(F32, [D, NKV, H, B], nb=nb, data=A + 2 * H * D * 4)
    m = g.graph_tensor(F16, [NKV, NQ], data=A) if mask else None
    params = params if params is not None else (g.f32_bits(0.125), 0, 0)
    return g.graph_tensor(F32, [D, H, NQ, B], op=g.OP_FLASH_ATTN_EXT, src=(q, k, v, m), op_params=params,
                          data=A)


def _conv(g, iw=20, ih=18, ic=32, oc=40, k=3, params=(1, 1, 1, 1, 1, 1), out=None):
    w = g.graph_tensor(F16, [k, k, ic, oc], data=A)
    x = g.graph_tensor(F32, [iw, ih, ic, 1], data=A)
    if out is None:
        s0, s1, p0, p1, d0, d1 = params
        out = [(iw + 2 * p0 - d0 * (k - 1) - 1) // s0 + 1, (ih + 2 * p1 - d1 * (k - 1) - 1) // s1 + 1, oc, 1]
    return g.graph_tensor(F32, out, op=g.OP_CONV_2D, src=(w, x), op_params=params, data=A)


def _convt(g, iw=10, ih=9, ic=40, oc=16, k=2, s=2, out=None):
    w = g.graph_tensor(F16, [k, k, oc, ic], data=A)
    x = g.graph_tensor(F32, [iw, ih, ic, 1], data=A)
    return g.graph_tensor(F32, out or [(iw - 1) * s + k, (ih - 1) * s + k, oc, 1], op=g.OP_CONV_TRANSPOSE_2D,
                          src=(w, x), op_params=(s,), data=A)


def _rows(g, stype=Q4_0, ncols=256, nrows=500, n=32, itype=I32):
    r = g.graph_tensor(stype, [ncols, nrows], data=A)
    i = g.graph_tensor(itype, [n], data=A)
    return g.graph_tensor(F32, [ncols, n], op=g.OP_GET_ROWS, src=(r, i), data=A)


@pytest.mark.parametrize("wtype", [Q8_0, Q4_0, Q4_1, F16, F32])
def test_supports_mul_mat_weight_types(g, wtype):
    assert g.supports_op(_mm(g, wtype))


def test_supports_the_forms_sam3_builds(g):
    assert g.supports_op(_mm(g, rows=(24, 24, 9)))        # windowed activations [K, 24, 24, 9] (sam3.cpp:3742)
    assert g.supports_op(_fa(g))                          # strided q/k/v views + F16 mask
    assert g.supports_op(_fa(g, D=16, NQ=7, NKV=4096, mask=False))  # decoder cross-attention shape
    assert g.supports_op(_conv(g))                        # ggml_conv_2d_s1_ph
    assert g.supports_op(_conv(g, iw=56, ih=42, ic=3, oc=32, k=14, params=(14, 14, 0, 0, 1, 1)))  # patch embed
    assert g.supports_op(_convt(g))
    for t in (F32, F16, Q4_0, Q4_1, Q8_0):
        assert g.supports_op(_rows(g, t))
    mm = _mm(g)
    bias = g.graph_tensor(F32, [96], data=A)
    assert g.supports_op(g.graph_tensor(F32, [96, 40], op=g.OP_ADD, src=(mm, bias), data=A))
    assert g.supports_op(g.graph_tensor(F32, [96, 40], op=g.OP_VIEW, src=(mm,), data=A))
    assert g.supports_op(g.graph_tensor(F32, [96, 40]))   # leaf
    # elementwise ops of the ViT / decoder graphs: residual add, broadcast multiply (LN affine), scale,
    # activations, ggml_norm, and the CONT that materialises a permuted view (sam3.cpp:3747-3767)
    x = g.graph_tensor(F32, [64, 24, 24, 9], data=A)
    row = g.graph_tensor(F32, [64], data=A)
    assert g.supports_op(g.graph_tensor(F32, [64, 24, 24, 9], op=g.OP_ADD, src=(x, x), data=A))
    assert g.supports_op(g.graph_tensor(F32, [64, 24, 24, 9], op=g.OP_MUL, src=(x, row), data=A))
    assert g.supports_op(g.graph_tensor(F32, [64, 24, 24, 9], op=g.OP_SCALE, src=(x,), op_params=(g.f32_bits(0.125),),
                                        data=A))
    for kind in (g.UNARY_RELU, g.UNARY_SIGMOID, g.UNARY_GELU_ERF, g.UNARY_GELU):
        assert g.supports_op(g.graph_tensor(F32, [64, 24, 24, 9], op=g.OP_UNARY, src=(x,), op_params=(kind,), data=A))
    assert g.supports_op(g.graph_tensor(F32, [64, 24, 24, 9], op=g.OP_NORM, src=(x,), op_params=(g.f32_bits(1e-6),),
                                        data=A))
    vmap = g.graph_tensor(F32, [64, 72, 72], data=A)  # ViT windows of 24 (sam3.cpp:3734, 3788); Hiera pads
    wins = g.graph_tensor(F32, [64, 24, 24, 9], op=g.OP_WIN_PART, src=(vmap,), op_params=(3, 3, 24), data=A)
    assert g.supports_op(wins)
    assert g.supports_op(g.graph_tensor(F32, [64, 72, 72], op=g.OP_WIN_UNPART, src=(wins,), op_params=(24,), data=A))
    assert g.supports_op(g.graph_tensor(F32, [96, 8, 8, 4], op=g.OP_WIN_PART, src=(
        g.graph_tensor(F32, [96, 14, 10], data=A),), op_params=(2, 2, 8), data=A))
    scores = g.graph_tensor(F32, [70, 20, 4, 2], data=A)
    for mask in (None, g.graph_tensor(F16, [70, 32], data=A), g.graph_tensor(F32, [70, 20, 4], data=A)):
        assert g.supports_op(g.graph_tensor(F32, [70, 20, 4, 2], op=g.OP_SOFT_MAX, src=(scores, mask),
                                            op_params=(g.f32_bits(0.125), 0), data=A))
    perm = g.graph_tensor(F32, [64, 9, 24, 24], nb=[4, 64 * 24 * 24 * 4, 64 * 4, 64 * 24 * 4], data=A)
    assert g.supports_op(g.graph_tensor(F32, [64, 9, 24, 24], op=g.OP_CONT, src=(perm,), data=A))
    assert g.supports_op(g.graph_tensor(F32, [64 * 9, 576], op=g.OP_CONT, src=(perm,), data=A))  # ggml_cont_2d


def _im2col(g, iw=56, ih=70, ic=3, k=14, s=14, is_2d=1, otype=F16, out=None):
    """The patch embedding's IM2COL (sam3.cpp:6726): kernel [14, 14, 3, OC] (shape only), image [W, H, 3, 1]."""
    w = g.graph_tensor(F16, [k, k, 3, 32])
    x = g.graph_tensor(F32, [iw, ih, ic, 1], data=A)
    out = out or [3 * k * k, (iw - k) // s + 1, (ih - k) // s + 1, 1]
    return g.graph_tensor(otype, out, op=g.OP_IM2COL, src=(w, x), op_params=(s, s, 0, 0, 1, 1, is_2d), data=A)


def _pool(g, op=0, out=None):
    x = g.graph_tensor(F32, [12, 10, 16, 1], data=A)
    return g.graph_tensor(F32, out or [6, 5, 16, 1], op=g.OP_POOL_2D, src=(x,), op_params=(op, 2, 2, 2, 2, 0, 0),
                          data=A)


def _dw(g, ktype=F32, out=None):
    k = g.graph_tensor(ktype, [3, 3, 1, 32], data=A)
    x = g.graph_tensor(F32, [20, 18, 32, 1], data=A)
    return g.graph_tensor(F32, out or [10, 9, 32, 1], op=g.OP_CONV_2D_DW, src=(k, x), op_params=(2, 2, 1, 1, 1, 1),
                          data=A)


def test_supports_the_shape_and_convolution_ops_sam3_builds(g):
    """The rest of the op set sam3.cpp's graphs use around the hot path: RoPE's SUB and CONCAT
    (sam3.cpp:3704-3708), REPEAT of a positional embedding (sam3.cpp:3825), the patch embedding as
    IM2COL + MUL_MAT of two graph tensors (sam3.cpp:6726-6742), attention scores as a batched MUL_MAT
    (sam3.cpp:8584), max and average pools (sam3.cpp:3918, 4748), PAD (sam3.cpp:4210), nearest UPSCALE
    (sam3.cpp:4586), the depthwise convolution (sam3.cpp:9089), GROUP_NORM (sam3.cpp:8923) and casts."""
    x = g.graph_tensor(F32, [64, 20, 4], data=A)
    assert g.supports_op(g.graph_tensor(F32, [64, 20, 4], op=g.OP_SUB, src=(x, g.graph_tensor(F32, [64], data=A)),
                                        data=A))
    assert g.supports_op(g.graph_tensor(F32, [64, 20, 8], op=g.OP_REPEAT, src=(x,), data=A))
    assert g.supports_op(g.graph_tensor(F32, [128, 20, 4], op=g.OP_CONCAT, src=(x, x), op_params=(0,), data=A))
    col = _im2col(g)
    assert g.supports_op(col)
    for otype in (F32, F16):
        assert g.supports_op(_im2col(g, otype=otype))
    patches = g.graph_tensor(F16, [588, 20], data=A)  # the IM2COL result, reshaped 2-D
    kern = g.graph_tensor(F16, [588, 32], data=A)     # patch_embed_w reshaped [KW*KH*IC, OC]
    assert g.supports_op(g.graph_tensor(F32, [20, 32], op=g.OP_MUL_MAT, src=(patches, kern), data=A))
    k = g.graph_tensor(F32, [64, 70, 4, 1], data=A)
    q = g.graph_tensor(F32, [64, 20, 8, 2], data=A)   # heads broadcast over src0's 4 heads, batch 2 over 1
    assert g.supports_op(g.graph_tensor(F32, [70, 20, 8, 2], op=g.OP_MUL_MAT, src=(k, q), data=A))
    assert g.supports_op(_pool(g)) and g.supports_op(_pool(g, op=1))
    assert g.supports_op(g.graph_tensor(F32, [10, 7], op=g.OP_PAD, src=(g.graph_tensor(F32, [8, 4], data=A),),
                                        op_params=(0, 2, 1, 2), data=A))
    assert g.supports_op(g.graph_tensor(F32, [16, 8, 3], op=g.OP_UPSCALE, src=(
        g.graph_tensor(F32, [8, 4, 3], data=A),), data=A))
    assert g.supports_op(_dw(g))
    assert g.supports_op(g.graph_tensor(F32, [8, 8, 32], op=g.OP_GROUP_NORM, src=(
        g.graph_tensor(F32, [8, 8, 32], data=A),), op_params=(8, g.f32_bits(1e-5)), data=A))
    assert g.supports_op(g.graph_tensor(F16, [8, 4], op=g.OP_CONT, src=(g.graph_tensor(F32, [8, 4], data=A),), data=A))
    assert g.supports_op(g.graph_tensor(F32, [32], op=g.OP_CONT, src=(g.graph_tensor(F16, [8, 4], data=A),), data=A))


def test_runtime_mul_mat_reads_its_src0_data(g):
    """A MUL_MAT whose src0 is an F32 / F16 tensor without a weight handle reads src0 from its data: no
    handle is asked for, and src0 needs its data like any other source."""
    a = g.graph_tensor(F32, [64, 70], data=A)
    mm = g.graph_tensor(F32, [70, 20], op=g.OP_MUL_MAT, src=(a, g.graph_tensor(F32, [64, 20], data=A)), data=A)
    assert g.graph_compute_status(None, [mm]) == g.STATUS_FAILED and "null backend" in g.last_error()
    a.data = None
    assert g.graph_compute_status(None, [mm]) == g.STATUS_FAILED
    assert "node 0 rejected: src0 data" in g.last_error(), g.last_error()
    a.data = A + 2  # f32 rows need 4-byte alignment
    assert g.graph_compute_status(None, [mm]) == g.STATUS_FAILED and "not 4-byte aligned" in g.last_error()


def test_im2col_reads_only_its_kernels_shape(g):
    col = _im2col(g)
    assert col.src[0].contents.data is None
    assert g.graph_compute_status(None, [col]) == g.STATUS_FAILED and "null backend" in g.last_error()


def _not_packed_rows(g):
    mm = _mm(g)
    mm.src[1].contents.nb[0] = 8
    return mm


def _bias_of_wrong_length(g):
    return g.graph_tensor(F32, [96, 40], op=g.OP_ADD, src=(_mm(g), g.graph_tensor(F32, [95], data=A)), data=A)


REJECTED = {
    "unknown op": lambda g: g.graph_tensor(F32, [4], op=99, data=A),
    "Q5_0 weight": lambda g: g.graph_tensor(F32, [96, 40], op=g.OP_MUL_MAT, src=(
        g.graph_tensor(6, [256, 96], nb=[22, 176, 176 * 96, 176 * 96]), g.graph_tensor(F32, [256, 40], data=A)),
        data=A),
    "K not a multiple of 32": lambda g: _mm(g, K=48),
    "x ne0 != K": lambda g: g.graph_tensor(F32, [96, 40], op=g.OP_MUL_MAT, src=(
        g.graph_tensor(Q8_0, [256, 96]), g.graph_tensor(F32, [224, 40], data=A)), data=A),
    "x f16": lambda g: g.graph_tensor(F32, [96, 40], op=g.OP_MUL_MAT, src=(
        g.graph_tensor(Q8_0, [256, 96]), g.graph_tensor(F16, [256, 40], data=A)), data=A),
    "x rows not packed": _not_packed_rows,
    "x dims not flattening": lambda g: g.graph_tensor(F32, [96, 4, 5], op=g.OP_MUL_MAT, src=(
        g.graph_tensor(Q8_0, [256, 96]),
        g.graph_tensor(F32, [256, 4, 5], nb=[4, 1024, 8192, 40960], data=A)), data=A),
    "result shape": lambda g: g.graph_tensor(F32, [95, 40], op=g.OP_MUL_MAT, src=(
        g.graph_tensor(Q8_0, [256, 96]), g.graph_tensor(F32, [256, 40], data=A)), data=A),
    "3-D weight": lambda g: g.graph_tensor(F32, [96, 40], op=g.OP_MUL_MAT, src=(
        g.graph_tensor(Q8_0, [256, 96, 2]), g.graph_tensor(F32, [256, 40], data=A)), data=A),
    "ADD of a src1 that does not repeat": lambda g: g.graph_tensor(F32, [96, 40], op=g.OP_ADD, src=(
        g.graph_tensor(F32, [96, 40], data=A), g.graph_tensor(F32, [96, 3], data=A)), data=A),
    "MUL f16": lambda g: g.graph_tensor(F32, [8, 4], op=g.OP_MUL, src=(
        g.graph_tensor(F16, [8, 4], data=A), g.graph_tensor(F32, [8], data=A)), data=A),
    "SCALE result shape": lambda g: g.graph_tensor(F32, [8, 5], op=g.OP_SCALE, src=(
        g.graph_tensor(F32, [8, 4], data=A),), op_params=(g.f32_bits(0.5),), data=A),
    "UNARY kind 9": lambda g: g.graph_tensor(F32, [8, 4], op=g.OP_UNARY, src=(g.graph_tensor(F32, [8, 4], data=A),),
                                             op_params=(9,), data=A),
    "NORM negative eps": lambda g: g.graph_tensor(F32, [8, 4], op=g.OP_NORM, src=(
        g.graph_tensor(F32, [8, 4], data=A),), op_params=(g.f32_bits(-1.0),), data=A),
    "SOFT_MAX max_bias": lambda g: g.graph_tensor(F32, [70, 20, 4], op=g.OP_SOFT_MAX, src=(
        g.graph_tensor(F32, [70, 20, 4], data=A),), op_params=(g.f32_bits(0.125), g.f32_bits(8.0)), data=A),
    "SOFT_MAX mask rows short": lambda g: g.graph_tensor(F32, [70, 20, 4], op=g.OP_SOFT_MAX, src=(
        g.graph_tensor(F32, [70, 20, 4], data=A), g.graph_tensor(F16, [70, 16], data=A)),
        op_params=(g.f32_bits(0.125), 0), data=A),
    "WIN_PART window count param": lambda g: g.graph_tensor(F32, [64, 24, 24, 9], op=g.OP_WIN_PART, src=(
        g.graph_tensor(F32, [64, 72, 72], data=A),), op_params=(3, 2, 24), data=A),
    "WIN_UNPART window count": lambda g: g.graph_tensor(F32, [64, 72, 72], op=g.OP_WIN_UNPART, src=(
        g.graph_tensor(F32, [64, 24, 24, 8], data=A),), op_params=(24,), data=A),
    "CONT from I32": lambda g: g.graph_tensor(F32, [8, 4], op=g.OP_CONT, src=(g.graph_tensor(I32, [8, 4], data=A),),
                                              data=A),
    "CONT element count": lambda g: g.graph_tensor(F32, [8, 5], op=g.OP_CONT, src=(
        g.graph_tensor(F32, [8, 4], data=A),), data=A),
    "ADD bias of the wrong length": _bias_of_wrong_length,
    "attention head dim 80": lambda g: _fa(g, D=80),
    "attention max_bias": lambda g: _fa(g, params=(g.f32_bits(0.125), g.f32_bits(8.0), 0)),
    "attention softcap": lambda g: _fa(g, params=(g.f32_bits(0.125), 0, g.f32_bits(30.0))),
    "attention mask shorter than NQ": lambda g: _fa_short_mask(g),
    "conv channel mismatch": lambda g: _conv_channel_mismatch(g),
    # span -1: C division would truncate it to one output column
    "conv kernel over the padded input": lambda g: _conv(g, iw=6, ih=6, k=7, params=(2, 2, 0, 0, 1, 1),
                                                         out=[1, 1, 40, 1]),
    "conv result shape": lambda g: _conv(g, out=[20, 17, 40, 1]),
    "conv zero stride": lambda g: _conv(g, params=(0, 1, 1, 1, 1, 1), out=[20, 18, 40, 1]),
    "conv transpose result shape": lambda g: _convt(g, out=[20, 17, 16, 1]),
    "runtime MUL_MAT batches that do not broadcast": lambda g: g.graph_tensor(F32, [70, 20, 6], op=g.OP_MUL_MAT,
        src=(g.graph_tensor(F32, [64, 70, 4], data=A), g.graph_tensor(F32, [64, 20, 6], data=A)), data=A),
    "runtime MUL_MAT K mismatch": lambda g: g.graph_tensor(F32, [70, 20], op=g.OP_MUL_MAT, src=(
        g.graph_tensor(F16, [64, 70], data=A), g.graph_tensor(F32, [60, 20], data=A)), data=A),
    "runtime MUL_MAT f16 result": lambda g: g.graph_tensor(F16, [70, 20], op=g.OP_MUL_MAT, src=(
        g.graph_tensor(F32, [64, 70], data=A), g.graph_tensor(F32, [64, 20], data=A)), data=A),
    "SUB shape": lambda g: g.graph_tensor(F32, [8, 5], op=g.OP_SUB, src=(
        g.graph_tensor(F32, [8, 4], data=A), g.graph_tensor(F32, [8], data=A)), data=A),
    "REPEAT not a multiple": lambda g: g.graph_tensor(F32, [8, 6], op=g.OP_REPEAT, src=(
        g.graph_tensor(F32, [8, 4], data=A),), data=A),
    "CONCAT shapes": lambda g: g.graph_tensor(F32, [8, 7], op=g.OP_CONCAT, src=(
        g.graph_tensor(F32, [8, 4], data=A), g.graph_tensor(F32, [8, 4], data=A)), op_params=(1,), data=A),
    "CONCAT dim 4": lambda g: g.graph_tensor(F32, [8, 8], op=g.OP_CONCAT, src=(
        g.graph_tensor(F32, [8, 4], data=A), g.graph_tensor(F32, [8, 4], data=A)), op_params=(4,), data=A),
    "IM2COL 1-D form": lambda g: _im2col(g, is_2d=0),
    "IM2COL result shape": lambda g: _im2col(g, out=[588, 4, 4, 1]),
    "IM2COL channel mismatch": lambda g: _im2col(g, ic=4),
    "POOL_2D op 2": lambda g: _pool(g, op=2),
    "POOL_2D result shape": lambda g: _pool(g, out=[5, 5, 16, 1]),
    "PAD circular": lambda g: g.graph_tensor(F32, [10, 4], op=g.OP_PAD, src=(g.graph_tensor(F32, [8, 4], data=A),),
                                             op_params=(1, 1, 0, 0, 0, 0, 0, 0, 1), data=A),
    "PAD result shape": lambda g: g.graph_tensor(F32, [11, 4], op=g.OP_PAD, src=(g.graph_tensor(F32, [8, 4], data=A),),
                                                 op_params=(1, 1), data=A),
    "UPSCALE bilinear": lambda g: g.graph_tensor(F32, [16, 8], op=g.OP_UPSCALE, src=(
        g.graph_tensor(F32, [8, 4], data=A),), op_params=(1,), data=A),
    "UPSCALE fractional factor": lambda g: g.graph_tensor(F32, [12, 8], op=g.OP_UPSCALE, src=(
        g.graph_tensor(F32, [8, 4], data=A),), data=A),
    "CONV_2D_DW f16 kernel": lambda g: _dw(g, ktype=F16),
    "CONV_2D_DW result shape": lambda g: _dw(g, out=[20, 20, 32, 1]),
    "GROUP_NORM zero groups": lambda g: g.graph_tensor(F32, [8, 8, 32], op=g.OP_GROUP_NORM, src=(
        g.graph_tensor(F32, [8, 8, 32], data=A),), op_params=(0, g.f32_bits(1e-5)), data=A),
    "get_rows f32 indices": lambda g: _rows(g, itype=F32),
    "get_rows Q4_0 with 48 columns": lambda g: _rows(g, Q4_0, ncols=48),
}


def _fa_short_mask(g):
    fa = _fa(g)
    fa.src[3].contents.ne[1] = 40  # NQ = 48
    return fa


def _conv_channel_mismatch(g):
    c = _conv(g)
    c.src[1].contents.ne[2] = 31
    return c


@pytest.mark.parametrize("case", sorted(REJECTED))
def test_rejects(g, case):
    node = REJECTED[case](g)
    assert not g.supports_op(node), case
    assert g.graph_compute_status(None, [node]) == g.STATUS_FAILED
    assert "node 0 rejected" in g.last_error(), g.last_error()


def test_valid_graph_passes_every_check_before_the_backend(g):
    """A graph of supported nodes with aligned data gets as far as the missing backend."""
    nodes = [_conv(g), _convt(g), _rows(g), _fa(g)]
    assert g.graph_compute_status(None, nodes) == g.STATUS_FAILED
    assert "null backend" in g.last_error(), g.last_error()
    assert g.graph_compute_status(None, []) == g.STATUS_FAILED
    assert "null backend" in g.last_error()


def test_unfused_adds_pass_the_checks(g):
    """An ADD away from its MUL_MAT, over an OUTPUT MUL_MAT or over one read twice runs as a plain ADD:
    the graph passes every check (it stops at the missing backend).  The MUL_MAT then needs its own
    aligned result buffer."""
    bias = g.graph_tensor(F32, [96], data=A)
    mm = _mm(g, data=A)
    add = g.graph_tensor(F32, [96, 40], op=g.OP_ADD, src=(mm, bias), data=A)
    graphs = [[mm, _conv(g), add], [mm, add, g.graph_tensor(F32, [96, 40], op=g.OP_VIEW, src=(mm,), data=A)]]
    for nodes in graphs:
        assert g.graph_compute_status(None, nodes) == g.STATUS_FAILED
        assert "no handle" in g.last_error(), g.last_error()  # reached pass 2: the MUL_MAT's weight handle
    mm.flags = g.TENSOR_FLAG_OUTPUT
    mm.data = None
    assert g.graph_compute_status(None, [mm, add]) == g.STATUS_FAILED
    assert "node 0 rejected: result data is null" in g.last_error(), g.last_error()
    mm.flags = 0
    assert g.graph_compute_status(None, [mm, add]) == g.STATUS_FAILED  # fused: the MUL_MAT writes the ADD's data
    assert "no handle" in g.last_error(), g.last_error()


def test_mul_mat_needs_an_uploaded_weight_handle(g):
    mm = _mm(g, data=A)
    assert g.graph_compute_status(None, [mm]) == g.STATUS_FAILED
    assert "node 0 rejected: MUL_MAT weight has no handle" in g.last_error(), g.last_error()


def test_elementwise_data_needs_element_alignment_only(g):
    x = g.graph_tensor(F32, [8, 4], data=A + 4)
    ok = g.graph_tensor(F32, [8, 4], op=g.OP_UNARY, src=(x,), op_params=(g.UNARY_RELU,), data=A + 36)
    assert g.graph_compute_status(None, [ok]) == g.STATUS_FAILED and "null backend" in g.last_error()
    h = g.graph_tensor(F16, [8, 4], data=A + 2)
    assert g.graph_compute_status(None, [g.graph_tensor(F16, [32], op=g.OP_CONT, src=(h,), data=A + 6)]) == \
        g.STATUS_FAILED and "null backend" in g.last_error()
    bad = g.graph_tensor(F32, [8, 4], op=g.OP_UNARY, src=(x,), op_params=(g.UNARY_RELU,), data=A + 2)
    assert g.graph_compute_status(None, [bad]) == g.STATUS_FAILED
    assert "not 4-byte aligned" in g.last_error()


def test_unaligned_or_missing_data_is_rejected(g):
    c = _conv(g)
    c.data = A + 4
    assert g.graph_compute_status(None, [c]) == g.STATUS_FAILED
    assert "node 0 rejected: result data" in g.last_error()
    c = _conv(g)
    c.src[1].contents.data = None
    assert g.graph_compute_status(None, [c]) == g.STATUS_FAILED
    assert "node 0 rejected: src1 data" in g.last_error()


def test_empty_nodes_are_skipped(g):
    """ggml backends skip nodes with a zero dimension; so does this one (even an otherwise odd node)."""
    e = g.graph_tensor(F32, [0, 4], op=99)
    assert g.supports_op(e)
    assert g.graph_compute_status(None, [e]) == g.STATUS_FAILED
    assert "null backend" in g.last_error()


def test_null_node_list_is_rejected(g):
    L = g.lib()
    assert L.sam3b200_graph_compute(None, None, 3) == g.STATUS_FAILED
    assert "null node list" in g.last_error()
