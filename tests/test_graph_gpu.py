"""sam3b200_graph_compute on the GPU: graphs shaped like the ones sam3.cpp hands to
ggml_backend_graph_compute (sam3.cpp:1019-1030) give bit for bit the results of the same ops called
one by one through the op-level entries, and a rejected graph launches nothing."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

F32, F16, Q8_0, I32 = 0, 1, 8, 26


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


def test_get_rows_mul_mat_bias_graph(oracle, b200, backend):
    """Token rows -> linear layer with its bias (the text encoder's first steps; the ADD fused into the
    MUL_MAT), Q8_0 tables and weights, 200 rows (tensor-core MUL_MAT)."""
    rng = np.random.default_rng(11)
    V, K, N, n = 500, 256, 384, 200
    emb_q = oracle.quantize_weights(Q8_0, rng.normal(0, 0.5, size=(V, K)).astype(np.float32))
    w_q = oracle.quantize_weights(Q8_0, rng.normal(0, 0.02, size=(N, K)).astype(np.float32))
    bias = rng.normal(0, 0.1, size=N).astype(np.float32)
    ids = rng.integers(0, V, size=n).astype(np.int32)
    d_emb, d_ids, d_bias = backend.upload(emb_q), backend.upload(ids), backend.upload(bias)
    W = backend.weight(Q8_0, w_q, K, N)
    rows, mm_out, out = backend.alloc(n * K * 4), backend.alloc(n * N * 4), backend.alloc(n * N * 4)

    t_emb = b200.graph_tensor(Q8_0, [K, V], data=d_emb.ptr)
    t_ids = b200.graph_tensor(I32, [n], data=d_ids.ptr)
    t_rows = b200.graph_tensor(F32, [K, n], op=b200.OP_GET_ROWS, src=(t_emb, t_ids), data=rows.ptr)
    t_w = b200.graph_tensor(Q8_0, [K, N], extra=W.h)
    t_mm = b200.graph_tensor(F32, [N, n], op=b200.OP_MUL_MAT, src=(t_w, t_rows), data=mm_out.ptr)
    t_b = b200.graph_tensor(F32, [N], data=d_bias.ptr)
    t_add = b200.graph_tensor(F32, [N, n], op=b200.OP_ADD, src=(t_mm, t_b), data=out.ptr,
                              flags=b200.TENSOR_FLAG_OUTPUT)
    backend.graph_compute([t_rows, t_mm, t_add])
    got = out.get((n, N), np.float32)

    rows2, out2 = backend.alloc(n * K * 4), backend.alloc(n * N * 4)
    backend.get_rows(Q8_0, d_emb, K, V, d_ids, n, rows2)
    backend.mul_mat(W, rows2, n, out2, bias=d_bias)
    backend.synchronize()
    assert np.array_equal(_bits(got), _bits(out2.get((n, N), np.float32)))
    x = oracle.get_rows(Q8_0, emb_q, K, ids)
    ref = oracle.mul_mat(Q8_0, w_q, K, N, x) + bias[None, :]
    assert np.array_equal(_bits(got), _bits(ref))
    W.free()


def test_flash_attn_graph_views_and_mask(b200, backend):
    """Two FLASH_ATTN_EXT nodes: strided q/k/v views into one qkv tensor under a causal F16 mask (fp32
    path), and contiguous unmasked D = 64 self-attention (tensor-core path)."""
    rng = np.random.default_rng(12)
    D, N, H, B = 64, 48, 2, 2
    qkv = rng.normal(0, 1, size=(B, N, 3, H, D)).astype(np.float32)
    mask = np.zeros((N, N), np.float16)
    mask[np.triu_indices(N, 1)] = -np.inf
    d_qkv, d_mask = backend.upload(qkv), backend.upload(mask)
    nb = [4, 3 * H * D * 4, D * 4, N * 3 * H * D * 4]
    base = d_qkv.ptr
    t_q = b200.graph_tensor(F32, [D, N, H, B], nb=nb, data=base)
    t_k = b200.graph_tensor(F32, [D, N, H, B], nb=nb, data=base + H * D * 4)
    t_v = b200.graph_tensor(F32, [D, N, H, B], nb=nb, data=base + 2 * H * D * 4)
    t_m = b200.graph_tensor(F16, [N, N], data=d_mask.ptr)
    out1 = backend.alloc(B * N * H * D * 4)
    t_fa1 = b200.graph_tensor(F32, [D, H, N, B], op=b200.OP_FLASH_ATTN_EXT, src=(t_q, t_k, t_v, t_m),
                              op_params=(b200.f32_bits(0.125), 0, 0), data=out1.ptr)

    N2 = 64
    q2, k2, v2 = (rng.normal(0, 1, size=(B, H, N2, D)).astype(np.float32) for _ in range(3))
    dq, dk, dv = backend.upload(q2), backend.upload(k2), backend.upload(v2)
    tq = b200.graph_tensor(F32, [D, N2, H, B], data=dq.ptr)
    tk = b200.graph_tensor(F32, [D, N2, H, B], data=dk.ptr)
    tv = b200.graph_tensor(F32, [D, N2, H, B], data=dv.ptr)
    out2 = backend.alloc(B * N2 * H * D * 4)
    t_fa2 = b200.graph_tensor(F32, [D, H, N2, B], op=b200.OP_FLASH_ATTN_EXT, src=(tq, tk, tv),
                              op_params=(b200.f32_bits(0.125), 0, 0), data=out2.ptr)
    backend.graph_compute([t_fa1, t_fa2])
    got1, got2 = out1.get((B, N, H, D), np.float32), out2.get((B, N2, H, D), np.float32)

    ref1, ref2 = backend.alloc(B * N * H * D * 4), backend.alloc(B * N2 * H * D * 4)
    e = [x // 4 for x in nb[1:]]
    backend.flash_attn_ext_view(base, base + H * D * 4, base + 2 * H * D * 4, d_mask.ptr, N, D, N, N, H, B, e, e, e,
                                0.125, ref1)
    backend.flash_attn_ext(dq, dk, dv, D, N2, H, B, 0.125, ref2)
    backend.synchronize()
    assert np.array_equal(_bits(got1), _bits(ref1.get((B, N, H, D), np.float32)))
    assert np.array_equal(_bits(got2), _bits(ref2.get((B, N2, H, D), np.float32)))


def test_conv_chain_graph(b200, backend):
    """CONV_2D (3x3, pad 1) feeding CONV_TRANSPOSE_2D (2x2, stride 2), as in the neck and the decoder."""
    rng = np.random.default_rng(13)
    iw, ih, ic, oc, oc2 = 20, 18, 32, 40, 16
    w1 = rng.normal(0, 0.1, size=(oc, ic, 3, 3)).astype(np.float16)
    x = rng.normal(0, 1, size=(ic, ih, iw)).astype(np.float32)
    w2 = rng.normal(0, 0.1, size=(oc, oc2, 2, 2)).astype(np.float16)
    dw1, dx, dw2 = backend.upload(w1), backend.upload(x), backend.upload(w2)
    c, ct = backend.alloc(oc * ih * iw * 4), backend.alloc(oc2 * 2 * ih * 2 * iw * 4)
    t_w1 = b200.graph_tensor(F16, [3, 3, ic, oc], data=dw1.ptr)
    t_x = b200.graph_tensor(F32, [iw, ih, ic, 1], data=dx.ptr)
    t_c = b200.graph_tensor(F32, [iw, ih, oc, 1], op=b200.OP_CONV_2D, src=(t_w1, t_x), op_params=(1, 1, 1, 1, 1, 1),
                            data=c.ptr)
    t_w2 = b200.graph_tensor(F16, [2, 2, oc2, oc], data=dw2.ptr)
    t_ct = b200.graph_tensor(F32, [2 * iw, 2 * ih, oc2, 1], op=b200.OP_CONV_TRANSPOSE_2D, src=(t_w2, t_c),
                             op_params=(2,), data=ct.ptr)
    backend.graph_compute([t_c, t_ct])
    got = ct.get((oc2, 2 * ih, 2 * iw), np.float32)

    c2, ct2 = backend.alloc(oc * ih * iw * 4), backend.alloc(oc2 * 2 * ih * 2 * iw * 4)
    backend.conv_2d(dw1, dx, iw, ih, ic, oc, 3, 3, 1, 1, 1, 1, 1, 1, c2)
    backend.conv_transpose_2d(dw2, c2, iw, ih, oc, oc2, 2, 2, 2, ct2)
    backend.synchronize()
    assert np.array_equal(_bits(got), _bits(ct2.get((oc2, 2 * ih, 2 * iw), np.float32)))


def test_rejected_graph_launches_nothing_and_unfused_bias_matches_fused(b200, backend):
    """A graph with one node the backend does not run is refused before any launch; an ADD over a
    MUL_MAT that is also an output runs unfused (MUL_MAT, then the elementwise ADD) and gives the bits
    of the fused pair."""
    rng = np.random.default_rng(14)
    K, N, n = 128, 64, 16
    W = backend.weight(Q8_0, oracle_free_q8(rng, N, K), K, N)
    x, b = backend.alloc(n * K * 4), backend.alloc(N * 4)
    y1, y2, y3 = (backend.alloc(n * N * 4) for _ in range(3))
    x.set(rng.normal(0, 1, size=(n, K)).astype(np.float32))
    b.set(rng.normal(0, 1, size=N).astype(np.float32))
    t_x, t_b = b200.graph_tensor(F32, [K, n], data=x.ptr), b200.graph_tensor(F32, [N], data=b.ptr)
    t_w = b200.graph_tensor(Q8_0, [K, N], extra=W.h)
    t_mm = b200.graph_tensor(F32, [N, n], op=b200.OP_MUL_MAT, data=y1.ptr, flags=b200.TENSOR_FLAG_OUTPUT,
                             src=(t_w, t_x))
    t_add = b200.graph_tensor(F32, [N, n], op=b200.OP_ADD, src=(t_mm, t_b), data=y2.ptr)
    odd = b200.graph_tensor(F32, [N, n], op=99, src=(t_add,), data=y3.ptr)
    before = backend.launches
    with pytest.raises(b200.B200Error, match="node 2 rejected"):
        backend.graph_compute([t_mm, t_add, odd])
    assert backend.launches == before
    backend.graph_compute([t_mm, t_add])  # unfused: t_mm is an output
    unfused = y2.get((n, N), np.float32)
    t_mm.flags = 0
    t_add.data = y3.ptr
    backend.graph_compute([t_mm, t_add])  # fused into the MUL_MAT epilogue
    assert np.array_equal(_bits(unfused), _bits(y3.get((n, N), np.float32)))
    W.free()


def _gelu_tanh_f16(x):
    h = x.astype(np.float16).astype(np.float64)
    y = (0.5 * h * (1.0 + np.tanh(0.7978845608028654 * h * (1.0 + 0.044715 * h * h)))).astype(np.float16)
    y = y.astype(np.float32)
    return np.where(x <= -10, 0.0, np.where(x >= 10, x, y)).astype(np.float32)


def _norm_ref(x, eps):
    mean = (x.astype(np.float64).sum(-1, keepdims=True) / x.shape[-1]).astype(np.float32)
    v = (x - mean).astype(np.float32)
    var = ((v * v).astype(np.float64).sum(-1, keepdims=True) / x.shape[-1]).astype(np.float32)
    sc = (np.float32(1.0) / np.sqrt(var + np.float32(eps))).astype(np.float32)
    return (v * sc).astype(np.float32)


def test_elementwise_chain_graph(b200, backend):
    """LayerNorm-style chain in one graph: NORM -> MUL (weight row) -> ADD (bias row) -> GELU_ERF ->
    SCALE -> ADD (residual); every node checked against numpy applied to the GPU's own input of that node."""
    rng = np.random.default_rng(15)
    E, T1, T2 = 96, 10, 3
    x = rng.normal(0, 2, size=(T2, T1, E)).astype(np.float32)
    w, bvec = rng.normal(1, 0.2, size=E).astype(np.float32), rng.normal(0, 0.2, size=E).astype(np.float32)
    dx, dw, db = backend.upload(x), backend.upload(w), backend.upload(bvec)
    bufs = [backend.alloc(x.nbytes) for _ in range(6)]
    t_x = b200.graph_tensor(F32, [E, T1, T2], data=dx.ptr)
    t_w, t_b = b200.graph_tensor(F32, [E], data=dw.ptr), b200.graph_tensor(F32, [E], data=db.ptr)
    shape = [E, T1, T2]
    t0 = b200.graph_tensor(F32, shape, op=b200.OP_NORM, src=(t_x,), op_params=(b200.f32_bits(1e-5),),
                           data=bufs[0].ptr)
    t1 = b200.graph_tensor(F32, shape, op=b200.OP_MUL, src=(t0, t_w), data=bufs[1].ptr)
    t2 = b200.graph_tensor(F32, shape, op=b200.OP_ADD, src=(t1, t_b), data=bufs[2].ptr)
    t3 = b200.graph_tensor(F32, shape, op=b200.OP_UNARY, src=(t2,), op_params=(b200.UNARY_GELU_ERF,),
                           data=bufs[3].ptr)
    t4 = b200.graph_tensor(F32, shape, op=b200.OP_SCALE, src=(t3,), op_params=(b200.f32_bits(0.5),),
                           data=bufs[4].ptr)
    t5 = b200.graph_tensor(F32, shape, op=b200.OP_ADD, src=(t4, t_x), data=bufs[5].ptr)
    before = backend.launches
    backend.graph_compute([t0, t1, t2, t3, t4, t5])
    assert backend.launches - before == 6
    o = [bf.get(x.shape, np.float32) for bf in bufs]
    np.testing.assert_allclose(o[0], _norm_ref(x, 1e-5), rtol=1e-5, atol=1e-6)
    assert np.array_equal(_bits(o[1]), _bits(o[0] * w))
    assert np.array_equal(_bits(o[2]), _bits(o[1] + bvec))
    import math
    erf = np.vectorize(math.erf)
    ref3 = 0.5 * o[2].astype(np.float64) * (1.0 + erf(o[2].astype(np.float64) / math.sqrt(2.0)))
    np.testing.assert_allclose(o[3], ref3, rtol=1e-6, atol=2e-6)
    assert np.array_equal(_bits(o[4]), _bits(o[3] * np.float32(0.5)))
    assert np.array_equal(_bits(o[5]), _bits(o[4] + x))


def test_unary_and_cont_graph(b200, backend):
    """RELU, SIGMOID, GELU (the CPU backend's fp16 tanh table); CONT of a permuted view (the head split of
    sam3.cpp:3747-3767), a CONT that reshapes (ggml_cont_2d), and an F16 CONT."""
    rng = np.random.default_rng(16)
    x = np.concatenate([rng.normal(0, 3, size=4000), [-12.0, -10.0, 0.0, 10.0, 12.5]]).astype(np.float32)
    dx = backend.upload(x)
    outs = [backend.alloc(x.nbytes) for _ in range(3)]
    t_x = b200.graph_tensor(F32, [x.size], data=dx.ptr)
    nodes = [b200.graph_tensor(F32, [x.size], op=b200.OP_UNARY, src=(t_x,), op_params=(k,), data=o.ptr)
             for k, o in zip((b200.UNARY_RELU, b200.UNARY_SIGMOID, b200.UNARY_GELU), outs)]
    D, N, H, B = 16, 12, 3, 2
    qkv = rng.normal(0, 1, size=(B, N, 3, H, D)).astype(np.float32)
    dq = backend.upload(qkv)
    # k as a view [D, N, H, B] (token stride 3*H*D), permuted to [D, H, N, B] and made contiguous
    t_k = b200.graph_tensor(F32, [D, H, N, B], nb=[4, D * 4, 3 * H * D * 4, N * 3 * H * D * 4], data=dq.ptr + H * D * 4)
    c1, c2 = backend.alloc(B * N * H * D * 4), backend.alloc(B * N * H * D * 4)
    nodes.append(b200.graph_tensor(F32, [D, H, N, B], op=b200.OP_CONT, src=(t_k,), data=c1.ptr))
    nodes.append(b200.graph_tensor(F32, [D * H, N * B], op=b200.OP_CONT, src=(t_k,), data=c2.ptr))
    h = rng.normal(0, 1, size=(7, 33)).astype(np.float16)
    dh, ch = backend.upload(h), backend.alloc(h.nbytes)
    t_h = b200.graph_tensor(F16, [7, 33], nb=[33 * 2, 2, 7 * 33 * 2, 7 * 33 * 2], data=dh.ptr)  # transposed view
    nodes.append(b200.graph_tensor(F16, [7, 33], op=b200.OP_CONT, src=(t_h,), data=ch.ptr))
    backend.graph_compute(nodes)
    relu, sig, gelu = (o.get(x.shape, np.float32) for o in outs)
    assert np.array_equal(relu, np.where(x > 0, x, 0).astype(np.float32))
    np.testing.assert_allclose(sig, 1.0 / (1.0 + np.exp(-x.astype(np.float64))), rtol=0, atol=1e-6)
    np.testing.assert_allclose(gelu, _gelu_tanh_f16(x), rtol=2e-3, atol=1e-3)
    kk = qkv[:, :, 1]  # [B, N, H, D]: memory order of [D, H, N, B]
    assert np.array_equal(c1.get(kk.shape, np.float32), kk)
    assert np.array_equal(c2.get(kk.shape, np.float32), kk)
    assert np.array_equal(ch.get((33, 7), np.float16), h.T)


def oracle_free_q8(rng, N, K):
    """Q8_0 blocks built directly (scale 1/64 as fp16, codes in [-127, 127]): the weight bytes only need to be
    valid blocks here."""
    blocks = np.zeros((N, K // 32, 34), np.uint8)
    blocks[:, :, 0:2] = np.frombuffer(np.float16(1 / 64).tobytes(), np.uint8)
    blocks[:, :, 2:] = rng.integers(-127, 128, size=(N, K // 32, 32)).astype(np.int8).view(np.uint8)
    return blocks.reshape(N, -1)


def _softmax_ref(v):
    v = v.astype(np.float64)
    e = np.exp(v - v.max(-1, keepdims=True))
    return e / e.sum(-1, keepdims=True)


def test_soft_max_graph(b200, backend):
    """SOFT_MAX_EXT as the decoder's attention builds it: scaled scores [NKV, NQ, heads, batch] under an F16
    mask with padded rows (shared by every head), an F32 mask per head, and no mask."""
    rng = np.random.default_rng(17)
    NKV, NQ, H, B = 70, 20, 4, 2
    x = rng.normal(0, 3, size=(B, H, NQ, NKV)).astype(np.float32)
    m16 = np.zeros((24, NKV), np.float16)
    m16[np.triu_indices(24, 1, NKV)] = -np.inf
    m32 = rng.normal(0, 1, size=(H, NQ, NKV)).astype(np.float32)
    dx, dm16, dm32 = backend.upload(x), backend.upload(m16), backend.upload(m32)
    outs = [backend.alloc(x.nbytes) for _ in range(3)]
    t_x = b200.graph_tensor(F32, [NKV, NQ, H, B], data=dx.ptr)
    masks = [b200.graph_tensor(F16, [NKV, 24], data=dm16.ptr), b200.graph_tensor(F32, [NKV, NQ, H], data=dm32.ptr),
             None]
    nodes = [b200.graph_tensor(F32, [NKV, NQ, H, B], op=b200.OP_SOFT_MAX, src=(t_x, m),
                               op_params=(b200.f32_bits(0.125), 0), data=o.ptr) for m, o in zip(masks, outs)]
    backend.graph_compute(nodes)
    v = (x * np.float32(0.125)).astype(np.float32)
    refs = [_softmax_ref((v + m16[:NQ].astype(np.float32)).astype(np.float32)),
            _softmax_ref((v + m32[None]).astype(np.float32)), _softmax_ref(v)]
    for o, ref in zip(outs, refs):
        got = o.get(x.shape, np.float32)
        np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-7)
    assert np.all(outs[0].get(x.shape, np.float32)[:, :, 0, 1:] == 0)  # query 0 sees key 0 only


def test_window_partition_graph(b200, backend):
    """ggml_win_part / ggml_win_unpart (sam3.cpp:3734, 3788) with zero padding (10 x 9 map, windows of 4):
    the windows against numpy, and the round trip exact."""
    rng = np.random.default_rng(18)
    C, W, H, w = 8, 10, 9, 4
    npx, npy = 3, 3
    x = rng.normal(0, 1, size=(H, W, C)).astype(np.float32)
    dx, dwin, dback = backend.upload(x), backend.alloc(npx * npy * w * w * C * 4), backend.alloc(x.nbytes)
    t_x = b200.graph_tensor(F32, [C, W, H], data=dx.ptr)
    t_win = b200.graph_tensor(F32, [C, w, w, npx * npy], op=b200.OP_WIN_PART, src=(t_x,), op_params=(npx, npy, w),
                              data=dwin.ptr)
    t_back = b200.graph_tensor(F32, [C, W, H], op=b200.OP_WIN_UNPART, src=(t_win,), op_params=(w,), data=dback.ptr)
    backend.graph_compute([t_win, t_back])
    xp = np.zeros((npy * w, npx * w, C), np.float32)
    xp[:H, :W] = x
    ref = np.stack([xp[py * w:(py + 1) * w, px * w:(px + 1) * w] for py in range(npy) for px in range(npx)])
    assert np.array_equal(dwin.get(ref.shape, np.float32), ref)
    assert np.array_equal(dback.get(x.shape, np.float32), x)


def test_layout_ops_graph(b200, backend):
    """SUB with a broadcast row (RoPE, sam3.cpp:3704), REPEAT (sam3.cpp:3825), CONCAT along dims 0 and 1
    (sam3.cpp:3708, 8278), zero PAD on both sides (sam3.cpp:4210), nearest 2x UPSCALE (sam3.cpp:4586) and
    the F32 <-> F16 casts, each bit for bit against numpy."""
    rng = np.random.default_rng(21)
    x = rng.normal(0, 1, size=(3, 5, 8)).astype(np.float32)   # ggml [8, 5, 3]
    y = rng.normal(0, 1, size=(3, 5, 8)).astype(np.float32)
    row = rng.normal(0, 1, size=8).astype(np.float32)
    dx, dy, drow = backend.upload(x), backend.upload(y), backend.upload(row)
    t_x, t_y = b200.graph_tensor(F32, [8, 5, 3], data=dx.ptr), b200.graph_tensor(F32, [8, 5, 3], data=dy.ptr)
    t_row = b200.graph_tensor(F32, [8], data=drow.ptr)
    out = {}

    def node(name, ttype, ne, op, src, params=(), nbytes=None):
        count = int(np.prod(ne))
        buf = backend.alloc(nbytes or count * (2 if ttype == F16 else 4))
        out[name] = (buf, ne, ttype)
        return b200.graph_tensor(ttype, ne, op=op, src=src, op_params=params, data=buf.ptr)

    nodes = [
        node("sub", F32, [8, 5, 3], b200.OP_SUB, (t_x, t_row)),
        node("repeat", F32, [16, 5, 6], b200.OP_REPEAT, (t_x,)),
        node("cat0", F32, [16, 5, 3], b200.OP_CONCAT, (t_x, t_y), (0,)),
        node("cat1", F32, [8, 10, 3], b200.OP_CONCAT, (t_x, t_y), (1,)),
        node("pad", F32, [11, 9, 3], b200.OP_PAD, (t_x,), (1, 2, 0, 4, 0, 0, 0, 0)),
        node("up", F32, [16, 10, 3], b200.OP_UPSCALE, (t_x,), (0,)),
        node("to16", F16, [8, 5, 3], b200.OP_CONT, (t_x,)),
    ]
    nodes.append(node("to32", F32, [8, 5, 3], b200.OP_CONT, (nodes[-1],)))
    backend.graph_compute(nodes)

    def get(name):
        buf, ne, ttype = out[name]
        return buf.get(tuple(reversed(ne)), np.float16 if ttype == F16 else np.float32)

    assert np.array_equal(_bits(get("sub")), _bits(x - row))
    assert np.array_equal(get("repeat"), np.tile(x, (2, 1, 2)))
    assert np.array_equal(get("cat0"), np.concatenate([x, y], axis=2))
    assert np.array_equal(get("cat1"), np.concatenate([x, y], axis=1))
    assert np.array_equal(get("pad"), np.pad(x, ((0, 0), (0, 4), (1, 2))))
    assert np.array_equal(get("up"), x.repeat(2, axis=1).repeat(2, axis=2))
    assert np.array_equal(get("to16"), x.astype(np.float16))
    assert np.array_equal(get("to32"), x.astype(np.float16).astype(np.float32))


def _im2col_ref(x, KW, KH, s0, s1, p0, p1, d0, d1):
    """x [N, C, H, W] -> [N, OH, OW, C*KH*KW] (ggml's IM2COL element order), zero outside the image."""
    N, C, H, W = x.shape
    OW = (W + 2 * p0 - d0 * (KW - 1) - 1) // s0 + 1
    OH = (H + 2 * p1 - d1 * (KH - 1) - 1) // s1 + 1
    xp = np.zeros((N, C, H + 2 * p1 + s1 * OH + d1 * KH, W + 2 * p0 + s0 * OW + d0 * KW), x.dtype)
    xp[:, :, p1:p1 + H, p0:p0 + W] = x
    col = np.zeros((N, OH, OW, C, KH, KW), x.dtype)
    for ky in range(KH):
        for kx in range(KW):
            col[:, :, :, :, ky, kx] = xp[:, :, ky * d1:ky * d1 + s1 * OH:s1, kx * d0:kx * d0 + s0 * OW:s0].transpose(0, 2, 3, 1)
    return col.reshape(N, OH, OW, C * KH * KW)


def test_im2col_and_mul_mat_of_graph_tensors(b200, backend):
    """The patch embedding as sam3.cpp:6726-6742 builds it: IM2COL of the image into F16 columns, then a
    MUL_MAT of that graph tensor (src0) with the F16 kernel reshaped to [KW*KH*IC, OC] (src1) -- the
    fp16 tensor-core path, K = 588 zero-padded to 592.  The columns are bit-exact; the product is
    checked against float64 of the same fp16 operands at 1e-5 of the largest output."""
    rng = np.random.default_rng(22)
    IC, H, W, KH, KW, OC = 3, 140, 126, 14, 14, 160
    img = rng.normal(0, 1, size=(1, IC, H, W)).astype(np.float32)
    kern = (rng.normal(0, 0.05, size=(OC, IC, KH, KW))).astype(np.float16)
    d_img, d_k = backend.upload(img), backend.upload(kern)
    OH, OW, K = H // KH, W // KW, IC * KH * KW
    cols = backend.alloc(OH * OW * K * 2)
    res = backend.alloc(OC * OH * OW * 4)
    t_k = b200.graph_tensor(F16, [KW, KH, IC, OC], data=d_k.ptr)
    t_img = b200.graph_tensor(F32, [W, H, IC, 1], data=d_img.ptr)
    t_col = b200.graph_tensor(F16, [K, OW, OH, 1], op=b200.OP_IM2COL, src=(t_k, t_img),
                              op_params=(KW, KH, 0, 0, 1, 1, 1), data=cols.ptr)
    t_col2 = b200.graph_tensor(F16, [K, OW * OH], op=b200.OP_VIEW, src=(t_col,), data=cols.ptr)
    t_k2 = b200.graph_tensor(F16, [K, OC], op=b200.OP_VIEW, src=(t_k,), data=d_k.ptr)
    t_mm = b200.graph_tensor(F32, [OW * OH, OC], op=b200.OP_MUL_MAT, src=(t_col2, t_k2), data=res.ptr)
    before = backend.launches
    backend.graph_compute([t_col, t_col2, t_k2, t_mm])
    assert backend.launches - before == 4  # IM2COL, two fp16 operand packs, the tensor-core GEMM
    col_ref = _im2col_ref(img, KW, KH, KW, KH, 0, 0, 1, 1).astype(np.float16)
    assert np.array_equal(cols.get((OH * OW, K), np.float16), col_ref.reshape(OH * OW, K))
    ref = kern.reshape(OC, K).astype(np.float64) @ col_ref.reshape(OH * OW, K).astype(np.float64).T  # [OC, OH*OW]
    got = res.get((OC, OH * OW), np.float32)
    assert np.abs(got - ref).max() <= 1e-5 * np.abs(ref).max()


@pytest.mark.parametrize("otype", [F32, F16])
def test_im2col_padding_stride_dilation(b200, backend, otype):
    """A 3 x 3 IM2COL with stride 2, padding 1 and dilation 2 over an odd-sized map of 5 channels and 2
    images: every column element, zero where the window leaves the image."""
    rng = np.random.default_rng(23)
    N, C, H, W, s, p, d = 2, 5, 13, 11, 2, 1, 2
    x = rng.normal(0, 1, size=(N, C, H, W)).astype(np.float32)
    dx = backend.upload(x)
    ref = _im2col_ref(x, 3, 3, s, s, p, p, d, d)
    buf = backend.alloc(ref.size * (2 if otype == F16 else 4))
    t_k = b200.graph_tensor(F16, [3, 3, C, 7])
    t_x = b200.graph_tensor(F32, [W, H, C, N], data=dx.ptr)
    t = b200.graph_tensor(otype, [C * 9, ref.shape[2], ref.shape[1], N], op=b200.OP_IM2COL, src=(t_k, t_x),
                          op_params=(s, s, p, p, d, d, 1), data=buf.ptr)
    backend.graph_compute([t])
    dt = np.float16 if otype == F16 else np.float32
    assert np.array_equal(buf.get(ref.shape, dt), ref.astype(dt))


def test_batched_mul_mat_of_graph_tensors(b200, backend):
    """Attention scores as the decoder builds them (ggml_mul_mat(K, Q), sam3.cpp:8584, 10218): F32 src0
    [64, 70, 4 heads, 1] broadcast over src1 [64, 20, 8, 2]; then F16 src0 with a batch (src1 rounded to
    fp16 first, ggml-cpu's rule) and a 2-D F32 product of odd sizes.  fp32 FMA accumulation against
    float64: within 1e-5 of the largest output."""
    rng = np.random.default_rng(24)
    cases = [((1, 4, 70, 64), np.float32, (2, 8, 20, 64)), ((1, 3, 33, 40), np.float16, (1, 6, 65, 40)),
             ((1, 1, 129, 77), np.float32, (1, 1, 131, 77))]
    for sa, dta, sb in cases:
        a = rng.normal(0, 1, size=sa).astype(dta)
        b = rng.normal(0, 1, size=sb).astype(np.float32)
        da, db = backend.upload(a), backend.upload(b)
        ne_a, ne_b = list(reversed(sa)), list(reversed(sb))
        ne_o = [ne_a[1], ne_b[1], ne_b[2], ne_b[3]]
        o = backend.alloc(int(np.prod(ne_o)) * 4)
        t_a = b200.graph_tensor(F16 if dta == np.float16 else F32, ne_a, data=da.ptr)
        t_b = b200.graph_tensor(F32, ne_b, data=db.ptr)
        t = b200.graph_tensor(F32, ne_o, op=b200.OP_MUL_MAT, src=(t_a, t_b), data=o.ptr)
        backend.graph_compute([t])
        bb = b.astype(np.float16) if dta == np.float16 else b
        r2, r3 = sb[1] // sa[1], sb[0] // sa[0]
        aa = np.repeat(np.repeat(a.astype(np.float64), r2, axis=1), r3, axis=0)
        ref = np.einsum("xynk,xymk->xymn", aa, bb.astype(np.float64))
        got = o.get(ref.shape, np.float32)
        assert np.abs(got - ref).max() <= 1e-5 * np.abs(ref).max(), sa


def test_pool_dw_conv_group_norm_graph(b200, backend):
    """Max pool 2x2/2 (sam3.cpp:3918) and an average pool with padding (sam3.cpp:4748 pools whole maps),
    the depthwise 3x3 convolution with stride 2, padding 1 (sam3.cpp:4777), and GROUP_NORM(8) of 32
    channels (sam3.cpp:8923), against numpy."""
    rng = np.random.default_rng(25)
    N, C, H, W = 2, 32, 15, 18
    x = rng.normal(0, 2, size=(N, C, H, W)).astype(np.float32)
    kdw = rng.normal(0, 0.3, size=(C, 1, 3, 3)).astype(np.float32)
    dx, dk = backend.upload(x), backend.upload(kdw)
    t_x = b200.graph_tensor(F32, [W, H, C, N], data=dx.ptr)
    t_k = b200.graph_tensor(F32, [3, 3, 1, C], data=dk.ptr)
    bmax, bavg = backend.alloc(N * C * 7 * 9 * 4), backend.alloc(N * C * 8 * 6 * 4)
    bdw, bgn = backend.alloc(N * C * 8 * 9 * 4), backend.alloc(x.nbytes)
    nodes = [
        b200.graph_tensor(F32, [9, 7, C, N], op=b200.OP_POOL_2D, src=(t_x,), op_params=(0, 2, 2, 2, 2, 0, 0),
                          data=bmax.ptr),
        b200.graph_tensor(F32, [6, 8, C, N], op=b200.OP_POOL_2D, src=(t_x,), op_params=(1, 3, 3, 3, 2, 1, 1),
                          data=bavg.ptr),
        b200.graph_tensor(F32, [9, 8, C, N], op=b200.OP_CONV_2D_DW, src=(t_k, t_x), op_params=(2, 2, 1, 1, 1, 1),
                          data=bdw.ptr),
        b200.graph_tensor(F32, [W, H, C, N], op=b200.OP_GROUP_NORM, src=(t_x,), op_params=(8, b200.f32_bits(1e-5)),
                          data=bgn.ptr),
    ]
    backend.graph_compute(nodes)
    # max pool 2x2 stride 2: floor((18 - 2) / 2) + 1 = 9, (15 - 2) // 2 + 1 = 7
    mx = x[:, :, :14, :18].reshape(N, C, 7, 2, 9, 2).max(axis=(3, 5))
    assert np.array_equal(bmax.get(mx.shape, np.float32), mx)
    # average 3x3, stride (3, 2), padding 1, divided by 9 whatever the overlap
    xp = np.zeros((N, C, H + 2, W + 2), np.float64)
    xp[:, :, 1:-1, 1:-1] = x
    avg = np.zeros((N, C, 8, 6))
    for oy in range(8):
        for ox in range(6):
            avg[:, :, oy, ox] = xp[:, :, 2 * oy:2 * oy + 3, 3 * ox:3 * ox + 3].sum(axis=(2, 3)) / 9
    np.testing.assert_allclose(bavg.get(avg.shape, np.float32), avg, rtol=1e-5, atol=1e-6)
    dw = np.zeros((N, C, 8, 9))
    for ky in range(3):
        for kx in range(3):
            dw += xp[:, :, ky:ky + 16:2, kx:kx + 18:2] * kdw[None, :, 0, ky, kx, None, None]
    np.testing.assert_allclose(bdw.get(dw.shape, np.float32), dw, rtol=1e-5, atol=1e-5)
    g = x.reshape(N, 8, -1).astype(np.float64)
    gn = ((g - g.mean(-1, keepdims=True)) / np.sqrt(g.var(-1, keepdims=True) + 1e-5)).reshape(x.shape)
    np.testing.assert_allclose(bgn.get(x.shape, np.float32), gn, rtol=1e-5, atol=1e-5)
