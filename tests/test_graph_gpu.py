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


def test_rejected_graph_launches_nothing(b200, backend):
    """An ADD over a MUL_MAT whose result is also an output cannot be fused: the graph is refused before
    any launch and the backend stays usable."""
    rng = np.random.default_rng(14)
    K, N, n = 128, 64, 16
    W = backend.weight(Q8_0, oracle_free_q8(rng, N, K), K, N)
    x, b, y1, y2 = backend.alloc(n * K * 4), backend.alloc(N * 4), backend.alloc(n * N * 4), backend.alloc(n * N * 4)
    t_mm = b200.graph_tensor(F32, [N, n], op=b200.OP_MUL_MAT, data=y1.ptr, flags=b200.TENSOR_FLAG_OUTPUT, src=(
        b200.graph_tensor(Q8_0, [K, N], extra=W.h), b200.graph_tensor(F32, [K, n], data=x.ptr)))
    t_add = b200.graph_tensor(F32, [N, n], op=b200.OP_ADD, src=(t_mm, b200.graph_tensor(F32, [N], data=b.ptr)),
                              data=y2.ptr)
    before = backend.launches
    with pytest.raises(b200.B200Error, match="node 1 rejected"):
        backend.graph_compute([t_mm, t_add])
    assert backend.launches == before
    t_mm.flags = 0  # the same graph without the OUTPUT flag runs
    x.set(rng.normal(0, 1, size=(n, K)).astype(np.float32))
    b.set(np.zeros(N, np.float32))
    backend.graph_compute([t_mm, t_add])
    assert backend.launches > before
    W.free()


def oracle_free_q8(rng, N, K):
    """Q8_0 blocks built directly (scale 1/64 as fp16, codes in [-127, 127]): the weight bytes only need to be
    valid blocks here."""
    blocks = np.zeros((N, K // 32, 34), np.uint8)
    blocks[:, :, 0:2] = np.frombuffer(np.float16(1 / 64).tobytes(), np.uint8)
    blocks[:, :, 2:] = rng.integers(-127, 128, size=(N, K // 32, 32)).astype(np.int8).view(np.uint8)
    return blocks.reshape(N, -1)
