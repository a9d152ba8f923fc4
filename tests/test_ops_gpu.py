"""Op-level entry points of the drop-in boundary (the ggml ops sam3.cpp's
graphs dispatch besides MUL_MAT), through the C ABI, against the oracle."""
import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("batch,heads,N", [(1, 2, 64), (2, 3, 200), (9, 2, 576), (1, 1, 8)])
def test_flash_attn_ext_matches_oracle(oracle, backend, batch, heads, N):
    """GGML_OP_FLASH_ATTN_EXT (sam3.cpp:3778): bf16 tensor-core attention within 1e-2 of the f32 oracle."""
    rng = np.random.default_rng(batch * 1000 + heads * 100 + N)
    q, k, v = (rng.normal(0, 1, size=(batch * heads, N, 64)).astype(np.float32) for _ in range(3))
    scale = 0.125
    dq, dk, dv = backend.upload(q), backend.upload(k), backend.upload(v)
    out = backend.alloc(batch * N * heads * 64 * 4)
    backend.flash_attn_ext(dq, dk, dv, 64, N, heads, batch, scale, out)
    backend.synchronize()
    got = out.get((batch * N, heads * 64), np.float32)
    ref = oracle.attention(q, k, v, batch, N, heads, scale)
    err = np.abs(got - ref).max() / np.abs(ref).max()
    assert err <= 1e-2, err


def test_flash_attn_ext_rejects_unsupported(b200, backend):
    buf = backend.alloc(4096)
    with pytest.raises(b200.B200Error):
        backend.flash_attn_ext(buf, buf, buf, 80, 8, 1, 1, 0.1, buf)  # head dim 80


# GGML_OP_CONV_TRANSPOSE_2D: the case table of the reference's own CPU-vs-Metal test
# (tests/test_metal_conv_transpose_2d.cpp:48-56): name, in_w, in_h, in_c, out_c, kw, kh, stride,
# seed, max-abs tolerance; inputs from the same generator (:93-111).
CONVT_CASES = [
    ("cpu_ref_stride1", 3, 2, 2, 3, 2, 2, 1, 0x1234, 1e-5),
    ("cpu_ref_stride2", 3, 2, 2, 3, 2, 2, 2, 0x2345, 1e-5),
    ("cpu_ref_stride3", 3, 2, 2, 3, 2, 2, 3, 0x3456, 1e-5),
    ("small_rect", 5, 4, 3, 4, 3, 2, 1, 0x4567, 1e-5),
    ("medium_stride2", 8, 7, 5, 6, 3, 3, 2, 0x5678, 1e-4),
    ("sam_first", 72, 72, 1024, 512, 2, 2, 2, 0x6789, 2e-3),
    ("sam_second", 144, 144, 512, 256, 2, 2, 2, 0x789A, 2e-3),
]


def _gen_values(n: int, seed: int, scale: float) -> np.ndarray:
    """The reference test's value generator: an LCG step on (idx ^ seed), folded, mapped to
    (x % 511 - 255) * scale."""
    x = (np.arange(n, dtype=np.uint64) & 0xFFFFFFFF).astype(np.uint32) ^ np.uint32(seed)
    x = x * np.uint32(1664525) + np.uint32(1013904223)
    x ^= x >> np.uint32(16)
    return ((x % np.uint32(511)).astype(np.int64) - 255).astype(np.float32) * np.float32(scale)


@pytest.mark.parametrize("case", CONVT_CASES, ids=[c[0] for c in CONVT_CASES])
def test_conv_transpose_2d_reference_cases(oracle, backend, case):
    name, iw, ih, ic, oc, kw, kh, stride, seed, tol = case
    w = _gen_values(kw * kh * oc * ic, seed ^ 0x2468ACE, 1.0 / 128.0).astype(np.float16).reshape(ic, oc, kh, kw)
    x = _gen_values(iw * ih * ic, seed ^ 0x13579BD, 1.0 / 256.0).reshape(ic, ih, iw)
    ow, oh = (iw - 1) * stride + kw, (ih - 1) * stride + kh
    dw, dx = backend.upload(w), backend.upload(x)
    out = backend.alloc(oc * oh * ow * 4)
    backend.conv_transpose_2d(dw, dx, iw, ih, ic, oc, kw, kh, stride, out)
    backend.synchronize()
    got = out.get((oc, oh, ow), np.float32)
    ref = oracle.conv_transpose_2d(w, x, stride)
    assert np.abs(got - ref).max() <= tol, (name, float(np.abs(got - ref).max()))


CONV2D_CASES = [  # iw, ih, ic, oc, kw, kh, s0, s1, p0, p1, d0, d1
    (56, 42, 3, 32, 14, 14, 14, 14, 0, 0, 1, 1),   # ggml_conv_2d_sk_p0: patch embedding (sam3.cpp:3819)
    (24, 20, 64, 48, 1, 1, 1, 1, 0, 0, 1, 1),      # 1x1 (neck, sam3.cpp:3889)
    (20, 18, 32, 40, 3, 3, 1, 1, 1, 1, 1, 1),      # ggml_conv_2d_s1_ph (sam3.cpp:3891)
    (64, 48, 3, 96, 7, 7, 4, 4, 3, 3, 1, 1),       # Hiera patch embedding (sam3.cpp:4474)
    (33, 31, 16, 24, 3, 3, 2, 2, 1, 1, 1, 1),      # memory-encoder downsampling (sam3.cpp:11541)
    (15, 13, 8, 8, 3, 3, 1, 2, 2, 1, 2, 1),        # dilation, unequal strides and pads
]


@pytest.mark.parametrize("case", CONV2D_CASES)
def test_conv_2d_matches_oracle(oracle, backend, case):
    iw, ih, ic, oc, kw, kh, s0, s1, p0, p1, d0, d1 = case
    rng = np.random.default_rng(iw * 7 + ic)
    w = rng.normal(0, 0.1, size=(oc, ic, kh, kw)).astype(np.float16)
    x = rng.normal(0, 1, size=(ic, ih, iw)).astype(np.float32)
    ref = oracle.conv_2d(w, x, s0, s1, p0, p1, d0, d1)
    out = backend.alloc(ref.size * 4)
    backend.conv_2d(backend.upload(w), backend.upload(x), iw, ih, ic, oc, kw, kh, s0, s1, p0, p1, d0, d1, out)
    backend.synchronize()
    got = out.get(ref.shape, np.float32)
    # same fp16 rounding of the input as the oracle; only the fp32 summation order differs
    assert np.abs(got - ref).max() / np.abs(ref).max() <= 1e-4


@pytest.mark.parametrize("qtype", [0, 1, 2, 3, 8])
def test_get_rows_bit_exact(oracle, backend, qtype):
    rng = np.random.default_rng(qtype)
    nrows, ncols = 300, 256
    w = rng.normal(0, 0.5, size=(nrows, ncols)).astype(np.float32)
    if qtype == 0:
        rows = w.view(np.uint8).reshape(nrows, -1)
    elif qtype == 1:
        rows = w.astype(np.float16).view(np.uint8).reshape(nrows, -1)
    else:
        rows = oracle.quantize_weights(qtype, w)
    idx = rng.integers(0, nrows, size=77).astype(np.int32)
    idx[:3] = [0, nrows - 1, 0]
    out = backend.alloc(idx.size * ncols * 4)
    backend.get_rows(qtype, backend.upload(np.ascontiguousarray(rows)), ncols, nrows, backend.upload(idx), idx.size, out)
    backend.synchronize()
    got = out.get((idx.size, ncols), np.float32)
    ref = oracle.get_rows(qtype, rows, ncols, idx)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_get_rows_index_out_of_range_reports(b200, backend):
    rows = np.arange(4 * 32, dtype=np.float32).reshape(4, 32)
    idx = np.array([1, 7, 2], np.int32)
    out = backend.alloc(3 * 32 * 4)
    backend.get_rows(0, backend.upload(rows), 32, 4, backend.upload(idx), 3, out)
    with pytest.raises(b200.B200Error):
        backend.synchronize()
    backend.synchronize()  # the error word was cleared
    got = out.get((3, 32), np.float32)
    assert np.array_equal(got[0], rows[1]) and not got[1].any() and np.array_equal(got[2], rows[2])


def test_conv_rejects_bad_shapes(b200, backend):
    buf = backend.alloc(4096)
    with pytest.raises(b200.B200Error):
        backend.conv_2d(buf, buf, 4, 4, 1, 1, 7, 7, 1, 1, 0, 0, 1, 1, buf)  # kernel larger than the input
    with pytest.raises(b200.B200Error):
        backend.conv_transpose_2d(buf, buf, 0, 4, 1, 1, 2, 2, 2, buf)
    with pytest.raises(b200.B200Error):
        backend.get_rows(8, buf, 48, 4, buf, 1, buf)  # Q8_0 rows need a multiple of 32 columns


def _contig_nb(D, N, H):
    return (D, N * D, H * N * D)


@pytest.mark.parametrize("D,NQ,NKV,H,B", [(16, 40, 56, 8, 2), (32, 64, 64, 4, 1), (96, 49, 196, 2, 3),
                                          (256, 33, 70, 1, 2), (64, 24, 100, 2, 1)])
def test_flash_attn_ext_general_shapes(oracle, backend, D, NQ, NKV, H, B):
    """Head dims of the SAM decoder (16), Hiera (96) and memory attention (256); cross-attention shapes."""
    rng = np.random.default_rng(D + NQ + NKV)
    q = rng.normal(0, 1, size=(B, H, NQ, D)).astype(np.float32)
    k = rng.normal(0, 1, size=(B, H, NKV, D)).astype(np.float32)
    v = rng.normal(0, 1, size=(B, H, NKV, D)).astype(np.float32)
    scale = 1.0 / np.sqrt(D)
    dq, dk, dv = backend.upload(q), backend.upload(k), backend.upload(v)
    out = backend.alloc(B * NQ * H * D * 4)
    backend.flash_attn_ext_view(dq.ptr, dk.ptr, dv.ptr, None, 0, D, NQ, NKV, H, B, _contig_nb(D, NQ, H),
                                _contig_nb(D, NKV, H), _contig_nb(D, NKV, H), scale, out)
    backend.synchronize()
    ref = oracle.attention_general(q, k, v, scale)
    assert rel_err(out.get(ref.shape, np.float32), ref) <= 1e-4  # fp32 path


def test_flash_attn_ext_causal_mask_and_dead_row(oracle, backend):
    """The text encoder's causal F16 mask (sam3.cpp:3934-3951), padded rows, and a row whose keys are all
    masked (zeros)."""
    D, N, H, B, ld = 64, 32, 4, 2, 40
    rng = np.random.default_rng(9)
    q, k, v = (rng.normal(0, 1, size=(B, H, N, D)).astype(np.float32) for _ in range(3))
    mask = np.zeros((N, ld), np.float16)
    mask[np.triu_indices(N, 1)] = -np.inf
    mask[5, :] = -np.inf  # every key of query row 5 removed
    out = backend.alloc(B * N * H * D * 4)
    dq, dk, dv, dm = backend.upload(q), backend.upload(k), backend.upload(v), backend.upload(mask)  # kept alive
    backend.flash_attn_ext_view(dq.ptr, dk.ptr, dv.ptr, dm.ptr, ld, D, N, N, H, B, _contig_nb(D, N, H),
                                _contig_nb(D, N, H), _contig_nb(D, N, H), 0.125, out)
    backend.synchronize()
    got = out.get((B, N, H, D), np.float32)
    ref = oracle.attention_general(q, k, v, 0.125, mask[:, :N].astype(np.float32))
    assert np.all(got[:, 5] == 0)
    assert rel_err(got, ref) <= 1e-4


def test_flash_attn_ext_permuted_views(oracle, backend):
    """q, k, v as strided views into one qkv tensor ([3*H*D, N, B] memory, as the ViT's qkv projection
    output is split at sam3.cpp:3747-3767), passed with their ggml strides."""
    D, N, H, B = 64, 50, 3, 2
    rng = np.random.default_rng(4)
    qkv = rng.normal(0, 1, size=(B, N, 3, H, D)).astype(np.float32)
    d = backend.upload(qkv)
    nb = (3 * H * D, D, N * 3 * H * D)  # token, head, batch
    base = d.ptr
    out = backend.alloc(B * N * H * D * 4)
    backend.flash_attn_ext_view(base, base + H * D * 4, base + 2 * H * D * 4, None, 0, D, N, N, H, B, nb, nb, nb,
                                0.125, out)
    backend.synchronize()
    q, k, v = (qkv[:, :, i].transpose(0, 2, 1, 3) for i in range(3))
    ref = oracle.attention_general(q, k, v, 0.125)
    assert rel_err(out.get(ref.shape, np.float32), ref) <= 1e-4


def test_flash_attn_ext_view_rejects(b200, backend):
    buf = backend.alloc(4096)
    nb = (24, 24, 24)
    with pytest.raises(b200.B200Error):
        backend.flash_attn_ext_view(buf.ptr, buf.ptr, buf.ptr, None, 0, 24, 1, 1, 1, 1, nb, nb, nb, 0.1, buf)
    with pytest.raises(b200.B200Error):  # mask rows shorter than the key count
        backend.flash_attn_ext_view(buf.ptr, buf.ptr, buf.ptr, buf.ptr, 4, 16, 2, 8, 1, 1, nb, nb, nb, 0.1, buf)
