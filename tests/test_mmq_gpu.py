"""GPU parity of the MUL_MAT path (ggml_mul_mat with Q8_0 / Q4_0 / Q4_1 / F16 /
F32 weights, sam3.cpp:3742,3783,3796,3799) against the CPU oracle, through the
C ABI.

Rows up to 64 with f32 output take the skinny kernel (weights read once per
CTA, dp4a dots), larger SIMT cases the one-output-per-thread kernel; both
fold the blocks in the same order.

Bar (stated per test):
  * int32 block dots: bit-exact (the MMA path's own dots, dumped);
  * f32 output: bit-exact with the oracle's block-ordered fma sequence,
    which also satisfies the north-star bound max|d|/max|ref| <= 1e-2.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

IMPLS = ["TC", "SIMT"]


def _case(oracle, qt, M, K, N, seed, x_scale=1.0):
    rng = np.random.default_rng(seed)
    w = rng.normal(0, 0.02, size=(N, K)).astype(np.float32)
    x = (rng.normal(0, 1, size=(M, K)) * x_scale).astype(np.float32)
    bias = rng.normal(0, 0.02, size=(N,)).astype(np.float32)
    return oracle.quantize_weights(qt, w), x, bias


def _impl(b200, name):
    return {"TC": b200.MMQ_TC, "SIMT": b200.MMQ_SIMT}[name]


@pytest.mark.parametrize("impl", IMPLS)
@pytest.mark.parametrize("qt", [8, 2])
@pytest.mark.parametrize("M,K,N", [(200, 256, 384), (128, 64, 256), (37, 96, 136), (1, 32, 8)])
def test_block_dots_bit_exact(oracle, b200, backend, impl, qt, M, K, N):
    wq, x, _ = _case(oracle, qt, M, K, N, seed=M * 7 + K + N)
    prev = backend.set_mmq_impl(_impl(b200, impl))
    try:
        w = backend.weight(qt, wq, K, N)
        xd = backend.upload(x)
        got = backend.mul_mat_block_dots(w, xd, M)
        w.free()
    finally:
        backend.set_mmq_impl(prev)
    ref = oracle.block_dots(qt, wq, K, N, x)
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("impl", IMPLS)
@pytest.mark.parametrize("qt", [8, 2])
@pytest.mark.parametrize("M,K,N", [(200, 256, 384), (300, 1024, 512), (5, 64, 40), (129, 4736 // 4, 264),
                                   (32, 1024, 1000), (64, 96, 72), (65, 64, 40)])
def test_mul_mat_f32_matches_oracle(oracle, b200, backend, impl, qt, M, K, N):
    wq, x, bias = _case(oracle, qt, M, K, N, seed=M + 3 * K + N)
    prev = backend.set_mmq_impl(_impl(b200, impl))
    try:
        w = backend.weight(qt, wq, K, N)
        xd, bd = backend.upload(x), backend.upload(bias)
        yd = backend.alloc(M * N * 4)
        backend.mul_mat(w, xd, M, yd, bias=bd)
        backend.synchronize()
        got = yd.get((M, N), np.float32)
        w.free()
    finally:
        backend.set_mmq_impl(prev)
    ref = oracle.mul_mat(qt, wq, K, N, x) + bias[None, :]
    err = np.max(np.abs(got - ref)) / np.max(np.abs(ref))
    assert err <= 1e-2
    assert np.array_equal(got, ref), f"not bit-exact: max rel {err:.3e}"


def test_mul_mat_row_strides_and_zero_rows(oracle, b200, backend):
    """ldx > K, ldd > N, and all-zero activation rows (amax = 0 -> d = 0)."""
    M, K, N, ldx, ldd = 70, 128, 200, 160, 204
    wq, x, bias = _case(oracle, 8, M, K, N, seed=11)
    x[3] = 0.0
    x[40, :32] = 0.0
    xs = np.zeros((M, ldx), np.float32)
    xs[:, :K] = x
    w = backend.weight(8, wq, K, N)
    xd, bd = backend.upload(xs), backend.upload(bias)
    yd = backend.alloc(M * ldd * 4)
    backend.mul_mat(w, xd, M, yd, bias=bd, ldx=ldx, ldy=ldd)
    backend.synchronize()
    got = yd.get((M, ldd), np.float32)[:, :N]
    ref = oracle.mul_mat(8, wq, K, N, x) + bias[None, :]
    assert np.array_equal(got, ref)
    w.free()


@pytest.mark.parametrize("qt", [8, 2])
@pytest.mark.parametrize("K,N", [(1024, 3072), (1024, 1024), (1024, 4736), (4736, 1024)])
def test_vit_shapes_sampled_rows(oracle, b200, backend, qt, K, N):
    """Full ViT-32 GEMM shapes (M = 5184 tokens); the oracle checks a
    sample of rows spread over every M tile including the ragged last one.
    Q4_0 weights stay 4-bit in device memory; the tensor-core kernel unpacks
    each stage's nibbles in shared memory."""
    M = 5184
    wq, x, bias = _case(oracle, qt, M, K, N, seed=K + N)
    w = backend.weight(qt, wq, K, N)
    xd, bd = backend.upload(x), backend.upload(bias)
    yd = backend.alloc(M * N * 4)
    backend.set_mmq_impl(b200.MMQ_AUTO)
    backend.mul_mat(w, xd, M, yd, bias=bd)
    backend.synchronize()
    got = yd.get((M, N), np.float32)
    rows = np.unique(np.concatenate([np.arange(0, M, 97), [M - 1, M - 64, 5120, 127, 128]]))
    ref = oracle.mul_mat(qt, wq, K, N, x[rows]) + bias[None, :]
    assert np.array_equal(got[rows], ref)
    w.free()


def test_bad_weight_type_is_rejected(b200, backend):
    blocks = np.zeros(64, np.uint8)
    with pytest.raises(b200.B200Error):
        backend.weight(6, blocks, 32, 1)   # ggml Q5_0: not a sam3.cpp weight type
    with pytest.raises(b200.B200Error):
        backend.weight(8, blocks, 48, 1)   # K not a multiple of 32
    with pytest.raises(b200.B200Error):
        backend.weight(1, blocks, 12, 1)   # F16 rows must be a multiple of 8 (16-byte TMA pitch)


@pytest.mark.parametrize("impl", IMPLS)
@pytest.mark.parametrize("M,K,N", [(200, 256, 384), (37, 96, 136), (1, 32, 8), (300, 1024, 520)])
def test_q4_1_bit_exact(oracle, b200, backend, impl, M, K, N):
    """Q4_1 weights x Q8_1 activations (ggml vec_dot_q4_1_q8_1): block dots of the nibble codes and the
    f32 output, whose per-block sum is fma(I, d_w d_x, acc) then fma(m_w, s_x, acc), bit-exact.  On the
    tensor cores the nibbles are unpacked in shared memory as unsigned codes and m_w s_x comes from a
    third MMA next to the block dot and the scale product."""
    wq, x, bias = _case(oracle, 3, M, K, N, seed=M + 11 * K + N)
    w = backend.weight(3, wq, K, N)
    dx, db = backend.upload(x), backend.upload(bias)
    prev = backend.set_mmq_impl(_impl(b200, impl))
    try:
        dots = backend.mul_mat_block_dots(w, dx, M)
        y = backend.alloc(M * N * 4)
        backend.mul_mat(w, dx, M, y, bias=db)
        backend.synchronize()
    finally:
        backend.set_mmq_impl(prev)
    assert np.array_equal(dots, oracle.block_dots(3, wq, K, N, x))
    assert np.array_equal(y.get((M, N), np.float32), oracle.mul_mat(3, wq, K, N, x) + bias[None, :])
    w.free()


@pytest.mark.parametrize("qt", [1, 0])
@pytest.mark.parametrize("M,K,N", [(200, 256, 384), (37, 96, 136), (5184, 1024, 1024)])
def test_dense_weights_within_bound(oracle, b200, backend, qt, M, K, N):
    """F16 weights (x rounded to fp16 as ggml's vec_dot_type) and F32 weights (stored as fp16 here) on the
    fp16 tensor-core GEMM: max|d| / max|ref| <= 1e-2 against the oracle's fp32 dots."""
    rng = np.random.default_rng(M + K + N + qt)
    w = rng.normal(0, 0.02, size=(N, K)).astype(np.float32)
    x = rng.normal(0, 1, size=(M, K)).astype(np.float32)
    bias = rng.normal(0, 0.02, size=(N,)).astype(np.float32)
    blocks = w.astype(np.float16) if qt == 1 else w
    wt = backend.weight(qt, blocks, K, N)
    dx, db, y = backend.upload(x), backend.upload(bias), backend.alloc(M * N * 4)
    backend.mul_mat(wt, dx, M, y, bias=db)
    backend.synchronize()
    got = y.get((M, N), np.float32)
    rows = np.arange(0, M, max(1, M // 200))
    ref = oracle.mul_mat(qt, np.ascontiguousarray(blocks).view(np.uint8), K, N, x[rows]) + bias[None, :]
    err = np.abs(got[rows] - ref).max() / np.abs(ref).max()
    assert err <= 1e-2, err
    wt.free()


@pytest.mark.parametrize("qt", [8, 2])
@pytest.mark.parametrize("M,K,N", [(5184, 1024, 3072), (5184, 1024, 1024), (5184, 1024, 4736), (5184, 4736, 1024),
                                   (300, 96, 288), (77, 1024, 520), (1, 64, 32)])
def test_mul_mat_dq16_against_oracle(oracle, b200, backend, qt, M, K, N):
    """sam3b200_mul_mat_dq16: the same Q8_0 activation codes and weight blocks, each element dequantised to
    fp16 and multiplied on the fp16 tensor cores with fp32 accumulation over K.  Against the oracle's exact
    block-ordered sum it differs by rounding only: held to 1e-3 (max|d| / max|ref|, ten times inside the
    north-star 1e-2), on a sample of rows spread over every 128-row tile including the ragged last one."""
    wq, x, bias = _case(oracle, qt, M, K, N, seed=M + 5 * K + N)
    w = backend.weight(qt, wq, K, N)
    xd, bd = backend.upload(x), backend.upload(bias)
    yd = backend.alloc(M * N * 4)
    for _ in range(2):  # the second call reuses the weight's fp16 copy made by the first
        backend.mul_mat_dq16(w, xd, M, yd, bias=bd)
        backend.synchronize()
    got = yd.get((M, N), np.float32)
    rows = np.unique(np.clip(np.concatenate([np.arange(0, M, 97), [M - 1, M - 64, 5120, 127, 128]]), 0, M - 1))
    ref = oracle.mul_mat(qt, wq, K, N, x[rows]) + bias[None, :]
    err = np.max(np.abs(got[rows] - ref)) / np.max(np.abs(ref))
    assert err <= 1e-3, err
    w.free()


def test_mul_mat_dq16_refuses_other_weight_types(b200, backend):
    K, N, M = 64, 32, 8
    w = backend.weight(b200.TYPE_F16, np.zeros((N, K), np.float16).view(np.uint8), K, N)
    x, y = backend.alloc(M * K * 4), backend.alloc(M * N * 4)
    with pytest.raises(b200.B200Error, match="not supported"):
        backend.mul_mat_dq16(w, x, M, y)
    w.free()
