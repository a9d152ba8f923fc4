"""CPU tests of the oracle itself: pinned against the gguf golden vectors,
plus internal consistency of the block-dot formula."""
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "quants_golden.npz")


@pytest.mark.parametrize("name,qt", [("q8_0", 8), ("q4_0", 2), ("q4_1", 3)])
@pytest.mark.parametrize("src", ["w", "x", "edge"])
def test_weight_quantisers_match_gguf(oracle, name, qt, src):
    g = np.load(GOLDEN)
    rows = g[src]
    q = oracle.quantize_weights(qt, rows)
    assert np.array_equal(q, g[f"{name}_{src}_q"])
    dq = oracle.dequantize(qt, q, rows.shape[1])
    assert np.array_equal(dq, g[f"{name}_{src}_dq"])


def test_fp16_roundtrip_rne(oracle):
    L = oracle.lib()
    # halfway cases round to even; overflow saturates to inf; subnormals kept
    cases = {1.0: 0x3C00, 65504.0: 0x7BFF, 65520.0: 0x7C00, 1.0 + 2 ** -11: 0x3C00,
             1.0 + 3 * 2 ** -11: 0x3C02, 2 ** -24: 0x0001, 2 ** -25: 0x0000, -0.0: 0x8000}
    for f, bits in cases.items():
        assert L.orc_fp32_to_fp16(f) == bits, f


def test_activation_rule_vs_weight_rule(oracle):
    """The activation quantiser (x86 rule: 127/amax, round-half-even) and the
    reference weight quantiser (1/(amax/127), roundf) agree on scales always
    and on codes except at rounding ties."""
    rng = np.random.default_rng(1)
    x = rng.normal(0, 1, size=(64, 1024)).astype(np.float32)
    a = oracle.quantize_activations(oracle.Q8_0, x).reshape(64, 32, 34)
    w = oracle.quantize_weights(oracle.Q8_0, x).reshape(64, 32, 34)
    assert np.array_equal(a[..., :2], w[..., :2])
    diff = (a[..., 2:].view(np.int8).astype(int) - w[..., 2:].view(np.int8).astype(int))
    assert np.abs(diff).max() <= 1
    assert (diff != 0).mean() < 1e-3


def test_q8_1_sum_field(oracle):
    rng = np.random.default_rng(2)
    x = rng.normal(0, 1, size=(4, 128)).astype(np.float32)
    q = oracle.quantize_activations(oracle.Q8_1, x).reshape(4, 4, 36)
    # s = fp16(d * sum(q)) with the unrounded fp32 d = amax / 127
    d = (np.abs(x.reshape(4, 4, 32)).max(-1) / np.float32(127)).astype(np.float32)
    s = q[..., 2:4].copy().view(np.float16).astype(np.float32)[..., 0]
    qs = q[..., 4:].view(np.int8).astype(np.int64).sum(-1)
    assert np.array_equal(s, (d * qs.astype(np.float32)).astype(np.float16).astype(np.float32))


@pytest.mark.parametrize("qt", [8, 2, 3])
def test_mul_mat_matches_dequantised_float(oracle, qt):
    """The block formula equals the float product of the dequantised operands
    up to fp32 rounding."""
    rng = np.random.default_rng(3)
    K, N, M = 256, 48, 17
    w = rng.normal(0, 0.02, size=(N, K)).astype(np.float32)
    x = rng.normal(0, 1, size=(M, K)).astype(np.float32)
    wq = oracle.quantize_weights(qt, w)
    y = oracle.mul_mat(qt, wq, K, N, x)
    vt = 9 if qt == 3 else 8
    xq = oracle.quantize_activations(vt, x)
    ref = oracle.dequantize(vt, xq, K).astype(np.float64) @ oracle.dequantize(qt, wq, K).astype(np.float64).T
    if qt == 3:
        # Q4_1 uses the fp16-rounded s = d*sum(q) term, so it differs from the
        # dequantised product by the rounding of s.
        assert np.max(np.abs(y - ref)) / np.max(np.abs(ref)) < 2e-3
    else:
        assert np.max(np.abs(y - ref)) / np.max(np.abs(ref)) < 1e-5


def test_block_dots_consistent_with_mul_mat(oracle):
    rng = np.random.default_rng(4)
    K, N, M = 128, 8, 5
    w = rng.normal(0, 0.02, size=(N, K)).astype(np.float32)
    x = rng.normal(0, 1, size=(M, K)).astype(np.float32)
    wq = oracle.quantize_weights(8, w)
    bd = oracle.block_dots(8, wq, K, N, x)
    xq = oracle.quantize_activations(8, x).reshape(M, K // 32, 34)
    wqq = wq.reshape(N, K // 32, 34)
    dx = xq[..., :2].copy().view(np.float16).astype(np.float32)[..., 0]
    dw = wqq[..., :2].copy().view(np.float16).astype(np.float32)[..., 0]
    y = np.zeros((M, N), np.float32)
    for b in range(K // 32):
        y = (bd[:, :, b].astype(np.float32) * (dw[None, :, b] * dx[:, None, b]) + y).astype(np.float32)
    y2 = oracle.mul_mat(8, wq, K, N, x)
    assert np.max(np.abs(y - y2)) <= 1e-6 * np.max(np.abs(y2))
    qx = xq[..., 2:].view(np.int8).astype(np.int64)
    qw = wqq[..., 2:].view(np.int8).astype(np.int64)
    assert np.array_equal(bd, np.einsum("mbk,nbk->mnb", qx, qw).astype(np.int32))


@pytest.mark.parametrize("qt", [8, 2])  # Q8_0, Q4_0
@pytest.mark.parametrize("M,K,N", [(192, 1024, 384), (96, 4736, 256), (130, 96, 288)])
def test_dq16_arithmetic_within_rounding_of_the_exact_fold(oracle, qt, M, K, N):
    """The DQ16 arithmetic (Q8_0 activation codes and weight blocks dequantised to fp16, one fp16 product
    per element, wide accumulation) against the exact block-ordered fold of the same codes: they differ by
    the two fp16 roundings only, far inside the north-star 1e-2 (max|d| / max|ref|; observed ~3e-4)."""
    rng = np.random.default_rng(M + K + N + qt)
    w = rng.normal(0, 0.02, size=(N, K)).astype(np.float32)
    x = rng.normal(0, 1, size=(M, K)).astype(np.float32)
    wq = oracle.quantize_weights(qt, w)
    exact = oracle.mul_mat(qt, wq, K, N, x)
    dq = oracle.mul_mat_dq16(qt, wq, K, N, x)
    err = float(np.max(np.abs(dq - exact)) / np.max(np.abs(exact)))
    assert err <= 1e-3, err
    assert err > 0.0  # the roundings are real: the two arithmetics are not the same function
