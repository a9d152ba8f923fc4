"""Fusion encoder of the SAM3 detector (sam3.cpp:8033-8165) through the C ABI against the CPU oracle
(oracle/fenc_oracle.py): d_model 256, 8 heads, 6 layers, FFN 2048 (sam3.cpp:2655-2682), Q4_0 weights
as in config 4."""
import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu

D, HEADS, LAYERS, FFN = 256, 8, 6, 2048


def make_fenc_tensors(oracle, qtype=2, seed=0, layers=LAYERS):
    rng = np.random.default_rng(seed)
    gpu, ref = {}, {}

    def f32(name, arr):
        arr = np.ascontiguousarray(arr, np.float32)
        gpu[name], ref[name] = (0, arr, arr.shape[::-1]), arr

    def lin(name, K, N):
        q = oracle.quantize_weights(qtype, rng.normal(0, 1.0 / np.sqrt(K), size=(N, K)).astype(np.float32))
        gpu[name], ref[name] = (qtype, q, (K, N)), (qtype, q, K, N)

    for i in range(layers):
        p = f"fenc.layers.{i}."
        for a in ("sa", "ca"):
            lin(p + a + ".in_proj_weight", D, 3 * D)
            f32(p + a + ".in_proj_bias", rng.normal(0, 0.02, size=3 * D))
            lin(p + a + ".out_proj.weight", D, D)
            f32(p + a + ".out_proj.bias", rng.normal(0, 0.02, size=D))
        lin(p + "linear1.weight", D, FFN)
        f32(p + "linear1.bias", rng.normal(0, 0.02, size=FFN))
        lin(p + "linear2.weight", FFN, D)
        f32(p + "linear2.bias", rng.normal(0, 0.02, size=D))
        for n in ("norm1", "norm2", "norm3"):
            f32(p + n + ".weight", 1 + rng.normal(0, 0.1, size=D))
            f32(p + n + ".bias", rng.normal(0, 0.1, size=D))
    return gpu, ref


def make_inputs(H, T, n_valid, seed):
    rng = np.random.default_rng(seed)
    img = rng.normal(0, 1, size=(H * H, D)).astype(np.float32)
    prompt = rng.normal(0, 1, size=(T, D)).astype(np.float32)
    pos = rng.normal(0, 1, size=(H * H, D)).astype(np.float32)
    bias = np.where(np.arange(T) < n_valid, 0.0, -1.0e9).astype(np.float32)
    return img, prompt, pos, bias


def check(oracle, backend, H, T, n_valid, qtype=2, use_bias=True, seed=0):
    import fenc_oracle
    gpu, ref = make_fenc_tensors(oracle, qtype, seed)
    img, prompt, pos, bias = make_inputs(H, T, n_valid, seed + 1)
    bias = bias if use_bias else None
    fe = backend.fusion_encoder(dict(d_model=D, heads=HEADS, layers=LAYERS, ffn_dim=FFN, max_tokens=H * H,
                                     max_prompt=T))
    try:
        fe.load(gpu)
        got = fe.run(img, prompt, pos, bias)
    finally:
        fe.free()
    want = fenc_oracle.run(ref, LAYERS, HEADS, img, prompt, pos, bias)
    spread = rel_err(fenc_oracle.run(ref, LAYERS, HEADS, img, prompt, pos, bias, np.float32), want)
    bound = max(1e-2, 2 * spread)
    assert np.isfinite(got).all()
    assert rel_err(got, want) <= bound, (rel_err(got, want), bound)


@pytest.mark.parametrize("H,T,n_valid,qtype,use_bias", [
    (24, 32, 9, 2, True),     # padded text prompt, Q4_0
    (24, 32, 32, 8, False),   # no padding bias, Q8_0
    (24, 40, 17, 2, True),    # text + geometry tokens
])
def test_fenc_matches_oracle(oracle, backend, H, T, n_valid, qtype, use_bias):
    check(oracle, backend, H, T, n_valid, qtype, use_bias, seed=H + T)


def test_fenc_config4_size(oracle, backend):
    """Config 4: 72 x 72 image tokens, 32 text tokens of which 7 are valid."""
    check(oracle, backend, 72, 32, 7, 2, True, seed=4)


def test_fenc_padding_tokens_are_ignored(oracle, backend):
    """Tokens under a -1e9 bias do not reach the output: changing them leaves it bit-identical."""
    gpu, _ = make_fenc_tensors(oracle, 2, 3, layers=2)
    img, prompt, pos, bias = make_inputs(16, 32, 5, 4)
    fe = backend.fusion_encoder(dict(d_model=D, heads=HEADS, layers=2, ffn_dim=FFN, max_tokens=256, max_prompt=32))
    try:
        fe.load(gpu)
        a = fe.run(img, prompt, pos, bias)
        prompt2 = prompt.copy()
        prompt2[5:] = np.random.default_rng(9).normal(size=prompt2[5:].shape)
        b = fe.run(img, prompt2, pos, bias)
    finally:
        fe.free()
    assert np.array_equal(a, b)


def test_fenc_rejects(b200, backend):
    fe = backend.fusion_encoder(dict(d_model=D, heads=HEADS, layers=1, ffn_dim=FFN, max_tokens=16, max_prompt=4))
    try:
        x = np.zeros((16, D), np.float32)
        with pytest.raises(b200.B200Error):
            fe.run(x, np.zeros((4, D), np.float32), x)  # weights missing
        with pytest.raises(b200.B200Error):
            fe.run(x, np.zeros((5, D), np.float32), x)  # more prompt tokens than the capacity
    finally:
        fe.free()
    with pytest.raises(b200.B200Error):
        backend.fusion_encoder(dict(d_model=D, heads=3, layers=1, ffn_dim=FFN, max_tokens=16, max_prompt=4))
