"""Segmentation head of the SAM3 detector (sam3.cpp:8899-9058) through the C ABI against the CPU oracle
(oracle/seghead_oracle.py): the pixel decoder to 4 * feat, the instance head and the mask product;
Q4_0 linear weights with F32 convolution kernels (quantised files) and an F16 variant."""
import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu

D = 256


def make_seg_tensors(oracle, ftype=2, seed=0):
    rng = np.random.default_rng(seed)
    gpu, ref = {}, {}

    def f32(name, arr):
        arr = np.ascontiguousarray(arr, np.float32)
        gpu[name], ref[name] = (0, arr, arr.shape[::-1]), arr

    def lin(name, K, N):
        w = rng.normal(0, 1.0 / np.sqrt(K), size=(N, K)).astype(np.float32)
        if ftype == 1:
            w16 = w.astype(np.float16)
            gpu[name + ".weight"], ref[name + ".weight"] = (1, w16, (K, N)), (1, w16, K, N)
        else:
            q = oracle.quantize_weights(ftype, w)
            gpu[name + ".weight"], ref[name + ".weight"] = (ftype, q, (K, N)), (ftype, q, K, N)
        f32(name + ".bias", rng.normal(0, 0.02, size=N))

    def conv(name, o, c, k):
        w = rng.normal(0, 1.0 / np.sqrt(c * k * k), size=(o, c, k, k)).astype(np.float32)
        if ftype == 1:
            w16 = w.astype(np.float16)
            gpu[name], ref[name] = (1, w16, (k, k, c, o)), (1, w16.astype(np.float32))
        else:
            gpu[name], ref[name] = (0, w, (k, k, c, o)), (0, w)

    lin("seg.cross_attend_prompt.out_proj", D, D)
    w = rng.normal(0, 1 / 16, size=(3 * D, D)).astype(np.float32)
    if ftype == 1:
        w16 = w.astype(np.float16)
        gpu["seg.cross_attend_prompt.in_proj_weight"] = (1, w16, (D, 3 * D))
        ref["seg.cross_attend_prompt.in_proj_weight"] = (1, w16, D, 3 * D)
    else:
        q = oracle.quantize_weights(ftype, w)
        gpu["seg.cross_attend_prompt.in_proj_weight"] = (ftype, q, (D, 3 * D))
        ref["seg.cross_attend_prompt.in_proj_weight"] = (ftype, q, D, 3 * D)
    f32("seg.cross_attend_prompt.in_proj_bias", rng.normal(0, 0.02, size=3 * D))
    f32("seg.cross_attn_norm.weight", 1 + rng.normal(0, 0.1, size=D))
    f32("seg.cross_attn_norm.bias", rng.normal(0, 0.1, size=D))
    for i in range(3):
        conv(f"seg.pixel_decoder.conv_layers.{i}.weight", D, D, 3)
        f32(f"seg.pixel_decoder.conv_layers.{i}.bias", rng.normal(0, 0.1, size=D))
        f32(f"seg.pixel_decoder.norms.{i}.weight", 1 + rng.normal(0, 0.1, size=D))
        f32(f"seg.pixel_decoder.norms.{i}.bias", rng.normal(0, 0.1, size=D))
    conv("seg.instance_seg_head.weight", D, D, 1)
    f32("seg.instance_seg_head.bias", rng.normal(0, 0.1, size=D))
    for j in range(3):
        lin(f"seg.mask_predictor.mask_embed.layers.{j}", D, D)
    return gpu, ref


def check(oracle, backend, S, nq, T, n_valid, ftype, seed):
    import seghead_oracle
    gpu, ref = make_seg_tensors(oracle, ftype, seed)
    rng = np.random.default_rng(seed + 1)
    enc = rng.normal(0, 1, size=(S * S, D)).astype(np.float32)
    fpn0 = rng.normal(0, 1, size=(16 * S * S, D)).astype(np.float32)
    fpn1 = rng.normal(0, 1, size=(4 * S * S, D)).astype(np.float32)
    queries = rng.normal(0, 1, size=(nq, D)).astype(np.float32)
    text = rng.normal(0, 1, size=(T, D)).astype(np.float32)
    bias = np.where(np.arange(T) < n_valid, 0.0, -1.0e9).astype(np.float32)
    sh = backend.seg_head(dict(d_model=D, heads=8, feat=S, max_queries=nq, max_prompt=T))
    try:
        sh.load(gpu)
        got = sh.run(enc, fpn0, fpn1, queries, text, bias)
    finally:
        sh.free()
    want = seghead_oracle.run(ref, S, enc, fpn0, fpn1, queries, text, bias)
    assert got.shape == want.shape and np.isfinite(got).all()
    assert rel_err(got, want) <= 1e-2, rel_err(got, want)


def test_seghead_config4(oracle, backend):
    """Config 4: 72 x 72 encoder tokens -> 288 x 288 masks for 200 queries, Q4_0 weights."""
    check(oracle, backend, 72, 200, 32, 7, 2, seed=4)


def test_seghead_f16_small(oracle, backend):
    """F16 weight file (F16 convolution kernels: fp16-rounded im2col input) on a 16 x 16 grid."""
    check(oracle, backend, 16, 10, 8, 5, 1, seed=6)


def test_seghead_rejects(b200, backend):
    sh = backend.seg_head(dict(d_model=D, heads=8, feat=4, max_queries=2, max_prompt=2))
    try:
        z = np.zeros((16, D), np.float32)
        with pytest.raises(b200.B200Error):
            sh.run(z, np.zeros((256, D), np.float32), np.zeros((64, D), np.float32), z[:2], z[:2])  # no weights
    finally:
        sh.free()
