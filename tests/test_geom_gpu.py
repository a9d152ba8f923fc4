"""Geometry (exemplar-prompt) encoder transformer of the SAM3 detector (sam3.cpp:7677-7800) through the
C ABI against the CPU oracle (oracle/geom_oracle.py): 3 layers over box + CLS tokens attending to the
72 x 72 image tokens, Q4_0 weights."""
import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu

D, HEADS, LAYERS, FFN = 256, 8, 3, 2048


def make_geom_tensors(oracle, qtype=2, seed=0):
    rng = np.random.default_rng(seed)
    gpu, ref = {}, {}

    def f32(name, arr):
        arr = np.ascontiguousarray(arr, np.float32)
        gpu[name], ref[name] = (0, arr, arr.shape[::-1]), arr

    def lin(name, K, N):
        q = oracle.quantize_weights(qtype, rng.normal(0, 1.0 / np.sqrt(K), size=(N, K)).astype(np.float32))
        gpu[name], ref[name] = (qtype, q, (K, N)), (qtype, q, K, N)

    for i in range(LAYERS):
        p = f"geom.layers.{i}."
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
    f32("geom.encode_norm.weight", 1 + rng.normal(0, 0.1, size=D))
    f32("geom.encode_norm.bias", rng.normal(0, 0.1, size=D))
    return gpu, ref


@pytest.mark.parametrize("n_boxes,H", [(1, 72), (4, 72), (7, 24)])
def test_geom_matches_oracle(oracle, backend, n_boxes, H):
    import geom_oracle
    gpu, ref = make_geom_tensors(oracle, 2, seed=n_boxes)
    rng = np.random.default_rng(H + n_boxes)
    x = rng.normal(0, 1, size=(n_boxes + 1, D)).astype(np.float32)
    img = rng.normal(0, 1, size=(H * H, D)).astype(np.float32)
    pe = rng.normal(0, 1, size=(H * H, D)).astype(np.float32)
    ge = backend.geometry_encoder(dict(d_model=D, heads=HEADS, layers=LAYERS, ffn_dim=FFN, max_tokens=8,
                                       max_image_tokens=H * H))
    try:
        ge.load(gpu)
        got = ge.run(x, img, pe)
    finally:
        ge.free()
    want = geom_oracle.run(ref, LAYERS, HEADS, x, img, pe)
    bound = max(1e-2, 2 * rel_err(geom_oracle.run(ref, LAYERS, HEADS, x, img, pe, np.float32), want))
    assert np.isfinite(got).all()
    assert rel_err(got, want) <= bound, (rel_err(got, want), bound)


def test_geom_rejects(b200, backend):
    ge = backend.geometry_encoder(dict(d_model=D, heads=HEADS, layers=1, ffn_dim=FFN, max_tokens=2,
                                       max_image_tokens=16))
    try:
        with pytest.raises(b200.B200Error):
            ge.run(np.zeros((2, D), np.float32), np.zeros((16, D), np.float32), np.zeros((16, D), np.float32))
        with pytest.raises(b200.B200Error):
            ge.run(np.zeros((3, D), np.float32), np.zeros((16, D), np.float32), np.zeros((16, D), np.float32))
    finally:
        ge.free()
