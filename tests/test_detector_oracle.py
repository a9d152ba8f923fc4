"""CPU properties of the detector oracles (fusion encoder, DETR decoder, segmentation head, geometry
encoder) on small inputs: the structure the GPU parity tests rely on."""
import numpy as np

from test_ddec_gpu import make_ddec_tensors
from test_fenc_gpu import make_fenc_tensors
from test_geom_gpu import make_geom_tensors

D = 256


def test_fenc_oracle_ignores_padded_prompt_tokens(oracle):
    import fenc_oracle
    _, ref = make_fenc_tensors(oracle, 2, 0, layers=2)
    rng = np.random.default_rng(1)
    img, pos = rng.normal(size=(16, D)).astype(np.float32), rng.normal(size=(16, D)).astype(np.float32)
    prompt = rng.normal(size=(8, D)).astype(np.float32)
    bias = np.where(np.arange(8) < 3, 0.0, -1e9).astype(np.float32)
    a = fenc_oracle.run(ref, 2, 8, img, prompt, pos, bias)
    prompt[3:] = rng.normal(size=(5, D))
    np.testing.assert_array_equal(a, fenc_oracle.run(ref, 2, 8, img, prompt, pos, bias))


def test_ddec_oracle_box_code_and_refinement(oracle):
    import ddec_oracle
    d = np.linspace(-1, 1, 41, dtype=np.float32)
    np.testing.assert_array_equal(ddec_oracle.rpb_log(-d), -ddec_oracle.rpb_log(d))
    assert abs(ddec_oracle.rpb_log(np.float32([0.875]))[0] - 1.0) < 1e-6  # log2(8) / log2(8)
    boxes = np.float32([[0.5, 0.25, 0.1, 0.2]])
    s = ddec_oracle.sine_embed(boxes)
    assert s.shape == (1, 512)
    np.testing.assert_allclose(s[0, 1], np.cos(np.float32(2 * np.pi) * np.float32(0.25)), atol=1e-6)  # cy first
    hp = dict(d_model=D, heads=8, layers=1, ffn_dim=2048, num_queries=6, feat=4)
    _, ref = make_ddec_tensors(oracle, hp, 2, 3)
    rng = np.random.default_rng(4)
    out = ddec_oracle.run(hp, ref, rng.normal(size=(16, D)).astype(np.float32),
                          rng.normal(size=(16, D)).astype(np.float32), rng.normal(size=(5, D)).astype(np.float32))
    assert out["queries"].shape == (7, D) and out["scores"].shape == (6,)
    assert np.all((out["boxes"] > 0) & (out["boxes"] < 1)) and np.all(np.abs(out["scores"]) <= 12)


def test_seghead_oracle_pieces():
    import seghead_oracle
    rng = np.random.default_rng(5)
    prev = rng.normal(size=(4, 3)).astype(np.float32)  # 2 x 2 map, 3 channels
    up = seghead_oracle.up2_add(np.zeros((16, 3), np.float32), prev, 4).reshape(4, 4, 3)
    np.testing.assert_array_equal(up[1, 1], prev[0])
    np.testing.assert_array_equal(up[3, 2], prev[3])
    x = rng.normal(size=(64, 16)).astype(np.float32) * 3 + 5
    y = seghead_oracle.group_norm_relu(x, 8, np.ones(16), np.zeros(16))
    z = seghead_oracle.group_norm_relu(-x, 8, -np.ones(16), np.zeros(16))  # relu(n) and relu(-(-n))
    np.testing.assert_allclose(y, z, atol=1e-5)


def test_geom_oracle_is_permutation_equivariant(oracle):
    import geom_oracle
    _, ref = make_geom_tensors(oracle, 2, 6)
    rng = np.random.default_rng(7)
    x = rng.normal(size=(5, D)).astype(np.float32)
    img, pe = rng.normal(size=(16, D)).astype(np.float32), rng.normal(size=(16, D)).astype(np.float32)
    perm = np.array([3, 0, 4, 1, 2])
    a = geom_oracle.run(ref, 3, 8, x, img, pe)
    b = geom_oracle.run(ref, 3, 8, x[perm], img, pe)
    np.testing.assert_allclose(a[perm], b, rtol=1e-4, atol=1e-4)
