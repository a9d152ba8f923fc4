"""DETR decoder of the SAM3 detector with scoring and presence head (sam3.cpp:8171-8888) through the
C ABI against the CPU oracle (oracle/ddec_oracle.py): d_model 256, 8 heads, 6 layers, FFN 2048, 200
queries over the 72 x 72 image tokens (config 4), Q4_0 weights; the K = 2 boxRPB layer in F32 as the
weight-type rule leaves it (sam3.cpp:2722-2734)."""
import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu

D, NH, FFN = 256, 8, 2048


def make_ddec_tensors(oracle, hp, qtype=2, seed=0):
    rng = np.random.default_rng(seed)
    gpu, ref = {}, {}
    NQ = hp["num_queries"]

    def f32(name, arr):
        arr = np.ascontiguousarray(arr, np.float32)
        gpu[name], ref[name] = (0, arr, arr.shape[::-1]), arr

    def lin(name, K, N, std=None):
        w = rng.normal(0, std or 1.0 / np.sqrt(K), size=(N, K)).astype(np.float32)
        q = oracle.quantize_weights(qtype, w)
        gpu[name + ".weight"], ref[name + ".weight"] = (qtype, q, (K, N)), (qtype, q, K, N)
        f32(name + ".bias", rng.normal(0, 0.02, size=N))

    def norm(name):
        f32(name + ".weight", 1 + rng.normal(0, 0.1, size=D))
        f32(name + ".bias", rng.normal(0, 0.1, size=D))

    f32("ddec.query_embed.weight", rng.normal(0, 1, size=(NQ, D)))
    f32("ddec.presence_token.weight", rng.normal(0, 1, size=(1, D)))
    f32("ddec.reference_points.weight", rng.normal(0, 1, size=(NQ, 4)))
    norm("ddec.norm")
    norm("ddec.presence_token_out_norm")
    norm("scoring.prompt_mlp.out_norm")
    for j in range(3):
        lin(f"ddec.bbox_embed.layers.{j}", D, 4 if j == 2 else D, std=0.02 if j == 2 else None)
        lin(f"ddec.presence_token_head.layers.{j}", D, 1 if j == 2 else D)
    lin("ddec.ref_point_head.layers.0", 512, D)
    lin("ddec.ref_point_head.layers.1", D, D)
    for a in ("x", "y"):
        w0 = rng.normal(0, 0.7, size=(D, 2)).astype(np.float32)
        gpu[f"ddec.boxRPB_embed_{a}.layers.0.weight"] = (0, w0, (2, D))
        ref[f"ddec.boxRPB_embed_{a}.layers.0.weight"] = (0, w0)
        f32(f"ddec.boxRPB_embed_{a}.layers.0.bias", rng.normal(0, 0.1, size=D))
        lin(f"ddec.boxRPB_embed_{a}.layers.1", D, NH)
    lin("scoring.prompt_mlp.layers.0", D, FFN)
    lin("scoring.prompt_mlp.layers.1", FFN, D)
    lin("scoring.prompt_proj", D, D)
    lin("scoring.hs_proj", D, D)
    for i in range(hp["layers"]):
        p = f"ddec.layers.{i}."
        for a in ("sa", "ca", "ca_text"):
            w = oracle.quantize_weights(qtype, rng.normal(0, 1 / 16, size=(3 * D, D)).astype(np.float32))
            gpu[p + a + ".in_proj_weight"], ref[p + a + ".in_proj_weight"] = (qtype, w, (D, 3 * D)), (qtype, w, D, 3 * D)
            f32(p + a + ".in_proj_bias", rng.normal(0, 0.02, size=3 * D))
            lin(p + a + ".out_proj", D, D)
        lin(p + "linear1", D, FFN)
        lin(p + "linear2", FFN, D)
        for n in ("norm1", "norm2", "norm_ca_text", "norm3"):
            norm(p + n)
    return gpu, ref


def make_inputs(S, T, n_valid, seed):
    rng = np.random.default_rng(seed)
    enc = rng.normal(0, 1, size=(S * S, D)).astype(np.float32)
    pos = rng.normal(0, 1, size=(S * S, D)).astype(np.float32)
    text = rng.normal(0, 1, size=(T, D)).astype(np.float32)
    bias = np.where(np.arange(T) < n_valid, 0.0, -1.0e9).astype(np.float32)
    valid = np.where(np.arange(T) < n_valid, T / n_valid, 0.0).astype(np.float32)
    return enc, pos, text, bias, valid


def check(oracle, backend, hp, T, n_valid, masks=True, seed=0):
    import ddec_oracle
    gpu, ref = make_ddec_tensors(oracle, hp, 2, seed)
    enc, pos, text, bias, valid = make_inputs(hp["feat"], T, n_valid, seed + 1)
    if not masks:
        bias = valid = None
    dd = backend.detr_decoder(dict(hp, max_prompt=T))
    try:
        dd.load(gpu)
        got = dd.run(enc, pos, text, bias, valid)
    finally:
        dd.free()
    want = ddec_oracle.run(hp, ref, enc, pos, text, bias, valid)
    other = ddec_oracle.run(hp, ref, enc, pos, text, bias, valid, np.float32)
    for key in ("queries", "boxes", "scores"):
        bound = max(1e-2, 2 * rel_err(other[key], want[key]))
        assert np.isfinite(got[key]).all(), key
        assert rel_err(got[key], want[key]) <= bound, (key, rel_err(got[key], want[key]), bound)
    assert abs(got["presence"] - want["presence"]) <= 1e-2 * max(1.0, abs(want["presence"])) + \
        2 * abs(other["presence"] - want["presence"])


HP = dict(d_model=D, heads=NH, layers=6, ffn_dim=FFN, num_queries=200, feat=72)


def test_ddec_config4(oracle, backend):
    """Config 4's decoder: 200 queries over 72 x 72 tokens, 32 text tokens of which 7 are valid."""
    check(oracle, backend, HP, 32, 7, True, seed=4)


@pytest.mark.parametrize("feat,T,n_valid,masks", [(24, 32, 12, True), (24, 16, 16, False)])
def test_ddec_small_grids(oracle, backend, feat, T, n_valid, masks):
    check(oracle, backend, dict(HP, layers=2, num_queries=50, feat=feat), T, n_valid, masks, seed=feat + T)


def test_ddec_rejects(b200, backend):
    dd = backend.detr_decoder(dict(HP, layers=1, num_queries=4, feat=4, max_prompt=4))
    try:
        x = np.zeros((16, D), np.float32)
        with pytest.raises(b200.B200Error):
            dd.run(x, x, np.zeros((4, D), np.float32))  # weights missing
        with pytest.raises(b200.B200Error):
            dd.run(x, x, np.zeros((5, D), np.float32))  # more text tokens than the capacity
    finally:
        dd.free()
    with pytest.raises(b200.B200Error):
        backend.detr_decoder(dict(HP, heads=4, max_prompt=4))
