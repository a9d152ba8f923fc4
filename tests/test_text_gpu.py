"""SAM3 text encoder (the PCS path's text side, sam3.cpp:3943-4066) through the C ABI against the CPU
oracle (oracle/text_oracle.py), at config 4's sizes: width 1024, 24 layers, 32-token context, vocabulary
49408, Q4_0 linear weights."""
import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu

HP = dict(width=1024, heads=16, layers=24, ctx_len=32, vocab=49408, out_dim=256)


def make_text_tensors(oracle, hp, qtype=2, seed=0):
    rng = np.random.default_rng(seed)
    E = hp["width"]
    gpu, ref = {}, {}

    def f32(name, arr, ne):
        arr = np.ascontiguousarray(arr, np.float32)
        gpu[name], ref[name] = (0, arr, ne), arr

    def lin(name, K, N):
        q = oracle.quantize_weights(qtype, rng.normal(0, 0.02, size=(N, K)).astype(np.float32))
        gpu[name], ref[name] = (qtype, q, (K, N)), (qtype, q, K, N)

    f32("text.token_embed.weight", rng.normal(0, 0.02, size=(hp["vocab"], E)), (E, hp["vocab"]))
    f32("text.pos_embed", rng.normal(0, 0.01, size=(hp["ctx_len"], E)), (E, hp["ctx_len"]))
    for i in range(hp["layers"]):
        p = f"text.blocks.{i}."
        lin(p + "attn.in_proj.weight", E, 3 * E)
        f32(p + "attn.in_proj.bias", rng.normal(0, 0.02, size=3 * E), (3 * E,))
        lin(p + "attn.out_proj.weight", E, E)
        f32(p + "attn.out_proj.bias", rng.normal(0, 0.02, size=E), (E,))
        for n in ("ln_1", "ln_2"):
            f32(p + n + ".weight", 1 + rng.normal(0, 0.1, size=E), (E,))
            f32(p + n + ".bias", rng.normal(0, 0.1, size=E), (E,))
        lin(p + "mlp.fc1.weight", E, 4 * E)
        f32(p + "mlp.fc1.bias", rng.normal(0, 0.02, size=4 * E), (4 * E,))
        lin(p + "mlp.fc2.weight", 4 * E, E)
        f32(p + "mlp.fc2.bias", rng.normal(0, 0.02, size=E), (E,))
    f32("text.ln_final.weight", 1 + rng.normal(0, 0.1, size=E), (E,))
    f32("text.ln_final.bias", rng.normal(0, 0.1, size=E), (E,))
    lin("text.resizer.weight", E, hp["out_dim"])
    f32("text.resizer.bias", rng.normal(0, 0.02, size=hp["out_dim"]), (hp["out_dim"],))
    return gpu, ref


@pytest.fixture(scope="module")
def text_setup(oracle, backend):
    gpu, ref = make_text_tensors(oracle, HP, seed=7)
    enc = backend.text_encoder(HP)
    enc.load(gpu)
    yield enc, ref
    enc.free()


@pytest.mark.parametrize("n_ids", [1, 12, 32])
def test_text_encoder_matches_oracle(text_setup, n_ids):
    """Chained quantised layers amplify rounding-level differences, so the bound is 1e-2 or twice the
    spread between two valid oracle evaluations (attention in float64 and in float32), as for Hiera."""
    import text_oracle
    enc, ref = text_setup
    ids = np.random.default_rng(n_ids).integers(0, HP["vocab"], size=n_ids).astype(np.int32)
    got = enc.encode(ids)
    want = text_oracle.encode(HP, ref, ids)
    bound = max(1e-2, 2 * rel_err(text_oracle.encode(HP, ref, ids, np.float32), want))
    assert got.shape == (HP["ctx_len"], HP["out_dim"])
    assert rel_err(got, want) <= bound, (rel_err(got, want), bound)


def test_text_encoder_rejects(b200, backend):
    enc = backend.text_encoder(dict(HP, layers=1, vocab=100))
    try:
        with pytest.raises(b200.B200Error):
            enc.encode(np.array([1, 2], np.int32))  # weights missing
        with pytest.raises(b200.B200Error):
            enc.encode(np.array([100], np.int32))  # outside the vocabulary
    finally:
        enc.free()


def test_text_encoder_is_causal(text_setup):
    """Row j reads only tokens 0..j (causal mask; row-wise LayerNorm and MUL_MAT), so changing later tokens
    leaves the earlier rows bit-identical."""
    enc, _ = text_setup
    ids = np.random.default_rng(3).integers(0, HP["vocab"], size=20).astype(np.int32)
    a = enc.encode(ids)
    ids2 = ids.copy()
    ids2[10:] = (ids2[10:] + 17) % HP["vocab"]
    b = enc.encode(ids2)
    assert np.array_equal(a[:10], b[:10])
    assert not np.array_equal(a[10:], b[10:])
