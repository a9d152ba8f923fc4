"""Tracker memory attention (sam3.cpp:9228-9341) through the C ABI against the CPU oracle
(oracle/mem_attn_oracle.py): d_model 256, mem_dim 64, 4 layers, FFN 2048, as the SAM2/SAM3 trackers
register them (sam3.cpp:2008-2042)."""
import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu

D, MD, LAYERS, FFN = 256, 64, 4, 2048


def make_mem_tensors(oracle, qtype=8, seed=0):
    rng = np.random.default_rng(seed)
    gpu, ref = {}, {}

    def f32(name, arr):
        arr = np.ascontiguousarray(arr, np.float32)
        gpu[name], ref[name] = (0, arr, arr.shape[::-1]), arr

    def lin(name, K, N):
        q = oracle.quantize_weights(qtype, rng.normal(0, 1.0 / np.sqrt(K), size=(N, K)).astype(np.float32))
        gpu[name + ".weight"], ref[name + ".weight"] = (qtype, q, (K, N)), (qtype, q, K, N)
        f32(name + ".bias", rng.normal(0, 0.02, size=N))

    for i in range(LAYERS):
        p = f"mem_attn.layers.{i}."
        for n in ("sa.q_proj", "sa.k_proj", "sa.v_proj", "sa.out_proj", "ca.q_proj", "ca.out_proj"):
            lin(p + n, D, D)
        lin(p + "ca.k_proj", MD, D)
        lin(p + "ca.v_proj", MD, D)
        lin(p + "linear1", D, FFN)
        lin(p + "linear2", FFN, D)
        for n in ("norm1", "norm2", "norm3"):
            f32(p + n + ".weight", 1 + rng.normal(0, 0.1, size=D))
            f32(p + n + ".bias", rng.normal(0, 0.1, size=D))
    f32("mem_attn.norm.weight", 1 + rng.normal(0, 0.1, size=D))
    f32("mem_attn.norm.bias", rng.normal(0, 0.1, size=D))
    return gpu, ref


def make_inputs(H, n_frames, n_ptr, seed):
    """A current frame of H x H tokens, n_frames spatial memories of H x H tokens (their RoPE table the
    frame's table repeated, as sam3_propagate_single builds it) and n_ptr object-pointer tokens."""
    import mem_attn_oracle
    rng = np.random.default_rng(seed)
    N, M = H * H, n_frames * H * H + n_ptr
    curr = rng.normal(0, 1, size=(N, D)).astype(np.float32)
    spos = rng.normal(0, 1, size=(N, D)).astype(np.float32)
    prompt = rng.normal(0, 1, size=(M, MD)).astype(np.float32)
    ppos = rng.normal(0, 1, size=(M, MD)).astype(np.float32)
    rq = mem_attn_oracle.axial_cis(D, H, H)
    rk = np.concatenate([rq] * n_frames) if n_frames else None
    return curr, spos, prompt, ppos, rq, rk


def check(oracle, backend, H, n_frames, n_ptr, qtype=8, seed=0, drop_rope_k=False):
    import mem_attn_oracle
    gpu, ref = make_mem_tensors(oracle, qtype, seed)
    curr, spos, prompt, ppos, rq, rk = make_inputs(H, n_frames, n_ptr, seed + 1)
    if drop_rope_k:
        rk = None
    hp = dict(d_model=D, mem_dim=MD, layers=LAYERS, ffn_dim=FFN, max_tokens=H * H, max_mem_tokens=prompt.shape[0])
    ma = backend.mem_attention(hp)
    try:
        ma.load(gpu)
        got = ma.run(curr, spos, prompt, ppos, rq, rk, n_ptr)
    finally:
        ma.free()
    want = mem_attn_oracle.run(ref, LAYERS, curr, spos, prompt, ppos, rq, rk, n_ptr)
    spread = rel_err(mem_attn_oracle.run(ref, LAYERS, curr, spos, prompt, ppos, rq, rk, n_ptr, np.float32), want)
    bound = max(1e-2, 2 * spread)
    err = rel_err(got, want)
    assert np.isfinite(got).all()
    assert err <= bound, (err, bound)
    return err


@pytest.mark.parametrize("n_frames,n_ptr,qtype,drop_rope_k", [
    (2, 16, 8, False),   # spatial memories + object pointers, Q8_0
    (3, 0, 8, False),    # no object pointers
    (1, 8, 2, False),    # Q4_0 weights
    (2, 16, 8, True),    # no key rotation (rope_k absent)
    (0, 16, 8, False),   # object pointers only
])
def test_mem_attn_matches_oracle(oracle, backend, n_frames, n_ptr, qtype, drop_rope_k):
    check(oracle, backend, 32, n_frames, n_ptr, qtype, seed=n_frames + n_ptr, drop_rope_k=drop_rope_k)


def test_mem_attn_config5_size(oracle, backend):
    """Config 5's tracker (Hiera-B+ at 1024: 64 x 64 tokens), seven memory frames and 16 object pointers
    split into 64 tokens of mem_dim."""
    check(oracle, backend, 64, 7, 64, 8, seed=5)


def test_mem_attn_rejects(b200, backend):
    hp = dict(d_model=D, mem_dim=MD, layers=1, ffn_dim=FFN, max_tokens=16, max_mem_tokens=16)
    ma = backend.mem_attention(hp)
    try:
        x = np.zeros((16, D), np.float32)
        p = np.zeros((16, MD), np.float32)
        r = np.zeros((16, D // 2, 2), np.float32)
        with pytest.raises(b200.B200Error):
            ma.run(x, x, p, p, r, None, 0)  # weights missing
    finally:
        ma.free()
    with pytest.raises(b200.B200Error):
        backend.mem_attention(dict(hp, d_model=200))
