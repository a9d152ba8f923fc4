"""CPU checks of the memory-attention oracle (oracle/mem_attn_oracle.py)."""
import numpy as np

from test_mem_attn_gpu import LAYERS, make_inputs, make_mem_tensors


def test_rope_is_complex_rotation():
    import mem_attn_oracle
    rng = np.random.default_rng(0)
    x = rng.normal(size=(5, 8)).astype(np.float32)
    cs = mem_attn_oracle.axial_cis(8, 5, 1)
    z = (x[:, 0::2] + 1j * x[:, 1::2]) * (cs[..., 0] + 1j * cs[..., 1])
    y = mem_attn_oracle.rope(x, cs)
    np.testing.assert_allclose(y[:, 0::2], z.real, atol=1e-6)
    np.testing.assert_allclose(y[:, 1::2], z.imag, atol=1e-6)
    np.testing.assert_array_equal(mem_attn_oracle.rope(x, mem_attn_oracle.axial_cis(8, 1, 1).repeat(5, 0)), x)


def test_memory_order_does_not_matter(oracle):
    """Cross-attention is a set operation over the memory tokens: permuting them together with their RoPE
    rows leaves the result unchanged (up to summation order)."""
    import mem_attn_oracle
    _, ref = make_mem_tensors(oracle, 8, 1)
    c, s, p, pp, rq, rk = make_inputs(8, 2, 0, 2)
    a = mem_attn_oracle.run(ref, LAYERS, c, s, p, pp, rq, rk, 0)
    perm = np.random.default_rng(3).permutation(p.shape[0])
    b = mem_attn_oracle.run(ref, LAYERS, c, s, p[perm], pp[perm], rq, rk[perm], 0)
    np.testing.assert_allclose(a, b, rtol=1e-4, atol=1e-4)
