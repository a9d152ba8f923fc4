"""Op-level entry points of the drop-in boundary (the ggml ops sam3.cpp's
graphs dispatch besides MUL_MAT), through the C ABI, against the oracle."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("batch,heads,N", [(1, 2, 64), (2, 3, 200), (9, 2, 576), (1, 1, 8)])
def test_flash_attn_ext_matches_oracle(oracle, backend, batch, heads, N):
    """GGML_OP_FLASH_ATTN_EXT (sam3.cpp:3778): bf16 tensor-core attention within 1e-2 of the f32 oracle."""
    rng = np.random.default_rng(batch * 1000 + heads * 100 + N)
    q, k, v = (rng.normal(0, 1, size=(batch * heads, N, 64)).astype(np.float32) for _ in range(3))
    scale = 0.125
    dq, dk, dv = backend.upload(q), backend.upload(k), backend.upload(v)
    out = backend.alloc(batch * N * heads * 64 * 4)
    backend.flash_attn_ext(dq, dk, dv, 64, N, heads, batch, scale, out)
    backend.synchronize()
    got = out.get((batch * N, heads * 64), np.float32)
    ref = oracle.attention(q, k, v, batch, N, heads, scale)
    err = np.abs(got - ref).max() / np.abs(ref).max()
    assert err <= 1e-2, err


def test_flash_attn_ext_rejects_unsupported(b200, backend):
    buf = backend.alloc(4096)
    with pytest.raises(b200.B200Error):
        backend.flash_attn_ext(buf, buf, buf, 128, 8, 1, 1, 0.1, buf)  # head dim 128
    with pytest.raises(b200.B200Error):
        backend.flash_attn_ext(buf, buf, buf, 64, 12, 1, 1, 0.1, buf)  # N not a multiple of 8
