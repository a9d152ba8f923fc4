"""CPU checks of the text-encoder oracle (oracle/text_oracle.py) on a small configuration."""
import numpy as np

from test_text_gpu import make_text_tensors

SMALL = dict(width=64, heads=4, layers=2, ctx_len=8, vocab=50, out_dim=16)


def test_text_oracle_causal_and_padding(oracle):
    import text_oracle
    _, ref = make_text_tensors(oracle, SMALL, seed=1)
    a = text_oracle.encode(SMALL, ref, [5, 9, 11])
    assert a.shape == (8, 16) and np.isfinite(a).all()
    b = text_oracle.encode(SMALL, ref, [5, 9, 12])
    np.testing.assert_array_equal(a[:2], b[:2])  # later tokens do not reach earlier rows
    assert not np.array_equal(a[2:], b[2:])
    c = text_oracle.encode(SMALL, ref, [5, 9, 11, 0, 0])  # explicit zeros equal the implicit padding
    np.testing.assert_array_equal(a, c)
