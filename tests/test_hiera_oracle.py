"""CPU checks of the Hiera oracle's own pieces (no GPU)."""
import numpy as np
import pytest

import hiera_oracle


def test_tiny_block_metadata_matches_reference_rules():
    """Hiera-tiny (convert_sam2_to_ggml.py:81-84) under sam2_precompute_hiera_metadata's rules: the
    window size lags a block into each new stage, Q-stride at the first block of stages 1-3."""
    from hiera_model import hiera_tiny
    blocks, ends = hiera_oracle.metadata(hiera_tiny(1024))
    assert ends == [0, 2, 9, 11]
    got = [(b["dim_in"], b["dim_out"], b["heads"], b["ws"], b["q_stride"]) for b in blocks]
    assert got == [(96, 96, 1, 8, False), (96, 192, 2, 8, True), (192, 192, 2, 4, False),
                   (192, 384, 4, 4, True), (384, 384, 4, 14, False), (384, 384, 4, 0, False),
                   (384, 384, 4, 14, False), (384, 384, 4, 0, False), (384, 384, 4, 14, False),
                   (384, 384, 4, 0, False), (384, 768, 8, 14, True), (768, 768, 8, 7, False)]


@pytest.mark.parametrize("H,W,ws", [(16, 16, 8), (16, 16, 14), (8, 8, 7), (12, 10, 4)])
def test_window_partition_round_trip(H, W, ws):
    x = np.random.default_rng(H * W + ws).normal(size=(H, W, 5)).astype(np.float32)
    win, Hp, Wp = hiera_oracle.window_partition(x, ws)
    assert win.shape == ((Hp // ws) * (Wp // ws), ws * ws, 5)
    # window wy + nWh * wx holds rows ws*wy.. and columns ws*wx.. in row-major local order
    nWh = Hp // ws
    wy, wx = 1 % nWh, (1 // nWh)
    ref = np.zeros((ws, ws, 5), np.float32)
    blk = x[ws * wy:ws * wy + ws, ws * wx:ws * wx + ws]
    ref[:blk.shape[0], :blk.shape[1]] = blk
    assert np.array_equal(win[1].reshape(ws, ws, 5), ref)
    assert np.array_equal(hiera_oracle.window_unpartition(win, ws, Hp, Wp, H, W), x)


def test_gelu_table_semantics():
    x = np.array([-12.0, -10.0, -1.2345678, 0.0, 0.1, 3.3333333, 9.99, 10.0, 20.0], np.float32)
    g = hiera_oracle.gelu_ggml(x)
    assert g[0] == 0 and g[1] == 0 and g[7] == 10.0 and g[8] == 20.0
    # the table stores fp16 values of the tanh form
    assert np.array_equal(g[2:7], g[2:7].astype(np.float16).astype(np.float32))
    exact = 0.5 * x * (1 + np.tanh(np.sqrt(2 / np.pi) * (x + 0.044715 * x ** 3)))
    assert np.abs(g[2:7] - exact[2:7]).max() < 4e-3


def test_bicubic_identity_and_constant():
    src = np.random.default_rng(1).normal(size=(3, 7, 7)).astype(np.float32)
    assert np.allclose(hiera_oracle.bicubic_chw(src, 7, 7), src, atol=1e-6)  # same size: the taps reduce to 1
    c = np.full((2, 7, 7), 0.25, np.float32)
    assert np.allclose(hiera_oracle.bicubic_chw(c, 32, 20), 0.25, atol=1e-6)  # the kernel sums to one
