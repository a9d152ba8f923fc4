"""CPU checks of the memory-encoder oracle (oracle/mem_enc_oracle.py)."""
import numpy as np


def test_bilinear_same_size_is_identity():
    import mem_enc_oracle
    x = np.random.default_rng(0).normal(size=(17, 23)).astype(np.float32)
    np.testing.assert_array_equal(mem_enc_oracle.bilinear(x, 23, 17), x)


def test_conv3x3_s2_matches_loops():
    import mem_enc_oracle
    rng = np.random.default_rng(1)
    x = rng.normal(size=(3, 9, 8)).astype(np.float32)
    w = rng.normal(size=(5, 3, 3, 3)).astype(np.float32)
    b = rng.normal(size=5).astype(np.float32)
    y = mem_enc_oracle.conv3x3_s2(x, w, b, False)
    xp = np.pad(x.astype(np.float64), ((0, 0), (1, 1), (1, 1)))
    for o in range(5):
        for oy in range(5):
            for ox in range(4):
                ref = (xp[:, 2 * oy:2 * oy + 3, 2 * ox:2 * ox + 3] * w[o]).sum()
                assert abs(y[o, oy, ox] - (np.float32(ref) + b[o])) < 1e-5


def test_depthwise_matches_loops():
    import mem_enc_oracle
    rng = np.random.default_rng(2)
    H, C = 6, 4
    x = rng.normal(size=(H * H, C)).astype(np.float32)
    w = rng.normal(size=(C, 7, 7)).astype(np.float32)
    b = np.zeros(C, np.float32)
    y = mem_enc_oracle.depthwise7(x, H, w, b).reshape(H, H, C)
    xm = x.reshape(H, H, C)
    for c in range(C):
        for py in range(H):
            for px in range(H):
                s = sum(xm[iy, ix, c] * w[c, iy - py + 3, ix - px + 3]
                        for iy in range(max(0, py - 3), min(H, py + 4)) for ix in range(max(0, px - 3), min(H, px + 4)))
                assert abs(y[py, px, c] - s) < 1e-4
