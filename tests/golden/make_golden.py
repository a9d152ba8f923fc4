"""Generate the golden quantisation vectors in tests/golden/quants_golden.npz.

The vectors pin the oracle's weight quantisers and dequantisers to the gguf
0.19.0 Python package (gguf/quants.py), which mirrors ggml-quants.c's
reference quantisers bit for bit (its Q8_0 docstring says so) and is the
published algorithm sam3.cpp's examples/quantize.cpp:244 reaches through
ggml_quantize_chunk.  Run in a container where ``import gguf`` works:

    python tests/golden/make_golden.py

Inputs are seeded: N(0, 0.02) weight rows (the random-init distribution of
the benchmark configs) plus hand-made edge rows -- an all-zero block, a
block with a single non-zero, sign-symmetric maxima, exact .5 ties after
scaling, large magnitudes and denormal-range values.
"""
from __future__ import annotations

import os

import numpy as np


def edge_rows() -> np.ndarray:
    rows = []
    z = np.zeros(64, np.float32)
    rows.append(z.copy())                                   # all zero
    r = z.copy(); r[5] = 0.5; rows.append(r)                # single non-zero
    r = z.copy(); r[:32] = np.linspace(-1, 1, 32); r[32:] = -np.linspace(-1, 1, 32); rows.append(r)
    r = z.copy(); r[0] = 127.0; r[1:32] = np.arange(-15, 16) + 0.5; rows.append(r)   # .5 ties at id=1
    r = z.copy(); r[:] = 3.0e4 * np.sin(np.arange(64)); rows.append(r)               # large
    r = z.copy(); r[:] = 1e-6 * np.cos(np.arange(64)); rows.append(r)                # tiny
    r = z.copy(); r[:32] = -2.0; r[32:] = 2.0; rows.append(r)                        # constant blocks
    r = z.copy(); r[7] = -8.0; r[9] = 8.0; rows.append(r)                            # equal |max|, neg first
    return np.stack(rows).astype(np.float32)


def main() -> None:
    from gguf import quants
    from gguf.constants import GGMLQuantizationType as T

    rng = np.random.default_rng(20261201)
    w = rng.normal(0.0, 0.02, size=(24, 256)).astype(np.float32)
    x = rng.normal(0.0, 1.0, size=(8, 256)).astype(np.float32)
    edge = edge_rows()
    out = {"w": w, "x": x, "edge": edge}
    for name, qt in (("q8_0", T.Q8_0), ("q4_0", T.Q4_0), ("q4_1", T.Q4_1)):
        for src_name, src in (("w", w), ("x", x), ("edge", edge)):
            q = quants.quantize(src, qt)
            out[f"{name}_{src_name}_q"] = q
            out[f"{name}_{src_name}_dq"] = quants.dequantize(q, qt)
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "quants_golden.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, sorted(out))


if __name__ == "__main__":
    main()
