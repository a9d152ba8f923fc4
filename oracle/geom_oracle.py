"""CPU restatement of the SAM3 detector's geometry-encoder transformer (TEST INFRASTRUCTURE ONLY).

Only tests/ import this module, as the checker of the B200 geometry encoder.  It restates the layers
of sam3_build_geom_enc_graph (sam3.cpp:7677-7800) with numpy and the C oracle's quantised MUL_MAT:
pre-LN self-attention without positions, cross-attention to the image (keys from features +
positional code, values from features), ReLU FFN, final encode_norm; fused in_proj weights through
row views; attention in float64 (or float32 for the spread estimate).  Token-major maps.
"""
from __future__ import annotations

import numpy as np

import fenc_oracle
import hiera_oracle

F32 = np.float32


def run(t: dict, layers: int, heads: int, x, img, pe, attn_dtype=np.float64) -> np.ndarray:
    lin, ln = hiera_oracle.linear, hiera_oracle.layer_norm
    rows, mha = fenc_oracle.rows, fenc_oracle.mha
    x = x.astype(F32)
    D = x.shape[1]
    kin = (img + pe).astype(F32)
    for i in range(layers):
        p = f"geom.layers.{i}."
        W, B = t[p + "sa.in_proj_weight"], t[p + "sa.in_proj_bias"]
        xn = ln(x, t[p + "norm1.weight"], t[p + "norm1.bias"], 1e-5)
        a = mha(lin(rows(W, 0, D), xn, B[:D]), lin(rows(W, D, D), xn, B[D:2 * D]), lin(rows(W, 2 * D, D), xn, B[2 * D:]),
                heads, None, attn_dtype)
        x = (x + lin(t[p + "sa.out_proj.weight"], a, t[p + "sa.out_proj.bias"])).astype(F32)
        W, B = t[p + "ca.in_proj_weight"], t[p + "ca.in_proj_bias"]
        xn = ln(x, t[p + "norm2.weight"], t[p + "norm2.bias"], 1e-5)
        a = mha(lin(rows(W, 0, D), xn, B[:D]), lin(rows(W, D, D), kin, B[D:2 * D]), lin(rows(W, 2 * D, D), img, B[2 * D:]),
                heads, None, attn_dtype)
        x = (x + lin(t[p + "ca.out_proj.weight"], a, t[p + "ca.out_proj.bias"])).astype(F32)
        xn = ln(x, t[p + "norm3.weight"], t[p + "norm3.bias"], 1e-5)
        h = np.maximum(lin(t[p + "linear1.weight"], xn, t[p + "linear1.bias"]), F32(0))
        x = (x + lin(t[p + "linear2.weight"], h, t[p + "linear2.bias"])).astype(F32)
    return ln(x, t["geom.encode_norm.weight"], t["geom.encode_norm.bias"], 1e-5)
