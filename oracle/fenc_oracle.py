"""CPU restatement of the SAM3 detector's fusion encoder (TEST INFRASTRUCTURE ONLY).

Only tests/ import this module, as the checker of the B200 fusion encoder.  It
restates sam3_build_fenc_graph (sam3.cpp:8146-8165) and
sam3_fenc_layer_forward (:8033-8139) with numpy and the C oracle's quantised
MUL_MAT: the fused in_proj weights are used through row views, as the
reference's ggml_view_2d of them; the prompt padding bias is cast to fp16 as
sam3_expand_token_attn_bias does (:7550-7570); attention runs in float64 (or
float32 for the spread estimate).  Maps are token-major [tokens][channels].
"""
from __future__ import annotations

import math

import numpy as np

import hiera_oracle

F32 = np.float32


def rows(w: tuple, r0: int, n: int) -> tuple:
    """Rows [r0, r0 + n) of a (qtype, data [N][row bytes], K, N) weight."""
    qtype, data, K, _ = w
    return (qtype, np.ascontiguousarray(data[r0:r0 + n]), K, n)


def mha(q, k, v, heads: int, mask=None, dtype=np.float64, chunk=1024) -> np.ndarray:
    """Multi-head softmax(q k^T / sqrt(hd) + mask) v over token-major q [NQ][D], k, v [NK][D]; mask
    [NQ][NK] additive, shared by the heads, or [heads][NQ][NK] (an -inf entry removes the key).  Query
    chunks bound the memory."""
    NQ, D = q.shape
    hd = D // heads
    scale = 1.0 / math.sqrt(hd)
    out = np.empty((NQ, D), F32)
    for h in range(heads):
        sl = slice(h * hd, (h + 1) * hd)
        kh, vh = k[:, sl].astype(dtype), v[:, sl].astype(dtype)
        for i in range(0, NQ, chunk):
            s = (q[i:i + chunk, sl].astype(dtype) @ kh.T) * dtype(scale)
            if mask is not None:
                s = s + (mask[h] if mask.ndim == 3 else mask)[i:i + chunk].astype(dtype)
            m = s.max(axis=1, keepdims=True)
            p = np.exp(s - np.where(np.isfinite(m), m, 0))
            den = p.sum(axis=1, keepdims=True)
            out[i:i + chunk, sl] = ((p @ vh) / np.where(den > 0, den, 1)).astype(F32)
    return out


def bias_mask(bias, nq: int) -> np.ndarray | None:
    if bias is None:
        return None
    with np.errstate(over="ignore"):  # -1e9 -> -inf, as the fp16 cast of the reference
        b16 = np.asarray(bias, F32).astype(np.float16).astype(F32)
    return np.broadcast_to(b16, (nq, len(bias)))


def run(t: dict, layers: int, heads: int, img, prompt, pos, bias=None, attn_dtype=np.float64) -> np.ndarray:
    lin, ln = hiera_oracle.linear, hiera_oracle.layer_norm
    x = img.astype(F32)
    N, D = x.shape
    mask = bias_mask(bias, N)
    for i in range(layers):
        p = f"fenc.layers.{i}."
        sw, sb = t[p + "sa.in_proj_weight"], t[p + "sa.in_proj_bias"]
        cw, cb = t[p + "ca.in_proj_weight"], t[p + "ca.in_proj_bias"]
        xn = ln(x, t[p + "norm1.weight"], t[p + "norm1.bias"], 1e-5)
        qin = (xn + pos).astype(F32)
        q = lin(rows(sw, 0, D), qin, sb[:D])
        k = lin(rows(sw, D, D), qin, sb[D:2 * D])
        v = lin(rows(sw, 2 * D, D), xn, sb[2 * D:])
        a = mha(q, k, v, heads, None, attn_dtype)
        x = (x + lin(t[p + "sa.out_proj.weight"], a, t[p + "sa.out_proj.bias"])).astype(F32)
        xn = ln(x, t[p + "norm2.weight"], t[p + "norm2.bias"], 1e-5)
        q = lin(rows(cw, 0, D), xn, cb[:D])
        k = lin(rows(cw, D, D), prompt, cb[D:2 * D])
        v = lin(rows(cw, 2 * D, D), prompt, cb[2 * D:])
        a = mha(q, k, v, heads, mask, attn_dtype)
        x = (x + lin(t[p + "ca.out_proj.weight"], a, t[p + "ca.out_proj.bias"])).astype(F32)
        xn = ln(x, t[p + "norm3.weight"], t[p + "norm3.bias"], 1e-5)
        h = np.maximum(lin(t[p + "linear1.weight"], xn, t[p + "linear1.bias"]), F32(0))
        x = (x + lin(t[p + "linear2.weight"], h, t[p + "linear2.bias"])).astype(F32)
    return x
