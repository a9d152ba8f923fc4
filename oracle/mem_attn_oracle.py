"""CPU restatement of the tracker's memory attention (TEST INFRASTRUCTURE ONLY).

Only tests/ import this module, as the checker of the B200 memory attention.
It restates sam3_build_mem_attn_graph (sam3.cpp:9228-9341) with numpy and the
C oracle's quantised MUL_MAT (exact ggml block dots): input x = curr + 0.1 *
src_pos; per layer a pre-LN single-head self-attention with RoPE
(sam3_apply_rope, :3671-3710) on q and k, a cross-attention whose keys come
from prompt + prompt_pos and values from prompt (RoPE on q and on the first
M_total - n_obj_ptr_tokens keys), a ReLU feed-forward; final LayerNorm.
Attention runs in float64 (or float32 for the spread estimate).  Maps are
token-major [tokens][channels]; RoPE tables [tokens][D/2][2] (cos, sin).
"""
from __future__ import annotations

import math

import numpy as np

import hiera_oracle

F32 = np.float32


def axial_cis(dim: int, end_x: int, end_y: int, theta: float = 10000.0) -> np.ndarray:
    """sam3_compute_axial_cis (sam3.cpp:3559-3590) in f32: [N][dim/2][2] with x then y frequencies."""
    q = dim // 4
    freqs = (F32(1.0) / np.power(F32(theta), (np.arange(q, dtype=F32) * 4) / F32(dim))).astype(F32)
    idx = np.arange(end_x * end_y)
    tx = (idx % end_x).astype(F32)[:, None] * freqs[None]
    ty = (idx // end_x).astype(F32)[:, None] * freqs[None]
    ang = np.concatenate([tx, ty], axis=1).astype(F32)
    return np.stack([np.cos(ang), np.sin(ang)], axis=-1).astype(F32)


def rope(x: np.ndarray, cs: np.ndarray) -> np.ndarray:
    """(x[2j] + i x[2j+1]) (cos + i sin) with every product rounded to f32 before the sum."""
    xr, xi = x[:, 0::2].astype(F32), x[:, 1::2].astype(F32)
    c, s = cs[..., 0].astype(F32), cs[..., 1].astype(F32)
    out = np.empty_like(x, dtype=F32)
    out[:, 0::2] = (xr * c).astype(F32) - (xi * s).astype(F32)
    out[:, 1::2] = (xr * s).astype(F32) + (xi * c).astype(F32)
    return out


def attend(q, k, v, scale, dtype=np.float64, chunk=512) -> np.ndarray:
    """Single-head softmax(q k^T scale) v, in query chunks (matmul) to bound memory."""
    kd, vd = k.astype(dtype), v.astype(dtype)
    out = np.empty((q.shape[0], v.shape[1]), F32)
    for i in range(0, q.shape[0], chunk):
        s = (q[i:i + chunk].astype(dtype) @ kd.T) * dtype(scale)
        p = np.exp(s - s.max(axis=1, keepdims=True))
        out[i:i + chunk] = ((p @ vd) / p.sum(axis=1, keepdims=True)).astype(F32)
    return out


def run(t: dict, layers: int, curr, src_pos, prompt, prompt_pos, rope_q, rope_k, n_ptr: int,
        attn_dtype=np.float64) -> np.ndarray:
    lin, ln = hiera_oracle.linear, hiera_oracle.layer_norm
    D = curr.shape[1]
    M = prompt.shape[0]
    scale = 1.0 / math.sqrt(D)
    x = (curr.astype(F32) + (src_pos.astype(F32) * F32(0.1)).astype(F32)).astype(F32)
    kvpos = (prompt + prompt_pos).astype(F32)
    for i in range(layers):
        p = f"mem_attn.layers.{i}."
        P = lambda n, a: lin(t[p + n + ".weight"], a, t[p + n + ".bias"])
        xn = ln(x, t[p + "norm1.weight"], t[p + "norm1.bias"], 1e-5)
        q, k, v = rope(P("sa.q_proj", xn), rope_q), rope(P("sa.k_proj", xn), rope_q), P("sa.v_proj", xn)
        x = (x + P("sa.out_proj", attend(q, k, v, scale, attn_dtype))).astype(F32)
        xn = ln(x, t[p + "norm2.weight"], t[p + "norm2.bias"], 1e-5)
        q = rope(P("ca.q_proj", xn), rope_q)
        k, v = P("ca.k_proj", kvpos), P("ca.v_proj", prompt)
        ms = M - n_ptr
        if ms > 0 and rope_k is not None:
            k = np.concatenate([rope(k[:ms], rope_k), k[ms:]]).astype(F32)
        x = (x + P("ca.out_proj", attend(q, k, v, scale, attn_dtype))).astype(F32)
        xn = ln(x, t[p + "norm3.weight"], t[p + "norm3.bias"], 1e-5)
        h = np.maximum(P("linear1", xn), F32(0))
        x = (x + P("linear2", h)).astype(F32)
    return ln(x, t["mem_attn.norm.weight"], t["mem_attn.norm.bias"], 1e-5)
