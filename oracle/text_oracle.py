"""CPU restatement of the SAM3 text encoder (TEST INFRASTRUCTURE ONLY).

Only tests/ import this module, as the checker of the B200 text encoder.  It
restates sam3_build_text_encoder_graph (sam3.cpp:4040-4066) and
sam3_text_block_forward (:3957-4032) with numpy plus the C oracle's quantised
MUL_MAT (exact ggml block dots): token-embedding rows + positional embedding,
pre-LN blocks (ggml_norm eps 1e-5; 16-head attention with the causal mask of
sam3_fill_causal_mask, :3943-3950; GELU in erf form), final LayerNorm, resizer.
Maps are token-major [L][width].
"""
from __future__ import annotations

import math

import numpy as np

import hiera_oracle
import oracle

F32 = np.float32


def gelu_erf(x):
    from scipy.special import erf
    x = x.astype(F32)
    return (F32(0.5) * x * (F32(1.0) + erf(x * F32(0.70710678118654752440)).astype(F32))).astype(F32)


def encode(hp: dict, t: dict, ids, attn_dtype=np.float64) -> np.ndarray:
    """-> f32 [ctx_len][out_dim]; ids are padded with 0 to ctx_len."""
    E, L, H = hp["width"], hp["ctx_len"], hp["heads"]
    HD = E // H
    pid = np.zeros(L, np.int64)
    pid[:len(ids)] = ids
    x = (t["text.token_embed.weight"][pid] + t["text.pos_embed"]).astype(F32)
    mask = np.where(np.arange(L)[None, :] <= np.arange(L)[:, None], 0.0, -np.inf).astype(F32)
    lin = hiera_oracle.linear
    ln = hiera_oracle.layer_norm
    for i in range(hp["layers"]):
        p = f"text.blocks.{i}."
        xn = ln(x, t[p + "ln_1.weight"], t[p + "ln_1.bias"], 1e-5)
        qkv = lin(t[p + "attn.in_proj.weight"], xn, t[p + "attn.in_proj.bias"])
        heads = lambda a: a.reshape(1, L, H, HD).transpose(0, 2, 1, 3)
        o = oracle.attention_general(heads(qkv[:, :E]), heads(qkv[:, E:2 * E]), heads(qkv[:, 2 * E:]),
                                     1.0 / math.sqrt(HD), mask, attn_dtype).reshape(L, E)
        x = (x + lin(t[p + "attn.out_proj.weight"], o, t[p + "attn.out_proj.bias"])).astype(F32)
        xn = ln(x, t[p + "ln_2.weight"], t[p + "ln_2.bias"], 1e-5)
        h = gelu_erf(lin(t[p + "mlp.fc1.weight"], xn, t[p + "mlp.fc1.bias"]))
        x = (x + lin(t[p + "mlp.fc2.weight"], h, t[p + "mlp.fc2.bias"])).astype(F32)
    xn = ln(x, t["text.ln_final.weight"], t["text.ln_final.bias"], 1e-5)
    return lin(t["text.resizer.weight"], xn, t["text.resizer.bias"])
