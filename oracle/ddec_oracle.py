"""CPU restatement of the SAM3 detector's DETR decoder (TEST INFRASTRUCTURE ONLY).

Only tests/ import this module, as the checker of the B200 DETR decoder.  It
restates sam3_build_ddec_graph (sam3.cpp:8749-8888): the query sine code and
ref_point_head (sam3_build_sine_pos_embed_4d / sam3_build_query_pos,
:8200-8290), the box-relative bias (sam3_compute_box_rpb, :8293-8436), the
post-norm layer (sam3_ddec_layer_forward, :8438-8632), box refinement with
sam3_inverse_sigmoid (:8171-8181), sam3_dot_product_scoring (:8640-8739) and
the presence head -- with numpy and the C oracle's quantised MUL_MAT; the fused
in_proj weights through row views; attention in float64 (or float32 for the
spread estimate).  Maps are token-major [tokens][channels].
"""
from __future__ import annotations

import math

import numpy as np

import fenc_oracle
import hiera_oracle

F32 = np.float32


def sigmoid(x):
    return (F32(1) / (F32(1) + np.exp(-x.astype(F32)))).astype(F32)


def dim_t() -> np.ndarray:
    i = np.arange(64, dtype=F32)
    return (F32(2.0 * math.pi) / np.power(F32(10000.0), F32(2.0) * i / F32(128.0))).astype(F32)


def sine_embed(boxes: np.ndarray) -> np.ndarray:
    """[NQ][4] (cx, cy, w, h) -> [NQ][512]: coordinates in the order cy, cx, w, h, each 64 (sin, cos) pairs."""
    dt = dim_t()
    parts = []
    for c in (1, 0, 2, 3):
        a = (boxes[:, c:c + 1] * dt[None]).astype(F32)
        parts.append(np.stack([np.sin(a), np.cos(a)], axis=-1).reshape(len(boxes), 128))
    return np.concatenate(parts, axis=1).astype(F32)


def rpb_log(d: np.ndarray) -> np.ndarray:
    d8 = (d * F32(8)).astype(F32)
    lv = np.log((np.abs(d8) + F32(1)).astype(F32)).astype(F32)
    inv_ln2 = F32(1) / np.log(F32(2))       # 1.0f / logf(2.0f)
    inv_log2_8 = F32(1) / np.log2(F32(8))   # 1.0f / log2f(8.0f)
    lv = ((lv * inv_ln2).astype(F32) * inv_log2_8).astype(F32)
    return (np.sign(d8) * lv).astype(F32)


def box_rpb(t: dict, boxes: np.ndarray, S: int, heads: int) -> np.ndarray:
    """-> f32 [heads][NQ+1][S*S] (row 0, the presence token, zero)."""
    NQ = len(boxes)
    coord = (np.arange(S, dtype=F32) / F32(S)).astype(F32)
    out = {}
    for axis, name in ((0, "x"), (1, "y")):
        c, e = boxes[:, axis], boxes[:, 2 + axis]
        half = (e * F32(0.5)).astype(F32)
        lo, hi = (c - half).astype(F32), (c + half).astype(F32)
        d = np.stack([(coord[None] - lo[:, None]).astype(F32), (coord[None] - hi[:, None]).astype(F32)], -1)
        d = rpb_log(d).reshape(NQ * S, 2)
        ty, w0 = t[f"ddec.boxRPB_embed_{name}.layers.0.weight"]
        if ty == 1:
            d = d.astype(np.float16).astype(F32)
        h = ((d[:, 0:1] * w0[None, :, 0]).astype(F32) + (d[:, 1:2] * w0[None, :, 1]).astype(F32)).astype(F32)
        h = np.maximum((h + t[f"ddec.boxRPB_embed_{name}.layers.0.bias"]).astype(F32), F32(0))
        out[name] = hiera_oracle.linear(t[f"ddec.boxRPB_embed_{name}.layers.1.weight"], h,
                                        t[f"ddec.boxRPB_embed_{name}.layers.1.bias"]).reshape(NQ, S, heads)
    rx, ry = out["x"], out["y"]
    m = np.zeros((heads, NQ + 1, S, S), F32)
    m[:, 1:] = (ry.transpose(2, 0, 1)[:, :, :, None] + rx.transpose(2, 0, 1)[:, :, None, :]).astype(F32)
    return m.reshape(heads, NQ + 1, S * S)


def mlp(t: dict, pfx: str, x: np.ndarray, n: int) -> np.ndarray:
    for j in range(n):
        x = hiera_oracle.linear(t[f"{pfx}.layers.{j}.weight"], x, t[f"{pfx}.layers.{j}.bias"])
        if j < n - 1:
            x = np.maximum(x, F32(0))
    return x


def run(hp: dict, t: dict, enc, enc_pos, text, bias=None, valid=None, attn_dtype=np.float64) -> dict:
    lin, ln = hiera_oracle.linear, hiera_oracle.layer_norm
    rows, mha = fenc_oracle.rows, fenc_oracle.mha
    D, NQ, S, NH = hp["d_model"], hp["num_queries"], hp["feat"], hp["heads"]
    q = np.concatenate([t["ddec.presence_token.weight"].reshape(1, D), t["ddec.query_embed.weight"]]).astype(F32)
    boxes = sigmoid(t["ddec.reference_points.weight"])
    kin = (enc + enc_pos).astype(F32)
    tmask = fenc_oracle.bias_mask(bias, NQ + 1)
    for i in range(hp["layers"]):
        p = f"ddec.layers.{i}."
        qpos = np.zeros((NQ + 1, D), F32)
        qpos[1:] = mlp(t, "ddec.ref_point_head", sine_embed(boxes), 2)
        rpb = box_rpb(t, boxes, S, NH)
        W, B = t[p + "sa.in_proj_weight"], t[p + "sa.in_proj_bias"]
        qin = (q + qpos).astype(F32)
        a = mha(lin(rows(W, 0, D), qin, B[:D]), lin(rows(W, D, D), qin, B[D:2 * D]), lin(rows(W, 2 * D, D), q, B[2 * D:]),
                NH, None, attn_dtype)
        q = ln((q + lin(t[p + "sa.out_proj.weight"], a, t[p + "sa.out_proj.bias"])).astype(F32),
               t[p + "norm2.weight"], t[p + "norm2.bias"], 1e-5)
        W, B = t[p + "ca_text.in_proj_weight"], t[p + "ca_text.in_proj_bias"]
        a = mha(lin(rows(W, 0, D), (q + qpos).astype(F32), B[:D]), lin(rows(W, D, D), text, B[D:2 * D]),
                lin(rows(W, 2 * D, D), text, B[2 * D:]), NH, tmask, attn_dtype)
        q = ln((q + lin(t[p + "ca_text.out_proj.weight"], a, t[p + "ca_text.out_proj.bias"])).astype(F32),
               t[p + "norm_ca_text.weight"], t[p + "norm_ca_text.bias"], 1e-5)
        W, B = t[p + "ca.in_proj_weight"], t[p + "ca.in_proj_bias"]
        a = mha(lin(rows(W, 0, D), (q + qpos).astype(F32), B[:D]), lin(rows(W, D, D), kin, B[D:2 * D]),
                lin(rows(W, 2 * D, D), enc, B[2 * D:]), NH, rpb, attn_dtype)
        q = ln((q + lin(t[p + "ca.out_proj.weight"], a, t[p + "ca.out_proj.bias"])).astype(F32),
               t[p + "norm1.weight"], t[p + "norm1.bias"], 1e-5)
        h = np.maximum(lin(t[p + "linear1.weight"], q, t[p + "linear1.bias"]), F32(0))
        q = ln((q + lin(t[p + "linear2.weight"], h, t[p + "linear2.bias"])).astype(F32),
               t[p + "norm3.weight"], t[p + "norm3.bias"], 1e-5)
        objn = ln(q[1:], t["ddec.norm.weight"], t["ddec.norm.bias"], 1e-5)
        bd = mlp(t, "ddec.bbox_embed", objn, 3)
        x = np.clip(boxes, F32(1e-3), F32(1.0) - F32(1e-3)).astype(F32)
        inv = (np.log(x) - np.log((F32(1) - x).astype(F32))).astype(F32)
        boxes = sigmoid((inv + bd).astype(F32))
    objn = ln(q[1:], t["ddec.norm.weight"], t["ddec.norm.bias"], 1e-5)
    # scoring
    tm = mlp(t, "scoring.prompt_mlp", text, 2)
    tm = ln((tm + text).astype(F32), t["scoring.prompt_mlp.out_norm.weight"], t["scoring.prompt_mlp.out_norm.bias"], 1e-5)
    if valid is not None:
        tm = (tm * np.asarray(valid, F32)[:, None]).astype(F32)
    pooled = (tm.astype(np.float64).sum(0) / len(text)).astype(F32)[None]
    pp = lin(t["scoring.prompt_proj.weight"], pooled, t["scoring.prompt_proj.bias"])[0]
    hs = lin(t["scoring.hs_proj.weight"], objn, t["scoring.hs_proj.bias"])
    scores = np.clip(((hs.astype(np.float64) @ pp.astype(np.float64)).astype(F32) * F32(1.0 / math.sqrt(D))).astype(F32),
                     F32(-12), F32(12))
    pres = ln(q[:1], t["ddec.presence_token_out_norm.weight"], t["ddec.presence_token_out_norm.bias"], 1e-5)
    presence = float(mlp(t, "ddec.presence_token_head", pres, 3)[0, 0])
    return dict(queries=np.concatenate([q[:1], objn]).astype(F32), boxes=boxes, scores=scores, presence=presence)
