"""CPU restatement of the SAM3 detector's segmentation head (TEST INFRASTRUCTURE ONLY).

Only tests/ import this module, as the checker of the B200 segmentation head.
It restates sam3_build_seg_head_graph (sam3.cpp:8975-9058) and
sam3_pixel_decoder (:8899-8960) with numpy: the prompt cross-attention
(sam3_multihead_attn_fused, :7502-7548, with the fused in_proj through row
views and the padding bias cast to fp16), nearest 2x upsampling, the 3x3
convolutions in float64 (input rounded to fp16 for an F16 kernel, as ggml's
im2col), GroupNorm(8) as ggml_group_norm (double sums), ReLU, the 1x1 instance
head and the mask-embedding MLP, and the mask product.  Maps are token-major.
"""
from __future__ import annotations

import numpy as np

import fenc_oracle
import hiera_oracle

F32 = np.float32


def up2_add(fpn: np.ndarray, prev: np.ndarray, S: int) -> np.ndarray:
    """fpn [S*S][C] + nearest-2x(prev [(S/2)^2][C])."""
    C = fpn.shape[1]
    p = prev.reshape(S // 2, S // 2, C).repeat(2, axis=0).repeat(2, axis=1).reshape(S * S, C)
    return (fpn + p).astype(F32)


def conv3(x: np.ndarray, S: int, w: np.ndarray, b: np.ndarray, f16: bool) -> np.ndarray:
    """3x3, stride 1, padding 1 on token-major [S*S][C]; w [O][C][3][3] -> [S*S][O]."""
    C = x.shape[1]
    xin = x.astype(np.float16) if f16 else x
    xp = np.zeros((S + 2, S + 2, C), np.float64)
    xp[1:S + 1, 1:S + 1] = xin.reshape(S, S, C)
    acc = np.zeros((S * S, w.shape[0]), np.float64)
    for ky in range(3):
        for kx in range(3):
            acc += xp[ky:ky + S, kx:kx + S].reshape(S * S, C) @ w[:, :, ky, kx].astype(np.float64).T
    return (acc.astype(F32) + b.astype(F32)).astype(F32)


def group_norm_relu(x: np.ndarray, groups: int, w, b, eps: float = 1e-5) -> np.ndarray:
    P, C = x.shape
    cg = C // groups
    out = np.empty_like(x)
    for g in range(groups):
        blk = x[:, g * cg:(g + 1) * cg]
        mean = F32(blk.astype(np.float64).sum() / blk.size)
        d = (blk - mean).astype(F32)
        var = F32((d * d).astype(F32).astype(np.float64).sum() / blk.size)
        scale = F32(1) / np.sqrt(F32(var + F32(eps)))
        out[:, g * cg:(g + 1) * cg] = (d * scale).astype(F32)
    y = ((out * w.astype(F32)).astype(F32) + b.astype(F32)).astype(F32)
    return np.maximum(y, F32(0))


def run(t: dict, S: int, enc, fpn0, fpn1, queries, text, bias=None, attn_dtype=np.float64) -> np.ndarray:
    lin, ln = hiera_oracle.linear, hiera_oracle.layer_norm
    rows, mha = fenc_oracle.rows, fenc_oracle.mha
    D = enc.shape[1]
    W, B = t["seg.cross_attend_prompt.in_proj_weight"], t["seg.cross_attend_prompt.in_proj_bias"]
    xn = ln(enc, t["seg.cross_attn_norm.weight"], t["seg.cross_attn_norm.bias"], 1e-5)
    a = mha(lin(rows(W, 0, D), xn, B[:D]), lin(rows(W, D, D), text, B[D:2 * D]), lin(rows(W, 2 * D, D), text, B[2 * D:]),
            8, fenc_oracle.bias_mask(bias, len(enc)), attn_dtype)
    enc2 = (enc + lin(t["seg.cross_attend_prompt.out_proj.weight"], a, t["seg.cross_attend_prompt.out_proj.bias"])).astype(F32)
    p = enc2
    for i, (fpn, side) in enumerate(((fpn1, 2 * S), (fpn0, 4 * S))):
        ty, w = t[f"seg.pixel_decoder.conv_layers.{i}.weight"]
        m = conv3(up2_add(fpn, p, side), side, w, t[f"seg.pixel_decoder.conv_layers.{i}.bias"], ty == 1)
        p = group_norm_relu(m, 8, t[f"seg.pixel_decoder.norms.{i}.weight"], t[f"seg.pixel_decoder.norms.{i}.bias"])
    ty, w = t["seg.instance_seg_head.weight"]
    pin = p.astype(np.float16) if ty == 1 else p
    emb = ((pin.astype(np.float64) @ w.reshape(D, D).astype(np.float64).T).astype(F32) +
           t["seg.instance_seg_head.bias"]).astype(F32)
    me = queries
    for j in range(3):
        me = lin(t[f"seg.mask_predictor.mask_embed.layers.{j}.weight"], me, t[f"seg.mask_predictor.mask_embed.layers.{j}.bias"])
        if j < 2:
            me = np.maximum(me, F32(0))
    return (me.astype(np.float64) @ emb.astype(np.float64).T).astype(F32)
