"""CPU restatement of the tracker's memory encoder (TEST INFRASTRUCTURE ONLY).

Only tests/ import this module, as the checker of the B200 memory encoder.
It restates sam3_encode_memory (sam3.cpp:11510-11615) with numpy: the mask
preprocessing with sam3_bilinear_interpolate (:9617-9643) and the sigmoid
scale/bias (:11521-11524), the mask downsampler (ggml_conv_2d 3x3 s2 p1,
LayerNorm2d eps 1e-6 (sam3_layer_norm_2d, :1053-1064), ggml_gelu), the 1x1
convolutions, the CXBlock fuser (sam3_cxblock_forward, :9066-9108) and the
output projection, plus no_obj_embed_spatial for an occluded object.
Convolutions accumulate in float64; an F16 kernel rounds its input to fp16
(ggml's im2col of an F16 kernel is F16).  Weights: conv kernels as
(type, f32 array in ggml memory order); linear weights as (type, data, K, N)
with type 1 (F16) or a quantised type (the C oracle's exact MUL_MAT).
Maps are token-major [H*W][C] unless noted.
"""
from __future__ import annotations

import numpy as np

import hiera_oracle

F32 = np.float32


def bilinear(src: np.ndarray, dw: int, dh: int, sigmoid=None) -> np.ndarray:
    """sam3_bilinear_interpolate of [sh][sw] to [dh][dw]; sigmoid = (scale, bias) applies
    sigmoid(v) * scale + bias to the result."""
    sh, sw = src.shape
    fy = np.clip((np.arange(dh) + 0.5) * (sh / dh) - 0.5, 0.0, sh - 1)
    fx = np.clip((np.arange(dw) + 0.5) * (sw / dw) - 0.5, 0.0, sw - 1)
    y0 = np.minimum(fy.astype(np.int64), sh - 2)
    x0 = np.minimum(fx.astype(np.int64), sw - 2)
    wy = (fy - y0).astype(F32)[:, None]
    wx = (fx - x0).astype(F32)[None, :]
    m = src.astype(F32)
    a, b = m[y0][:, x0], m[y0][:, x0 + 1]
    c, d = m[y0 + 1][:, x0], m[y0 + 1][:, x0 + 1]
    ux, uy = (F32(1) - wx).astype(F32), (F32(1) - wy).astype(F32)
    top = ((ux * a).astype(F32) + (wx * b).astype(F32)).astype(F32)
    bot = ((ux * c).astype(F32) + (wx * d).astype(F32)).astype(F32)
    v = ((uy * top).astype(F32) + (wy * bot).astype(F32)).astype(F32)
    if sigmoid is not None:
        s = (F32(1) / (F32(1) + np.exp(-v))).astype(F32)
        v = ((s * F32(sigmoid[0])).astype(F32) + F32(sigmoid[1])).astype(F32)
    return v


def conv3x3_s2(x: np.ndarray, w: np.ndarray, b: np.ndarray, f16: bool) -> np.ndarray:
    """ggml_conv_2d(w, x, 2, 2, 1, 1, 1, 1): x [C][H][W] -> [O][H/2][W/2] (+ bias)."""
    if f16:
        x = x.astype(np.float16)
    C, H, W = x.shape
    OH, OW = (H - 1) // 2 + 1, (W - 1) // 2 + 1
    xp = np.zeros((C, H + 2, W + 2), np.float64)
    xp[:, 1:H + 1, 1:W + 1] = x
    acc = np.zeros((w.shape[0], OH, OW), np.float64)
    for ky in range(3):
        for kx in range(3):
            acc += np.einsum("oc,chw->ohw", w[:, :, ky, kx].astype(np.float64),
                             xp[:, ky:ky + 2 * OH:2, kx:kx + 2 * OW:2])
    return (acc.astype(F32) + b.astype(F32)[:, None, None]).astype(F32)


def pointwise(x_tok: np.ndarray, w: np.ndarray, b: np.ndarray, f16: bool) -> np.ndarray:
    """1x1 ggml_conv_2d on a token-major map: [P][C] x w [O][C] -> [P][O] (+ bias)."""
    xin = x_tok.astype(np.float16) if f16 else x_tok
    y = xin.astype(np.float64) @ w.reshape(w.shape[0], -1).astype(np.float64).T
    return (y.astype(F32) + b.astype(F32)).astype(F32)


def depthwise7(x: np.ndarray, H: int, w: np.ndarray, b: np.ndarray) -> np.ndarray:
    """ggml_conv_2d_dw_direct, 7x7, padding 3, on token-major [H*H][C] with w [C][7][7]."""
    C = x.shape[1]
    xp = np.zeros((H + 6, H + 6, C), np.float64)
    xp[3:H + 3, 3:H + 3] = x.reshape(H, H, C)
    acc = np.zeros((H, H, C), np.float64)
    for ky in range(7):
        for kx in range(7):
            acc += xp[ky:ky + H, kx:kx + H] * w[:, ky, kx].astype(np.float64)
    return (acc.astype(F32).reshape(H * H, C) + b.astype(F32)).astype(F32)


def linear_any(w: tuple, x: np.ndarray, b: np.ndarray) -> np.ndarray:
    qtype, data, K, N = w
    if qtype == 1:  # F16 weight: the activations go to fp16, products summed in f32 (float64 here)
        y = x.astype(np.float16).astype(np.float64) @ data.astype(np.float64).T
        return (y.astype(F32) + b.astype(F32)).astype(F32)
    return hiera_oracle.linear(w, x, b)


def encode(hp: dict, t: dict, mask_logits: np.ndarray, pix_feat: np.ndarray, obj_score: float) -> np.ndarray:
    """-> memory features [H*H][mem_dim]."""
    H, img = hp["feat"], hp["img"]
    I = 16 * H
    hi = bilinear(mask_logits, img, img, (hp["sigmoid_scale"], hp["sigmoid_bias"]))
    x = bilinear(hi, I, I)[None]  # [1][I][I]
    ln, gelu = hiera_oracle.layer_norm, hiera_oracle.gelu_ggml
    for ci, ni in ((0, 1), (3, 4), (6, 7), (9, 10)):
        ty, w = t[f"mem_enc.ds.{ci}.weight"]
        y = conv3x3_s2(x, w, t[f"mem_enc.ds.{ci}.bias"], ty == 1)
        C, h, wd = y.shape
        yt = ln(y.reshape(C, -1).T, t[f"mem_enc.ds.{ni}.weight"], t[f"mem_enc.ds.{ni}.bias"], 1e-6)
        x = gelu(yt).T.reshape(C, h, wd)
    ty, w = t["mem_enc.ds.12.weight"]
    ds = pointwise(x.reshape(x.shape[0], -1).T, w, t["mem_enc.ds.12.bias"], ty == 1)
    ty, w = t["mem_enc.pix_feat_proj.weight"]
    fused = (pointwise(pix_feat, w, t["mem_enc.pix_feat_proj.bias"], ty == 1) + ds).astype(F32)
    for i in range(hp["fuser_layers"]):
        p = f"mem_enc.fuser.{i}."
        hdw = depthwise7(fused, H, t[p + "dwconv.weight"][1].reshape(-1, 7, 7), t[p + "dwconv.bias"])
        hn = ln(hdw, t[p + "norm.weight"], t[p + "norm.bias"], 1e-6)
        m = gelu(linear_any(t[p + "pwconv1.weight"], hn, t[p + "pwconv1.bias"]))
        h2 = linear_any(t[p + "pwconv2.weight"], m, t[p + "pwconv2.bias"])
        fused = (fused + (h2 * t[p + "gamma"].astype(F32)).astype(F32)).astype(F32)
    ty, w = t["mem_enc.out_proj.weight"]
    out = pointwise(fused, w, t["mem_enc.out_proj.bias"], ty == 1)
    if obj_score <= 0.0 and "no_obj_embed_spatial" in t:
        out = (out + t["no_obj_embed_spatial"].astype(F32)).astype(F32)
    return out
