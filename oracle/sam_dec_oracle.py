"""CPU restatement of the SAM prompt encoder + mask decoder (TEST INFRASTRUCTURE ONLY).

Only tests/ import this module, as the checker of the B200 decoder.  It
restates sam3_segment_pvs (sam3.cpp:10765-11115) with numpy and the C
oracle's quantised MUL_MAT (oracle.mul_mat, exact ggml block dots):

  prompt tokens       sam3_collect_pvs_prompt_tokens       sam3.cpp:10365-10398
  positional enc.     sam3_pe_encode_coord / pe cache      sam3.cpp:10273-10363
  attention           sam3_sam_attention (8 heads)         sam3.cpp:10168-10271
  two-way block       sam3_twoway_block_forward            sam3.cpp:10442-10509
  decoder graph       sam3_build_sam_dec_graph             sam3.cpp:10548-10763
  mask resize         sam3_bilinear_interpolate            sam3.cpp:9617-9643

ggml semantics restated: ggml_norm (double sums; eps 1e-5 for the token and
key LayerNorms, 1e-6 for LayerNorm2d), ConvTranspose through an F16 kernel
with the input rounded to F16 (ggml_cast, sam3.cpp:1087), 1x1 convolutions
with F32 kernels, GELU in erf form, attention in float64.
Maps are token-major [H][W][C] unless noted.
"""
from __future__ import annotations

import math

import numpy as np

import hiera_oracle
import oracle

F32 = np.float32


def pe_encode(gauss: np.ndarray, xn: float, yn: float) -> np.ndarray:
    """Random Fourier encoding of a normalised point: [sin(2 pi c G); cos(2 pi c G)], c in [-1, 1]."""
    g = gauss.reshape(2, -1).astype(F32)
    c = np.array([2.0 * xn - 1.0, 2.0 * yn - 1.0], F32)
    dot = (c[0] * g[0] + c[1] * g[1]).astype(F32) * F32(2.0 * math.pi)
    return np.concatenate([np.sin(dot), np.cos(dot)]).astype(F32)


def dense_pe(gauss: np.ndarray, H: int) -> np.ndarray:
    return np.stack([np.stack([pe_encode(gauss, (c + 0.5) / H, (r + 0.5) / H) for c in range(H)]) for r in range(H)])


def sparse_tokens(t: dict, coords, labels, orig_w: int, orig_h: int, img: int) -> np.ndarray:
    out = []
    for (x, y), lab in zip(np.asarray(coords, F32).reshape(-1, 2), labels):
        px = F32(x) / F32(orig_w) * F32(img) + F32(0.5)
        py = F32(y) / F32(orig_h) * F32(img) + F32(0.5)
        out.append(pe_encode(t["sam_pe.pe_gaussian"], px / F32(img), py / F32(img)) +
                   t[f"sam_pe.point_embeddings.{lab}.weight"])
    out.append(t["sam_pe.not_a_point_embed.weight"])  # padding token
    return np.stack(out).astype(F32)


def linear(w, x, b):
    return hiera_oracle.linear(w, x, b)


def sam_attention(t: dict, pfx: str, q, k, v, dtype=np.float64) -> np.ndarray:
    Q, K, V = (linear(t[pfx + f".{n}_proj.weight"], a, t[pfx + f".{n}_proj.bias"]) for n, a in (("q", q), ("k", k), ("v", v)))
    ID = Q.shape[-1]
    heads = 8
    split = lambda a: a.reshape(1, a.shape[0], heads, ID // heads).transpose(0, 2, 1, 3)
    o = oracle.attention_general(split(Q), split(K), split(V), 1.0 / math.sqrt(ID // heads), dtype=dtype)
    return linear(t[pfx + ".out_proj.weight"], o.reshape(Q.shape[0], ID), t[pfx + ".out_proj.bias"])


def ln(x, w, b, eps=1e-5):
    return hiera_oracle.layer_norm(x, w, b, eps)


def gelu_erf(x):
    from scipy.special import erf
    x = x.astype(F32)
    return (F32(0.5) * x * (F32(1.0) + erf(x * F32(0.70710678118654752440)).astype(F32))).astype(F32)


def decode(hp: dict, t: dict, img_feats, feat_s0, feat_s1, coords, labels, orig_w, orig_h, img, tracking=False,
           all_tokens=False, attn_dtype=np.float64):
    """-> (mask logits [nmask][4H][4H], iou [nmask], obj logit, sam token [256]; with all_tokens the
    output tokens of every mask [nmask][256] instead).  tracking: the decode of a propagated video frame
    (sam3_propagate_single, sam3.cpp:11312-11347) -- no prompt but the padding token, and the
    memory-conditioned features go in without no_mem_embed (the PVS decode adds it, sam3.cpp:10926).
    attn_dtype: the attention arithmetic (float64; float32 is ggml-cpu's flash_attn_ext arithmetic for
    F32 q, k, v)."""
    D, H = 256, hp["feat_size"]
    nmask = hp["n_multimask"] + 1
    special = ([t["sam_dec.obj_score_token.weight"]] if hp["pred_obj_scores"] else []) + \
        [t["sam_dec.iou_token.weight"]] + list(t["sam_dec.mask_tokens.weight"].reshape(nmask, D))
    sparse = sparse_tokens(t, [] if tracking else coords, [] if tracking else labels, orig_w, orig_h, img)
    tok = np.concatenate([np.stack(special), sparse]).astype(F32)
    qpe = tok.copy()
    feats = img_feats.reshape(H * H, D) if tracking else (img_feats.reshape(H * H, D) + t["no_mem_embed"]).astype(F32)
    keys = (feats + t["sam_pe.no_mask_embed.weight"]).astype(F32)
    kpe = dense_pe(t["sam_pe.pe_gaussian"], H).reshape(H * H, D)
    for i in range(hp["depth"]):
        p = f"sam_dec.twoway.{i}."
        if i == 0:
            tok = ln(sam_attention(t, p + "sa", tok, tok, tok, attn_dtype), t[p + "norm1.weight"], t[p + "norm1.bias"])
        else:
            q = (tok + qpe).astype(F32)
            tok = ln((tok + sam_attention(t, p + "sa", q, q, tok, attn_dtype)).astype(F32), t[p + "norm1.weight"], t[p + "norm1.bias"])
        q, k = (tok + qpe).astype(F32), (keys + kpe).astype(F32)
        tok = ln((tok + sam_attention(t, p + "cross_attn_token_to_image", q, k, keys, attn_dtype)).astype(F32),
                 t[p + "norm2.weight"], t[p + "norm2.bias"])
        h = np.maximum(linear(t[p + "mlp.lin1.weight"], tok, t[p + "mlp.lin1.bias"]), F32(0))
        tok = ln((tok + linear(t[p + "mlp.lin2.weight"], h, t[p + "mlp.lin2.bias"])).astype(F32),
                 t[p + "norm3.weight"], t[p + "norm3.bias"])
        q, k = (tok + qpe).astype(F32), (keys + kpe).astype(F32)
        keys = ln((keys + sam_attention(t, p + "cross_attn_image_to_token", k, q, tok, attn_dtype)).astype(F32),
                  t[p + "norm4.weight"], t[p + "norm4.bias"])
    q, k = (tok + qpe).astype(F32), (keys + kpe).astype(F32)
    tok = ln((tok + sam_attention(t, "sam_dec.final_attn", q, k, keys, attn_dtype)).astype(F32),
             t["sam_dec.final_norm.weight"], t["sam_dec.final_norm.bias"])
    # upscaling (channel-major [C][h][w])
    src = keys.reshape(H, H, D).transpose(2, 0, 1)
    up1 = oracle.conv_transpose_2d(t["sam_dec.upscale.0.weight"].astype(np.float16), src, 2) + \
        t["sam_dec.upscale.0.bias"][:, None, None]
    f1 = feat_s1.reshape(2 * H, 2 * H, D).transpose(2, 0, 1).astype(np.float64)
    hs1 = np.einsum("oc,chw->ohw", t["sam_dec.conv_s1.weight"].reshape(64, D).astype(np.float64), f1)
    hs1 = (hs1.astype(F32) + t["sam_dec.conv_s1.bias"][:, None, None]).astype(F32)
    up1 = (up1.astype(F32) + hs1).astype(F32)
    up1 = ln(up1.transpose(1, 2, 0), t["sam_dec.upscale.1.weight"], t["sam_dec.upscale.1.bias"], 1e-6).transpose(2, 0, 1)
    up1 = gelu_erf(up1)
    up2 = oracle.conv_transpose_2d(t["sam_dec.upscale.3.weight"].astype(np.float16), up1, 2) + \
        t["sam_dec.upscale.3.bias"][:, None, None]
    f0 = feat_s0.reshape(4 * H, 4 * H, D).transpose(2, 0, 1).astype(np.float64)
    hs0 = np.einsum("oc,chw->ohw", t["sam_dec.conv_s0.weight"].reshape(32, D).astype(np.float64), f0)
    hs0 = (hs0.astype(F32) + t["sam_dec.conv_s0.bias"][:, None, None]).astype(F32)
    up2 = gelu_erf((up2.astype(F32) + hs0).astype(F32))
    s0 = 1 if hp["pred_obj_scores"] else 0

    def mlp3(pfx, x, sigmoid=False):
        for j in range(3):
            x = linear(t[f"{pfx}.layers.{j}.weight"], x, t[f"{pfx}.layers.{j}.bias"])
            if j < 2:
                x = np.maximum(x, F32(0))
        return (1.0 / (1.0 + np.exp(-x.astype(np.float64)))).astype(F32) if sigmoid else x

    hyp = np.stack([mlp3(f"sam_dec.hyper.{m}", tok[s0 + 1 + m][None])[0] for m in range(nmask)])
    masks = np.einsum("mc,chw->mhw", hyp.astype(np.float64), up2.astype(np.float64)).astype(F32)
    iou = mlp3("sam_dec.iou_prediction_head", tok[s0][None], sigmoid=True)[0]
    obj = float(mlp3("sam_dec.pred_obj_score_head", tok[0][None])[0][0]) if hp["pred_obj_scores"] else 10.0
    return masks, iou, obj, (tok[s0 + 1:s0 + 1 + nmask].copy() if all_tokens else tok[s0 + 1])


def resize_threshold(mask: np.ndarray, dw: int, dh: int) -> np.ndarray:
    """sam3_bilinear_interpolate (double coordinates, clamped) + logit > 0 -> uint8 255 / 0."""
    return np.where(resize_logits(mask, dw, dh) > 0, 255, 0).astype(np.uint8)


def resize_logits(mask: np.ndarray, dw: int, dh: int) -> np.ndarray:
    """The logits resize_threshold thresholds: sam3_bilinear_interpolate to dh x dw, f32."""
    sh, sw = mask.shape
    fy = np.clip((np.arange(dh) + 0.5) * (sh / dh) - 0.5, 0.0, sh - 1)
    fx = np.clip((np.arange(dw) + 0.5) * (sw / dw) - 0.5, 0.0, sw - 1)
    y0 = np.minimum(fy.astype(np.int64), sh - 2)
    x0 = np.minimum(fx.astype(np.int64), sw - 2)
    wy = (fy - y0).astype(F32)[:, None]
    wx = (fx - x0).astype(F32)[None, :]
    m = mask.astype(F32)
    a, b = m[y0][:, x0], m[y0][:, x0 + 1]
    c, d = m[y0 + 1][:, x0], m[y0 + 1][:, x0 + 1]
    return (1 - wy) * ((1 - wx) * a + wx * b) + wy * ((1 - wx) * c + wx * d)


def mask_iou(a: np.ndarray, b: np.ndarray) -> float:
    a, b = a > 0, b > 0
    u = np.logical_or(a, b).sum()
    return 1.0 if u == 0 else float(np.logical_and(a, b).sum() / u)
