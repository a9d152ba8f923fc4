"""CPU restatement of the SAM2 Hiera image encoder (TEST INFRASTRUCTURE ONLY).

Only tests/ import this module, as the checker of the B200 Hiera runner.  It
restates, in numpy plus the C oracle's quantised MUL_MAT (oracle.mul_mat,
exact ggml block-dot semantics), what the reference's graph computes:

  block metadata    sam2_precompute_hiera_metadata   sam3.cpp:1680-1740
  block forward     sam2_hiera_block_forward         sam3.cpp:4299-4461
  window partition  sam2_window_partition            sam3.cpp:4194-4232
  unpartition       sam2_window_unpartition          sam3.cpp:4243-4281
  2x2 max pool      sam2_maxpool_2d                  sam3.cpp:4287-4296
  trunk             sam2_build_hiera_graph           sam3.cpp:4467-4525
  positional emb.   sam2_compute_pos_embed + bicubic sam3.cpp:4076-4160
  FPN neck          sam2_build_fpn_neck_graph        sam3.cpp:4531-4583

ggml semantics restated: ggml_norm (double sums, f32 result), ggml_gelu on
the CPU backend (tanh form evaluated at fp16(x) and stored through an fp16
table, 0 below -10 and identity above 10), flash attention in float64 here
(the B200 path accumulates in fp32; both are compared within the 1e-2 bound).
Maps are token-major [H][W][C] (ggml [C, W, H, 1]).
"""
from __future__ import annotations

import math

import numpy as np

import oracle

F32 = np.float32


def metadata(hp: dict) -> tuple[list[dict], list[int]]:
    """Per-block dim_in, dim_out, heads, window (0 = global), q_stride, stage; and stage ends."""
    ends, cum = [], 0
    for s in hp["stages"]:
        cum += s
        ends.append(cum - 1)
    qpool = [ends[s] + 1 for s in range(3)][: hp["q_pool"]]
    blocks, cur, embed, nh = [], 0, hp["embed"], hp["heads"]
    for i in range(cum):
        ws = 0 if i in hp["global_idx"] else hp["window_spec"][cur]  # window lags a block
        dout = embed
        if i > 0 and i - 1 == ends[cur]:
            dout, nh, cur = embed * 2, nh * 2, cur + 1
        blocks.append(dict(dim_in=embed, dim_out=dout, heads=nh, ws=ws, q_stride=i in qpool, stage=cur))
        embed = dout
    return blocks, ends


def layer_norm(x: np.ndarray, w: np.ndarray, b: np.ndarray, eps: float) -> np.ndarray:
    """ggml_norm (mean and variance from double sums) * w + b, in f32."""
    x = x.astype(F32)
    n = x.shape[-1]
    mean = (x.astype(np.float64).sum(-1, keepdims=True) / n).astype(F32)
    d = (x - mean).astype(F32)
    var = ((d * d).astype(np.float64).sum(-1, keepdims=True) / n).astype(F32)
    scale = (F32(1.0) / np.sqrt((var + F32(eps)).astype(F32))).astype(F32)
    return ((d * scale).astype(F32) * w.astype(F32) + b.astype(F32)).astype(F32)


def gelu_ggml(x: np.ndarray) -> np.ndarray:
    """ggml_gelu on the CPU backend (GGML_GELU_FP16): table lookup at fp16(x)."""
    x = x.astype(F32)
    h = x.astype(np.float16).astype(F32)
    inner = F32(0.79788456080286535587989211986876) * h * (F32(1.0) + F32(0.044715) * h * h)
    g = (F32(0.5) * h * (F32(1.0) + np.tanh(inner.astype(F32)))).astype(np.float16).astype(F32)
    return np.where(x <= -10.0, F32(0.0), np.where(x >= 10.0, x, g)).astype(F32)


def linear(w: tuple, x: np.ndarray, bias: np.ndarray) -> np.ndarray:
    """ggml_mul_mat(w, x) + bias with w = (qtype, blocks, K, N): x [..., K] -> [..., N]."""
    qtype, wq, K, N = w
    shp = x.shape[:-1]
    y = oracle.mul_mat(qtype, wq, K, N, x.reshape(-1, K).astype(F32))
    return (y + bias.astype(F32)).astype(F32).reshape(*shp, N)


def maxpool2(x: np.ndarray) -> np.ndarray:
    """2x2 stride-2 max pool of [H][W][C] (floor)."""
    H, W = x.shape[0] // 2 * 2, x.shape[1] // 2 * 2
    x = x[:H, :W]
    return np.maximum(np.maximum(x[0::2, 0::2], x[0::2, 1::2]), np.maximum(x[1::2, 0::2], x[1::2, 1::2]))


def window_partition(x: np.ndarray, ws: int) -> tuple[np.ndarray, int, int]:
    """[H][W][C] -> [nW][ws*ws][C]; zero padding; window index wy + nWh * wx, token lx + ws * ly."""
    H, W, C = x.shape
    Hp, Wp = -(-H // ws) * ws, -(-W // ws) * ws
    xp = np.zeros((Hp, Wp, C), x.dtype)
    xp[:H, :W] = x
    nWh, nWw = Hp // ws, Wp // ws
    # [wy, ly, wx, lx, C] -> [wx, wy, ly, lx, C]
    t = xp.reshape(nWh, ws, nWw, ws, C).transpose(2, 0, 1, 3, 4)
    return t.reshape(nWw * nWh, ws * ws, C), Hp, Wp


def window_unpartition(y: np.ndarray, ws: int, Hp: int, Wp: int, H: int, W: int) -> np.ndarray:
    C = y.shape[-1]
    nWh, nWw = Hp // ws, Wp // ws
    t = y.reshape(nWw, nWh, ws, ws, C).transpose(1, 2, 0, 3, 4).reshape(Hp, Wp, C)
    return t[:H, :W]


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, heads: int, dtype=np.float64) -> np.ndarray:
    """softmax(q k^T / sqrt(hd)) v per window and head: q [B][Nq][C], k, v [B][N][C] -> [B][Nq][C].
    dtype: the arithmetic (float64 by default; float32 gives a second, equally valid evaluation;
    float16 rounds the operands the tensor-core attention multiplies -- q, k, v and the unnormalised
    probabilities -- to fp16 and sums in float64, the rounding of the GPU kernel's operands)."""
    B, Nq, C = q.shape
    hd = C // heads
    f16 = dtype == np.float16
    wd = np.float64 if f16 else dtype

    def heads_of(a, n):
        a = a.reshape(B, n, heads, hd).transpose(0, 2, 1, 3)
        return a.astype(np.float16).astype(wd) if f16 else a.astype(wd)

    qh, kh, vh = heads_of(q, Nq), heads_of(k, k.shape[1]), heads_of(v, v.shape[1])
    s = qh @ kh.transpose(0, 1, 3, 2) * wd(1.0 / math.sqrt(hd))
    s = np.exp(s - s.max(-1, keepdims=True))
    if f16:
        s = s.astype(np.float16).astype(wd)
    o = (s @ vh) / s.sum(-1, keepdims=True)
    return o.transpose(0, 2, 1, 3).reshape(B, Nq, C).astype(F32)


def block(meta: dict, wts: dict, x: np.ndarray, attn_dtype=np.float64) -> np.ndarray:
    """One Hiera block: x [H][W][dim_in] -> [H'][W'][dim_out]."""
    H, W, _ = x.shape
    Co, nh, ws, qs = meta["dim_out"], meta["heads"], meta["ws"], meta["q_stride"]
    normed = layer_norm(x, wts["norm1.weight"], wts["norm1.bias"], 1e-6)
    if meta["dim_in"] != Co:
        sc = linear(wts["proj.weight"], normed, wts["proj.bias"])
        if qs:
            sc = maxpool2(sc)
    elif qs:
        sc = maxpool2(x)
    else:
        sc = x
    if ws > 0:
        win, Hp, Wp = window_partition(normed, ws)
        wh = ww = ws
    else:
        win, Hp, Wp, wh, ww = normed.reshape(1, H * W, -1), H, W, H, W
    qkv = linear(wts["attn.qkv.weight"], win, wts["attn.qkv.bias"])
    q, k, v = qkv[..., :Co], qkv[..., Co:2 * Co], qkv[..., 2 * Co:]
    if qs:
        Bw = q.shape[0]
        q = np.stack([maxpool2(q[b].reshape(wh, ww, Co)) for b in range(Bw)])
        ph, pw = wh // 2, ww // 2
        q = q.reshape(Bw, ph * pw, Co)
    o = attention(q, k, v, nh, attn_dtype)
    o = linear(wts["attn.proj.weight"], o, wts["attn.proj.bias"])
    Ho, Wo = (H // 2, W // 2) if qs else (H, W)
    if ws > 0:
        wso = ws // 2 if qs else ws
        if qs:
            Hpo, Wpo = Ho + (wso - Ho % wso) % wso, Wo + (wso - Wo % wso) % wso
        else:
            Hpo, Wpo = Hp, Wp
        o = window_unpartition(o, wso, Hpo, Wpo, Ho, Wo)
    else:
        o = o.reshape(Ho, Wo, Co)
    res = (sc + o).astype(F32)
    n2 = layer_norm(res, wts["norm2.weight"], wts["norm2.bias"], 1e-6)
    h1 = gelu_ggml(linear(wts["mlp.fc1.weight"], n2, wts["mlp.fc1.bias"]))
    return (res + linear(wts["mlp.fc2.weight"], h1, wts["mlp.fc2.bias"])).astype(F32)


def bicubic_chw(src: np.ndarray, ho: int, wo: int) -> np.ndarray:
    """sam2_bicubic_interpolate_cpu (Keys a = -0.75, half-pixel centres, clamped taps), in f32."""
    C, hi, wi = src.shape

    def cubic(t):
        t = np.abs(t).astype(F32)
        return np.where(t < 1, (F32(1.25) * t - F32(2.25)) * t * t + F32(1.0),
                        np.where(t < 2, ((F32(-0.75) * t + F32(3.75)) * t - F32(6.0)) * t + F32(3.0), F32(0.0)))

    def taps(n_out, n_in):
        f = ((np.arange(n_out, dtype=F32) + F32(0.5)) * F32(n_in) / F32(n_out) - F32(0.5)).astype(F32)
        i0 = np.floor(f).astype(np.int64)
        d = (f - i0).astype(F32)
        idx = np.stack([np.clip(i0 + j, 0, n_in - 1) for j in (-1, 0, 1, 2)], 1)
        wts = np.stack([cubic(d - F32(j)) for j in (-1, 0, 1, 2)], 1)
        return idx, wts

    iy, wy = taps(ho, hi)
    ix, wx = taps(wo, wi)
    out = np.zeros((C, ho, wo), F32)
    for a in range(4):
        for b in range(4):
            out += (wy[:, a][None, :, None] * wx[:, b][None, None, :]).astype(F32) * src[:, iy[:, a]][:, :, ix[:, b]]
    return out


def pos_embed(bkg: np.ndarray, win: np.ndarray, S: int) -> np.ndarray:
    """bicubic(bkg [E][bh][bw] -> S x S) + tile(win [E][ws][ws]) -> token-major [S][S][E]."""
    ws = win.shape[1]
    pe = bicubic_chw(bkg.astype(F32), S, S) + np.tile(win.astype(F32), (1, S // ws + 1, S // ws + 1))[:, :S, :S]
    return pe.transpose(1, 2, 0).astype(F32)


def prefix(img_chw: np.ndarray, patch_w: np.ndarray, patch_b: np.ndarray, pe: np.ndarray) -> np.ndarray:
    """Conv2d(3 -> E, k 7, s 4, p 3) + bias + positional embedding -> [S][S][E]."""
    conv = oracle.conv_2d(patch_w.astype(F32), img_chw, 4, 4, 3, 3, f16=False)  # F32 kernel in the weight file
    return (conv + patch_b.astype(F32)[:, None, None]).transpose(1, 2, 0).astype(F32) + pe


def fpn(stage_outs: list, convs: list, top_down: list, scalp: int) -> list:
    """Laterals convs[3 - i] on stage i (1x1 conv + bias), top-down nearest-2x fusion, scalp."""
    lat = []
    for i, x in enumerate(stage_outs):
        w, b = convs[3 - i]  # w [D][C] f32
        lat.append((x.astype(np.float64) @ w.astype(np.float64).T + b).astype(F32))  # F32 1x1 kernel
    out, prev = [None] * 4, None
    for i in (3, 2, 1, 0):
        td = i in top_down
        if td and prev is not None:
            up = np.repeat(np.repeat(prev, 2, axis=0), 2, axis=1)
            out[i] = (lat[i] + up).astype(F32)
            prev = out[i]
        else:
            out[i] = lat[i]
            if td or prev is None:
                prev = out[i]
    return out[: 4 - scalp]


def encode(hp: dict, tensors: dict, img_chw: np.ndarray, attn_dtype=np.float64) -> tuple[list, list]:
    """Whole encoder: (stage outputs, FPN levels).  attn_dtype=np.float32 evaluates the attention in
    single precision, np.float16 with fp16 operands: the differences between the evaluations measure
    how far rounding-level differences travel through the quantised blocks."""
    blocks, ends = metadata(hp)
    S = (hp["img"] - 1) // 4 + 1
    pe = pos_embed(tensors["hiera.pos_embed"], tensors["hiera.pos_embed_window"], S)
    x = prefix(img_chw, tensors["hiera.patch_embed.weight"], tensors["hiera.patch_embed.bias"], pe)
    stages = []
    for i, meta in enumerate(blocks):
        p = f"hiera.blocks.{i}."
        x = block(meta, {k[len(p):]: v for k, v in tensors.items() if k.startswith(p)}, x, attn_dtype)
        if i in ends:
            stages.append(x)
    convs = [(tensors[f"fpn.convs.{j}.weight"], tensors[f"fpn.convs.{j}.bias"]) for j in range(4)]
    return stages, fpn(stages, convs, hp["fpn_top_down_levels"], hp["scalp"])
