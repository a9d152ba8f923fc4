"""Host-side model preparation for the B200 encoder: hyper-parameters, the
reference quantiser rule and seeded random-init weights.

The benchmark configurations of this project use random-init weights (no
checkpoints are available): N(0, 0.02) for every weight and bias, LayerNorm
weight 1 / bias 0, RoPE tables from compute_axial_cis, linear weights
quantised with the rule of the reference's quantize tool
(examples/quantize.cpp:195-245 -> ggml_quantize_chunk, i.e. ggml's
quantize_row_*_ref).  Tensor names and ggml shapes are those of
sam3_register_tensors (sam3.cpp:2529-2600).
"""
from __future__ import annotations

import numpy as np

F32, F16, Q4_0, Q4_1, Q8_0 = 0, 1, 2, 3, 8

# SAM3 visual encoder (sam3.cpp:74-98, visual_only): ViT-32 at 1008^2
SAM3_VIT = dict(img=1008, patch=14, embed=1024, depth=32, heads=16, mlp=4736, window=24,
                global_idx=(7, 15, 23, 31), pos_grid=24, neck_dim=256, wtype=Q8_0)

# SAM2.1 Hiera-tiny image encoder (config 1's backbone) at 1024
SAM2_HIERA_TINY = dict(img=1024, embed=96, heads=1, stages=[1, 2, 7, 2], q_pool=3, window_spec=[8, 4, 14, 7],
                       global_idx=[5, 7, 9], bkg_h=7, bkg_w=7, neck_dim=256, fpn_top_down_levels=[2, 3], scalp=1)

# SAM2.1 Hiera-base+ image encoder (config 5's tracker backbone) at 1024
SAM2_HIERA_BASE_PLUS = dict(img=1024, embed=112, heads=2, stages=[2, 3, 16, 3], q_pool=3, window_spec=[8, 4, 14, 7],
                            global_idx=[12, 16, 20], bkg_h=14, bkg_w=14, neck_dim=256, fpn_top_down_levels=[2, 3],
                            scalp=1)

# reduced configuration with the same structure (windows, a global block,
# 3x3 pos-embed tiling, all four neck scales) for CPU-checkable parity tests
SAM3_VIT_TEST = dict(img=672, patch=14, embed=256, depth=2, heads=4, mlp=1024, window=24,
                     global_idx=(1,), pos_grid=16, neck_dim=256, wtype=Q8_0)


def quantize_rows(qtype: int, w: np.ndarray) -> np.ndarray:
    """ggml_quantize_chunk (reference rule) over rows of f32 [N, K]; returns uint8 [N, row_bytes]."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    if k % 32:
        raise ValueError("row length must be a multiple of 32")
    blocks = w.reshape(-1, 32)
    if qtype == Q8_0:
        d = np.abs(blocks).max(axis=1, keepdims=True) / np.float32(127)
        with np.errstate(divide="ignore"):
            idv = np.where(d == 0, np.float32(0), np.float32(1) / d).astype(np.float32)
        v = (blocks * idv).astype(np.float32)
        q = (np.sign(v) * np.floor(np.abs(v) + np.float32(0.5))).astype(np.int8)  # roundf: half away from zero
        out = np.concatenate([d.astype(np.float16).view(np.uint8), q.view(np.uint8)], axis=1)
        return out.reshape(n, -1)
    if qtype == Q4_0:
        imax = np.abs(blocks).argmax(axis=1)[:, None]
        mx = np.take_along_axis(blocks, imax, axis=1)
        d = (mx / np.float32(-8)).astype(np.float32)
        with np.errstate(divide="ignore"):
            idv = np.where(d == 0, np.float32(0), np.float32(1) / d).astype(np.float32)
        q = np.trunc((blocks * idv).astype(np.float32) + np.float32(8.5)).astype(np.int32)
        q = np.clip(q, 0, 15).astype(np.uint8)
        packed = q[:, :16] | (q[:, 16:] << 4)
        out = np.concatenate([d.astype(np.float16).view(np.uint8), packed], axis=1)
        return out.reshape(n, -1)
    raise ValueError(f"unsupported quant type {qtype}")


def compute_axial_cis(dim: int, end_x: int, end_y: int, theta: float = 10000.0, scale: float = 1.0) -> np.ndarray:
    """RoPE table as stored in the weight file: [N][dim/2] (cos, sin) pairs,
    x frequencies first (sam3_compute_axial_cis, sam3.cpp:3559-3590)."""
    q = dim // 4
    freqs = (1.0 / np.power(np.float32(theta), np.arange(0, dim, 4, dtype=np.float32)[:q] / np.float32(dim))).astype(
        np.float32)
    t = np.arange(end_x * end_y, dtype=np.float32)
    tx = (t % end_x) * np.float32(scale)
    ty = np.floor(t / end_x) * np.float32(scale)
    ax = np.outer(tx, freqs).astype(np.float32)
    ay = np.outer(ty, freqs).astype(np.float32)
    out = np.empty((end_x * end_y, 2 * q, 2), np.float32)
    out[:, :q, 0], out[:, :q, 1] = np.cos(ax), np.sin(ax)
    out[:, q:, 0], out[:, q:, 1] = np.cos(ay), np.sin(ay)
    return out


def random_vit_weights(hp: dict, seed: int = 0) -> dict:
    """name -> (ggml type, array, ggml ne) for the visual encoder and tracker neck."""
    rng = np.random.default_rng(seed)
    E, p, M, D, G, g, ws = hp["embed"], hp["patch"], hp["mlp"], hp["neck_dim"], hp["img"] // hp["patch"], \
        hp["pos_grid"], hp["window"]
    wt = hp["wtype"]

    def normal(*shape):
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)).astype(np.float32)

    t = {}
    t["vit.patch_embed.proj.weight"] = (F32, normal(E, 3, p, p), (p, p, 3, E))
    t["vit.pos_embed"] = (F32, normal(g, g, E), (E, g, g, 1))
    t["vit.ln_pre.weight"] = (F32, np.ones(E, np.float32), (E,))
    t["vit.ln_pre.bias"] = (F32, np.zeros(E, np.float32), (E,))
    glob = set(hp["global_idx"])
    cis_win = compute_axial_cis(E // hp["heads"], ws, ws)
    cis_glob = compute_axial_cis(E // hp["heads"], G, G, scale=ws / G)
    for i in range(hp["depth"]):
        pre = f"vit.blocks.{i}."
        for ln in ("norm1", "norm2"):
            t[pre + ln + ".weight"] = (F32, np.ones(E, np.float32), (E,))
            t[pre + ln + ".bias"] = (F32, np.zeros(E, np.float32), (E,))
        for name, k, n in (("attn.qkv", E, 3 * E), ("attn.proj", E, E), ("mlp.lin1", E, M), ("mlp.lin2", M, E)):
            t[pre + name + ".weight"] = (wt, quantize_rows(wt, normal(n, k)), (k, n))
            t[pre + name + ".bias"] = (F32, normal(n), (n,))
        cis = cis_glob if i in glob else cis_win
        t[pre + "attn.freqs_cis"] = (F32, cis, (2, cis.shape[1], cis.shape[0]))
    MID = 512
    pre = "neck.trk."
    t[pre + "0.dconv_2x2_0.weight"] = (F32, normal(E, MID, 2, 2), (2, 2, MID, E))
    t[pre + "0.dconv_2x2_0.bias"] = (F32, normal(MID), (MID,))
    t[pre + "0.dconv_2x2_1.weight"] = (F32, normal(MID, D, 2, 2), (2, 2, D, MID))
    t[pre + "0.dconv_2x2_1.bias"] = (F32, normal(D), (D,))
    t[pre + "1.dconv_2x2.weight"] = (F32, normal(E, MID, 2, 2), (2, 2, MID, E))
    t[pre + "1.dconv_2x2.bias"] = (F32, normal(MID), (MID,))
    for s, cin in ((0, D), (1, MID), (2, E), (3, E)):
        t[pre + f"{s}.conv_1x1.weight"] = (F32, normal(D, cin, 1, 1), (1, 1, cin, D))
        t[pre + f"{s}.conv_1x1.bias"] = (F32, normal(D), (D,))
        t[pre + f"{s}.conv_3x3.weight"] = (F32, normal(D, D, 3, 3), (3, 3, D, D))
        t[pre + f"{s}.conv_3x3.bias"] = (F32, normal(D), (D,))
    return t


def random_det_neck_weights(hp: dict, seed: int = 0) -> dict:
    """The detector neck of a full SAM3 model ("neck.det.*", the tracker neck's shapes, sam3.cpp:2556-2600)."""
    t = random_vit_weights(dict(hp, depth=0), seed=seed)
    return {k.replace("neck.trk.", "neck.det."): v for k, v in t.items() if k.startswith("neck.trk.")}


def random_images(n: int, side: int, seed: int = 0) -> np.ndarray:
    """n seeded uniform uint8 RGB images, HWC."""
    rng = np.random.default_rng(seed)
    return rng.integers(0, 256, size=(n, side, side, 3), dtype=np.uint8)
