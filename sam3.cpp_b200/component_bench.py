"""Timing of the runners beside the visual encoder, at the sizes of the
benchmark configurations they serve (bench.py --workload pcs | video):

  pcs   : config 4's text-prompt detector per image -- text encoder (24 x
          1024, 32 tokens), fusion encoder (6 layers over 72 x 72 tokens),
          DETR decoder (6 layers, 200 queries, box-relative bias, scoring,
          presence) and segmentation head (200 masks of 288 x 288), Q4_0
          linear weights, chained through device pointers (*_run_device), as
          sam3_segment_pcs runs them after the image encoder.
  video : config 5's tracker stages per frame and object -- memory attention
          (4 layers, 64 x 64 current tokens against 7 memory frames + 16
          object pointers = 28,736 memory tokens) and memory encoder (mask
          logits 256 x 256 -> 64-channel memory), Q8_0 linear weights.

Weights are random-init N(0, 1/sqrt(K)) quantised with the reference rule;
one tensor per distinct shape is generated and shared by every layer of that
shape (timing does not depend on the values).  Inputs are seeded random
device buffers.  Times are CUDA events on the backend stream.
"""
from __future__ import annotations

import ctypes
import math

import numpy as np

F32, F16, Q4_0, Q8_0 = 0, 1, 2, 8


class _Weights:
    """name -> (ggml type, array, ne), one random array per (type, shape)."""

    def __init__(self, model_mod, qtype: int, seed: int = 0):
        self.m, self.qtype, self.rng, self.cache, self.t = model_mod, qtype, np.random.default_rng(seed), {}, {}

    def vec(self, name, n, base=0.0, std=0.02):
        key = ("v", n, base)
        if key not in self.cache:
            self.cache[key] = (base + self.rng.normal(0, std, size=n)).astype(np.float32)
        self.t[name] = (F32, self.cache[key], (n,))

    def f32(self, name, shape_rows_first):
        arr = self.rng.normal(0, 0.02, size=shape_rows_first).astype(np.float32)
        self.t[name] = (F32, arr, arr.shape[::-1])

    def lin(self, name, K, N, bias=True, wname=None):
        key = ("w", K, N)
        if key not in self.cache:
            w = self.rng.normal(0, 1.0 / math.sqrt(K), size=(N, K)).astype(np.float32)
            self.cache[key] = self.m.quantize_rows(self.qtype, w)
        self.t[wname or name + ".weight"] = (self.qtype, self.cache[key], (K, N))
        if bias:
            self.vec(name + ".bias", N)

    def in_proj(self, prefix, D):
        """A fused [D, 3D] in_proj_weight / in_proj_bias pair."""
        self.lin(prefix + ".in_proj", D, 3 * D, bias=False, wname=prefix + ".in_proj_weight")
        self.vec(prefix + ".in_proj_bias", 3 * D)

    def norm(self, name, n):
        self.vec(name + ".weight", n, 1.0, 0.1)
        self.vec(name + ".bias", n, 0.0, 0.1)


def pcs_weights(model_mod, vocab=49408, ctx=32, width=1024, layers=24, D=256):
    w = _Weights(model_mod, Q4_0)
    w.f32("text.token_embed.weight", (vocab, width))
    w.f32("text.pos_embed", (ctx, width))
    for i in range(layers):
        p = f"text.blocks.{i}."
        w.lin(p + "attn.in_proj", width, 3 * width)
        w.lin(p + "attn.out_proj", width, width)
        w.norm(p + "ln_1", width)
        w.norm(p + "ln_2", width)
        w.lin(p + "mlp.fc1", width, 4 * width)
        w.lin(p + "mlp.fc2", 4 * width, width)
    w.norm("text.ln_final", width)
    w.lin("text.resizer", width, D)
    text = w.t
    w.t = {}
    for i in range(6):
        p = f"fenc.layers.{i}."
        for a in ("sa", "ca"):
            w.in_proj(p + a, D)
            w.lin(p + a + ".out_proj", D, D)
        w.lin(p + "linear1", D, 2048)
        w.lin(p + "linear2", 2048, D)
        for n in ("norm1", "norm2", "norm3"):
            w.norm(p + n, D)
    fenc = w.t
    w.t = {}
    NQ, NH = 200, 8
    w.f32("ddec.query_embed.weight", (NQ, D))
    w.f32("ddec.presence_token.weight", (1, D))
    w.f32("ddec.reference_points.weight", (NQ, 4))
    for n in ("ddec.norm", "ddec.presence_token_out_norm", "scoring.prompt_mlp.out_norm"):
        w.norm(n, D)
    for j in range(3):
        w.lin(f"ddec.bbox_embed.layers.{j}", D, 4 if j == 2 else D)
        w.lin(f"ddec.presence_token_head.layers.{j}", D, 1 if j == 2 else D)
    w.lin("ddec.ref_point_head.layers.0", 512, D)
    w.lin("ddec.ref_point_head.layers.1", D, D)
    for a in ("x", "y"):
        w.t[f"ddec.boxRPB_embed_{a}.layers.0.weight"] = (F32, w.rng.normal(0, 0.7, size=(D, 2)).astype(np.float32),
                                                         (2, D))
        w.vec(f"ddec.boxRPB_embed_{a}.layers.0.bias", D)
        w.lin(f"ddec.boxRPB_embed_{a}.layers.1", D, NH)
    w.lin("scoring.prompt_mlp.layers.0", D, 2048)
    w.lin("scoring.prompt_mlp.layers.1", 2048, D)
    w.lin("scoring.prompt_proj", D, D)
    w.lin("scoring.hs_proj", D, D)
    for i in range(6):
        p = f"ddec.layers.{i}."
        for a in ("sa", "ca", "ca_text"):
            w.in_proj(p + a, D)
            w.lin(p + a + ".out_proj", D, D)
        w.lin(p + "linear1", D, 2048)
        w.lin(p + "linear2", 2048, D)
        for n in ("norm1", "norm2", "norm_ca_text", "norm3"):
            w.norm(p + n, D)
    ddec = w.t
    w.t = {}
    w.in_proj("seg.cross_attend_prompt", D)
    w.lin("seg.cross_attend_prompt.out_proj", D, D)
    w.norm("seg.cross_attn_norm", D)
    conv3 = w.rng.normal(0, 1.0 / math.sqrt(9 * D), size=(D, D, 3, 3)).astype(np.float32)
    for i in range(3):
        w.t[f"seg.pixel_decoder.conv_layers.{i}.weight"] = (F32, conv3, (3, 3, D, D))
        w.vec(f"seg.pixel_decoder.conv_layers.{i}.bias", D)
        w.norm(f"seg.pixel_decoder.norms.{i}", D)
    w.t["seg.instance_seg_head.weight"] = (F32, w.rng.normal(0, 1 / 16, size=(D, D, 1, 1)).astype(np.float32),
                                           (1, 1, D, D))
    w.vec("seg.instance_seg_head.bias", D)
    for j in range(3):
        w.lin(f"seg.mask_predictor.mask_embed.layers.{j}", D, D)
    return text, fenc, ddec, w.t


def video_weights(model_mod, D=256, MD=64):
    w = _Weights(model_mod, Q8_0)
    for i in range(4):
        p = f"mem_attn.layers.{i}."
        for n in ("sa.q_proj", "sa.k_proj", "sa.v_proj", "sa.out_proj", "ca.q_proj", "ca.out_proj"):
            w.lin(p + n, D, D)
        w.lin(p + "ca.k_proj", MD, D)
        w.lin(p + "ca.v_proj", MD, D)
        w.lin(p + "linear1", D, 2048)
        w.lin(p + "linear2", 2048, D)
        for n in ("norm1", "norm2", "norm3"):
            w.norm(p + n, D)
    w.norm("mem_attn.norm", D)
    attn = w.t
    w.t = {}
    ch = (1, 4, 16, 64, 256)
    for s, (ci, ni) in enumerate(((0, 1), (3, 4), (6, 7), (9, 10))):
        k = w.rng.normal(0, 1 / math.sqrt(9 * ch[s]), size=(ch[s + 1], ch[s], 3, 3)).astype(np.float32)
        w.t[f"mem_enc.ds.{ci}.weight"] = (F32, k, (3, 3, ch[s], ch[s + 1]))
        w.vec(f"mem_enc.ds.{ci}.bias", ch[s + 1])
        w.norm(f"mem_enc.ds.{ni}", ch[s + 1])
    for name, o in (("mem_enc.ds.12", D), ("mem_enc.pix_feat_proj", D), ("mem_enc.out_proj", MD)):
        w.t[name + ".weight"] = (F32, w.rng.normal(0, 1 / 16, size=(o, D, 1, 1)).astype(np.float32), (1, 1, D, o))
        w.vec(name + ".bias", o)
    for i in range(2):
        p = f"mem_enc.fuser.{i}."
        w.t[p + "dwconv.weight"] = (F32, w.rng.normal(0, 1 / 7, size=(D, 1, 7, 7)).astype(np.float32), (7, 7, 1, D))
        w.vec(p + "dwconv.bias", D)
        w.norm(p + "norm", D)
        w.lin(p + "pwconv1", D, 1024)
        w.lin(p + "pwconv2", 1024, D)
        w.vec(p + "gamma", D, 0.0, 0.5)
    return attn, w.t


def hiera_weights(model_mod, enc, hp: dict) -> dict:
    """Random-init weights of a SAM2 Hiera trunk + FPN, block shapes taken from the created encoder
    (sam3b200_hiera_block_info); linear weights Q8_0 where the row length allows it, else F16."""
    w = _Weights(model_mod, Q8_0, seed=11)
    E, ws0 = hp["embed"], hp["window_spec"][0]
    w.t["hiera.patch_embed.weight"] = (F32, w.rng.normal(0, 0.02, size=(E, 3, 7, 7)).astype(np.float32), (7, 7, 3, E))
    w.vec("hiera.patch_embed.bias", E)
    w.t["hiera.pos_embed"] = (F32, w.rng.normal(0, 0.02, size=(E, hp["bkg_h"], hp["bkg_w"])).astype(np.float32),
                              (hp["bkg_w"], hp["bkg_h"], E))
    w.t["hiera.pos_embed_window"] = (F32, w.rng.normal(0, 0.02, size=(E, ws0, ws0)).astype(np.float32),
                                     (ws0, ws0, E))
    def lin(name, K, N):
        # ggml's quantiser keeps a tensor whose row length is no multiple of 32 in F16
        if K % 32 == 0:
            w.lin(name, K, N)
            return
        arr = w.rng.normal(0, 1.0 / math.sqrt(K), size=(N, K)).astype(np.float16)
        w.t[name + ".weight"] = (F16, arr, (K, N))
        w.vec(name + ".bias", N)

    for i in range(sum(hp["stages"])):
        di, do = enc.block_info(i)[:2]
        p = f"hiera.blocks.{i}."
        w.norm(p + "norm1", di)
        w.norm(p + "norm2", do)
        lin(p + "attn.qkv", di, 3 * do)
        lin(p + "attn.proj", do, do)
        lin(p + "mlp.fc1", do, 4 * do)
        lin(p + "mlp.fc2", 4 * do, do)
        if di != do:
            lin(p + "proj", di, do)
    D = hp["neck_dim"]
    for j in range(4):
        C = E * 2 ** (3 - j)
        w.t[f"fpn.convs.{j}.weight"] = (F32, w.rng.normal(0, 0.02, size=(D, C)).astype(np.float32), (1, 1, C, D))
        w.vec(f"fpn.convs.{j}.bias", D)
    return w.t


def sam_dec_weights(model_mod, D=256) -> dict:
    """Random-init prompt encoder + mask decoder weights (sam3.cpp:1854-1968 names), Q8_0 linear weights."""
    w = _Weights(model_mod, Q8_0, seed=12)

    def f32(name, shape, std=1.0):
        arr = w.rng.normal(0, std, size=shape).astype(np.float32)
        w.t[name] = (F32, arr, arr.shape[::-1] if len(shape) > 1 else (shape[0], 1))

    def attn(pfx, idim):
        for n in ("q", "k", "v"):
            w.lin(f"{pfx}.{n}_proj", D, idim)
        w.lin(f"{pfx}.out_proj", idim, D)

    w.t["sam_pe.pe_gaussian"] = (F32, w.rng.normal(0, 1, size=(2, 128)).astype(np.float32), (128, 2))
    for i in range(4):
        f32(f"sam_pe.point_embeddings.{i}.weight", (D,))
    for n in ("sam_pe.not_a_point_embed.weight", "sam_pe.no_mask_embed.weight", "sam_dec.iou_token.weight",
              "sam_dec.obj_score_token.weight"):
        f32(n, (D,))
    w.t["no_mem_embed"] = (F32, w.rng.normal(0, 0.02, size=D).astype(np.float32), (D, 1, 1))
    w.t["sam_dec.mask_tokens.weight"] = (F32, w.rng.normal(0, 1, size=(4, D)).astype(np.float32), (D, 4))
    for i in range(2):
        p = f"sam_dec.twoway.{i}"
        attn(p + ".sa", D)
        attn(p + ".cross_attn_token_to_image", 128)
        attn(p + ".cross_attn_image_to_token", 128)
        for j in range(1, 5):
            w.norm(f"{p}.norm{j}", D)
        w.lin(p + ".mlp.lin1", D, 2048)
        w.lin(p + ".mlp.lin2", 2048, D)
    attn("sam_dec.final_attn", 128)
    w.norm("sam_dec.final_norm", D)
    w.t["sam_dec.upscale.0.weight"] = (F32, w.rng.normal(0, 0.05, size=(D, 64, 2, 2)).astype(np.float32), (2, 2, 64, D))
    w.vec("sam_dec.upscale.0.bias", 64)
    w.norm("sam_dec.upscale.1", 64)
    w.t["sam_dec.upscale.3.weight"] = (F32, w.rng.normal(0, 0.1, size=(64, 32, 2, 2)).astype(np.float32), (2, 2, 32, 64))
    w.vec("sam_dec.upscale.3.bias", 32)
    for name, oc in (("sam_dec.conv_s0", 32), ("sam_dec.conv_s1", 64)):
        w.t[name + ".weight"] = (F32, w.rng.normal(0, 0.05, size=(oc, D)).astype(np.float32), (1, 1, D, oc))
        w.vec(name + ".bias", oc)
    for m in range(4):
        for j in range(3):
            w.lin(f"sam_dec.hyper.{m}.layers.{j}", D, 32 if j == 2 else D)
    for head, nout in (("iou_prediction_head", 4), ("pred_obj_score_head", 1)):
        for j in range(3):
            w.lin(f"sam_dec.{head}.layers.{j}", D, nout if j == 2 else D)
    return w.t


def tracker_weights(D=256, MD=64, num_maskmem=7) -> dict:
    """Random-init object-pointer and temporal-code weights of the video tracker."""
    rng = np.random.default_rng(13)
    t = {}
    for j in range(3):
        t[f"obj_ptr_proj.layers.{j}.weight"] = rng.normal(0, 1 / 16, size=(D, D)).astype(np.float32)
        t[f"obj_ptr_proj.layers.{j}.bias"] = rng.normal(0, 0.1, size=D).astype(np.float32)
    t["no_obj_ptr"] = rng.normal(0, 1, size=D).astype(np.float32)
    t["obj_ptr_tpos_proj.weight"] = rng.normal(0, 1 / 16, size=(MD, D)).astype(np.float32)
    t["obj_ptr_tpos_proj.bias"] = rng.normal(0, 0.1, size=MD).astype(np.float32)
    t["mem_enc.tpos_enc"] = rng.normal(0, 0.1, size=(num_maskmem, MD)).astype(np.float32)
    return {k: (F32, v, v.shape[::-1]) for k, v in t.items()}


def _events(torch, stream):
    e = torch.cuda.Event(enable_timing=True)
    e.record(stream)
    return e


def run_pcs(b200, model_mod, be, steps: int, warmup: int) -> dict:
    import torch
    lib = b200.lib()
    D, G, L, NQ = 256, 72, 32, 200
    N = G * G
    text_t, fenc_t, ddec_t, seg_t = pcs_weights(model_mod)
    txt = be.text_encoder(dict(width=1024, heads=16, layers=24, ctx_len=L, vocab=49408, out_dim=D))
    fe = be.fusion_encoder(dict(d_model=D, heads=8, layers=6, ffn_dim=2048, max_tokens=N, max_prompt=L))
    dd = be.detr_decoder(dict(d_model=D, heads=8, layers=6, ffn_dim=2048, num_queries=NQ, feat=G, max_prompt=L))
    sh = be.seg_head(dict(d_model=D, heads=8, feat=G, max_queries=NQ, max_prompt=L))
    for r, t in ((txt, text_t), (fe, fenc_t), (dd, ddec_t), (sh, seg_t)):
        r.load(t)
    rng = np.random.default_rng(3)
    bufs = {k: be.upload(rng.normal(0, 1, size=(n, D)).astype(np.float32))
            for k, n in (("neck0", 16 * N), ("neck1", 4 * N), ("neck2", N), ("pe", N))}
    n_valid = 7
    bias = be.upload(np.where(np.arange(L) < n_valid, 0.0, -1.0e9).astype(np.float32))
    valid = be.upload(np.where(np.arange(L) < n_valid, L / n_valid, 0.0).astype(np.float32))
    ids = np.array([49406, 320, 1929, 537, 320, 2368, 49407], np.int32)
    text_p, q_p, b_p, s_p, p_p, cond_p = (ctypes.c_void_p() for _ in range(6))
    stream = torch.cuda.ExternalStream(be.stream)

    def step(marks=None):
        def mark():
            if marks is not None:
                marks.append(_events(torch, stream))
        mark()
        b200._check(lib.sam3b200_text_encode(txt.h, ids.ctypes.data, ids.size), "text_encode")
        b200._check(lib.sam3b200_text_output(txt.h, ctypes.byref(text_p), (ctypes.c_int64 * 2)()), "text_output")
        mark()
        b200._check(lib.sam3b200_fenc_run_device(fe.h, bufs["neck2"].ptr, text_p.value, bufs["pe"].ptr, bias.ptr, N, L),
                    "fenc")
        b200._check(lib.sam3b200_fenc_output(fe.h, ctypes.byref(cond_p)), "fenc_output")
        mark()
        b200._check(lib.sam3b200_ddec_run_device(dd.h, cond_p.value, bufs["pe"].ptr, text_p.value, bias.ptr, valid.ptr,
                                                 L), "ddec")
        b200._check(lib.sam3b200_ddec_outputs(dd.h, ctypes.byref(q_p), ctypes.byref(b_p), ctypes.byref(s_p),
                                              ctypes.byref(p_p)), "ddec_outputs")
        mark()
        b200._check(lib.sam3b200_seg_run_device(sh.h, cond_p.value, bufs["neck0"].ptr, bufs["neck1"].ptr,
                                                q_p.value + D * 4, NQ, text_p.value, bias.ptr, L), "seg")
        mark()

    for _ in range(warmup):
        step()
    be.synchronize()
    stages = np.zeros(4)
    for _ in range(steps):
        marks = []
        step(marks)
        be.synchronize()
        stages += [marks[i].elapsed_time(marks[i + 1]) for i in range(4)]
    stages /= steps
    for r in (txt, fe, dd, sh):
        r.free()
    total = float(stages.sum())
    return {"metric": "SAM3 PCS detector ms per image (text + fusion + DETR + seg head)", "value": total,
            "unit": "ms", "higher_is_better": False, "steps": steps, "warmup": warmup, "dtype": "int8/f32",
            "data": "synthetic", "n_gpus": 1,
            "config": {"workload": "cfg4 detector after the image encoder: 32 text tokens (7 valid), 72x72 image "
                                   "tokens, 200 queries, 288x288 masks, Q4_0 linear weights (random-init)"},
            "stages_ms": {"text_encoder": stages[0], "fusion_encoder": stages[1], "detr_decoder": stages[2],
                          "seg_head": stages[3]}}


def run_pvs(b200, model_mod, be, steps: int, warmup: int) -> dict:
    """Config 1 (SAM2.1 Hiera-tiny, PVS): a seeded uint8 1024^2 image -> SAM2 preprocessing -> Hiera-tiny
    trunk + FPN -> prompt encoder + mask decoder for one positive point -> the four masks at the image's
    size.  value: device-timed images/s with the image already on the device; e2e: the same step from a
    pinned host image with the masks read back (sam3b200_tensor_set / _get around it)."""
    import torch
    lib = b200.lib()
    hp = model_mod.SAM2_HIERA_TINY
    S = hp["img"]
    enc = be.hiera(hp)
    enc.load(hiera_weights(model_mod, enc, hp))
    dec = be.sam_decoder(dict(feat_size=S // 16, embed=256, depth=2, heads=8, mlp_dim=2048, n_multimask=3,
                              pred_obj_scores=1, max_points=16))
    dec.load(sam_dec_weights(model_mod))
    img = model_mod.random_images(1, S, seed=77)[0]
    src = be.upload(img)
    pinned = torch.from_numpy(img).pin_memory()
    chw = be.alloc(3 * S * S * 4)
    masks = be.alloc(4 * S * S)
    masks_host = torch.empty(4 * S * S, dtype=torch.uint8).pin_memory()
    point, label = [[0.41 * S, 0.43 * S]], [1]
    stream = torch.cuda.ExternalStream(be.stream)

    def step(marks=None):
        def mark():
            if marks is not None:
                marks.append(_events(torch, stream))
        mark()
        be.preprocess_sam2(src, S, S, S, chw)
        enc.encode_device(chw)
        mark()
        dec.run(enc.output_ptr(2), enc.output_ptr(0), enc.output_ptr(1), point, label, S, S, S)
        for m in range(4):
            b200._check(lib.sam3b200_sam_dec_mask(dec.h, m, S, S, masks.ptr + m * S * S), "sam_dec_mask")
        mark()

    def step_e2e():
        b200._check(lib.sam3b200_tensor_set(be.h, src.ptr, pinned.data_ptr(), 0, S * S * 3), "image set")
        step()
        b200._check(lib.sam3b200_tensor_get(be.h, masks.ptr, masks_host.data_ptr(), 0, 4 * S * S), "masks get")

    def timed(fn):
        be.synchronize()
        e0, e1 = _events(torch, stream), None
        for _ in range(steps):
            fn()
        e1 = _events(torch, stream)
        be.synchronize()
        return e0.elapsed_time(e1) / steps

    for _ in range(warmup):
        step()
        step_e2e()
    be.synchronize()
    stages = np.zeros(2)
    for _ in range(steps):
        marks = []
        step(marks)
        be.synchronize()
        stages += [marks[i].elapsed_time(marks[i + 1]) for i in range(2)]
    stages /= steps
    ms = timed(step)
    e2e_ms = timed(step_e2e)
    enc.free()
    dec.free()
    return {"metric": "SAM2.1 Hiera-tiny PVS images/s (preprocess + encode + one-point decode + 4 masks)",
            "value": 1000.0 / ms, "unit": "images/s", "higher_is_better": True, "steps": steps, "warmup": warmup,
            "ms_per_step": ms, "dtype": "int8 linear / fp16 attention", "data": "synthetic", "n_gpus": 1,
            "config": {"workload": "cfg1: SAM2.1 Hiera-tiny 1024^2, Q8_0 linear weights where the row length allows "
                                   "(random-init), one positive point, 4 masks at 1024^2"},
            "e2e": {"value": 1000.0 / e2e_ms, "unit": "images/s", "h2d_bytes_per_step": S * S * 3,
                    "d2h_bytes_per_step": 4 * S * S},
            "stages_ms": {"preprocess_and_encode": stages[0], "decode_and_masks": stages[1]}}


def run_video(b200, model_mod, be, steps: int, warmup: int) -> dict:
    import torch
    lib = b200.lib()
    D, MD, H, F, P = 256, 64, 64, 7, 16
    N, M = H * H, F * H * H + 4 * P
    attn_t, enc_t = video_weights(model_mod)
    ma = be.mem_attention(dict(d_model=D, mem_dim=MD, layers=4, ffn_dim=2048, max_tokens=N, max_mem_tokens=M))
    me = be.mem_encoder(dict(feat=H, img=1024, d_model=D, mem_dim=MD, fuser_layers=2, fuser_dim=1024,
                             sigmoid_scale=20.0, sigmoid_bias=-10.0, max_mask=(4 * H) ** 2))
    ma.load(attn_t)
    me.load(enc_t)
    rng = np.random.default_rng(5)

    def up(*shape):
        return be.upload(rng.normal(0, 1, size=shape).astype(np.float32))

    curr, spos, prompt, ppos = up(N, D), up(N, D), up(M, MD), up(M, MD)
    ang = rng.uniform(0, 6.28, size=(N, D // 2)).astype(np.float32)
    rq_h = np.stack([np.cos(ang), np.sin(ang)], -1).astype(np.float32)
    rope_q, rope_k = be.upload(rq_h), be.upload(np.concatenate([rq_h] * F))
    logits, pix = up(4 * H, 4 * H), up(N, D)
    stream = torch.cuda.ExternalStream(be.stream)

    def step(marks=None):
        if marks is not None:
            marks.append(_events(torch, stream))
        b200._check(lib.sam3b200_mem_attn_run_device(ma.h, curr.ptr, spos.ptr, prompt.ptr, ppos.ptr, rope_q.ptr,
                                                     rope_k.ptr, N, M, 4 * P), "mem_attn")
        if marks is not None:
            marks.append(_events(torch, stream))
        b200._check(lib.sam3b200_mem_enc_run_device(me.h, logits.ptr, 4 * H, 4 * H, pix.ptr, 1.0), "mem_enc")
        if marks is not None:
            marks.append(_events(torch, stream))

    for _ in range(warmup):
        step()
    be.synchronize()
    stages = np.zeros(2)
    for _ in range(steps):
        marks = []
        step(marks)
        be.synchronize()
        stages += [marks[0].elapsed_time(marks[1]), marks[1].elapsed_time(marks[2])]
    stages /= steps
    ma.free()
    me.free()
    attn_flop = 4 * (4 * N * N * D + 4 * N * M * D)  # q k^T and p v of the self and cross attention, 4 layers
    return {"metric": "SAM3/SAM2 tracker memory stages ms per frame and object", "value": float(stages.sum()),
            "unit": "ms", "higher_is_better": False, "steps": steps, "warmup": warmup, "dtype": "int8/f32",
            "data": "synthetic", "n_gpus": 1,
            "config": {"workload": "cfg5 per frame: memory attention over 64x64 tokens against 7 memory frames + "
                                   "16 object pointers (28,736 memory tokens), memory encoder from 256x256 mask "
                                   "logits, Q8_0 linear weights (random-init)"},
            "stages_ms": {"memory_attention": stages[0], "memory_encoder": stages[1]},
            "memory_attention_attn_tflops": attn_flop / (stages[0] / 1e3) / 1e12,
            "memory_attention_attn_flop": attn_flop}


# Config 2: the standalone MUL_MAT sweep at the SAM3 ViT-32 shapes
# (qkv, proj, fc1, fc2 of sam3_vit_block_forward, sam3.cpp:3742,3783,3796,3799).
MMQ_SHAPES = (("qkv", 1024, 3072), ("proj", 1024, 1024), ("fc1", 1024, 4736), ("fc2", 4736, 1024))


def win_part_rows(G: int, win: int) -> np.ndarray:
    """Source row of each row of ggml_win_part's order for a G x G token map (G % win == 0)."""
    nw = G // win
    rows = np.empty(G * G, np.int64)
    for t in range(G * G):
        tx, ty = t % G, t // G
        rows[((ty // win) * nw + tx // win) * win * win + (tx % win) + win * (ty % win)] = t
    return rows


def run_mmq(b200, model_mod, be, steps: int, warmup: int, peak_int8_tops: float | None) -> dict:
    """Q8_0 and Q4_0 weights at the four ViT shapes, M = 5184 tokens, in token
    order and in ggml_win_part order (9 windows x 576 tokens).  Per case:
    the MUL_MAT kernel alone (CUDA events around its launches, via the
    backend profiler) and the whole op (activation quantisation + kernel),
    as TOP/s of 2*M*K*N.  Activations N(0, 1), weights N(0, 0.02) quantised
    with the reference rule.  Both arithmetics: exact (int8 block dots, the
    fp32 block fold) and dq16 (the dequantised fp16 operands on the fp16
    tensor cores; its op time includes the quantise + dequantise passes)."""
    import torch
    stream = torch.cuda.ExternalStream(be.stream)
    G, win, M = 72, 24, 72 * 72
    rng = np.random.default_rng(2)
    perm = win_part_rows(G, win)
    out = []
    for (qtype, qname), arith in [((Q8_0, "Q8_0"), "exact"), ((Q4_0, "Q4_0"), "exact"),
                                  ((Q8_0, "Q8_0"), "dq16"), ((Q4_0, "Q4_0"), "dq16")]:
        op = be.mul_mat if arith == "exact" else be.mul_mat_dq16
        for name, K, N in MMQ_SHAPES:
            wq = model_mod.quantize_rows(qtype, rng.normal(0, 0.02, size=(N, K)).astype(np.float32))
            w = be.weight(qtype, wq, K, N)
            bias = be.upload(rng.normal(0, 0.02, size=N).astype(np.float32))
            x = rng.standard_normal((M, K), dtype=np.float32)
            y = be.alloc(M * N * 4)
            for order, xs in (("tokens", x), ("win_part", x[perm])):
                xd = be.upload(np.ascontiguousarray(xs))
                for _ in range(warmup):
                    op(w, xd, M, y, bias=bias)
                be.synchronize()
                be.profile(True)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                for _ in range(steps):
                    op(w, xd, M, y, bias=bias)
                e1.record(stream)
                be.synchronize()
                op_ms = e0.elapsed_time(e1) / steps
                k_ms, k_n = be.profile_read(0)
                be.profile(False)
                k_ms /= max(k_n, 1)
                ops = 2.0 * M * K * N
                rec = {"type": qname, "arith": arith, "layer": name, "M": M, "K": K, "N": N, "order": order,
                       "kernel_us": k_ms * 1e3, "op_us": op_ms * 1e3,
                       "kernel_tops": ops / (k_ms * 1e-3) / 1e12, "op_tops": ops / (op_ms * 1e-3) / 1e12}
                if peak_int8_tops:
                    rec["kernel_frac_int8"] = rec["kernel_tops"] / peak_int8_tops
                out.append(rec)
                xd.free()
            y.free()
            bias.free()
            w.free()
    return {"sweep": out}
