"""ctypes front end of the CPU oracle (TEST INFRASTRUCTURE ONLY).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg
import this module, and only as the checker or the timed CPU restatement.
The product library never calls into it.  See ggml_oracle.h for what the
oracle restates and where each formula comes from.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

F32, F16, Q4_0, Q4_1, Q8_0, Q8_1 = 0, 1, 2, 3, 8, 9
BLOCK_BYTES = {Q8_0: 34, Q4_0: 18, Q4_1: 20, Q8_1: 36}
QK = 32

_lib = None


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        L.orc_fp32_to_fp16.restype = ctypes.c_uint16
        L.orc_fp32_to_fp16.argtypes = [ctypes.c_float]
        L.orc_row_size.restype = i64
        L.orc_row_size.argtypes = [i32, i64]
        for name in ("orc_quantize_q8_0_ref", "orc_quantize_q4_0_ref", "orc_quantize_q4_1_ref",
                     "orc_quantize_q8_0_act", "orc_quantize_q8_1_act"):
            getattr(L, name).argtypes = [vp, vp, i64]
            getattr(L, name).restype = None
        L.orc_quantize_chunk.argtypes = [i32, vp, vp, i64, i64]
        L.orc_quantize_chunk.restype = i64
        L.orc_dequantize_row.argtypes = [i32, vp, vp, i64]
        L.orc_dequantize_row.restype = None
        L.orc_vec_dot.argtypes = [i32, i64, vp, vp]
        L.orc_vec_dot.restype = ctypes.c_float
        L.orc_mul_mat.argtypes = [i32, vp, i64, i64, vp, i64, i64, vp, i64, i32]
        L.orc_mul_mat.restype = None
        L.orc_mul_mat_block_dots.argtypes = [i32, vp, i64, i64, vp, i64, vp, i32]
        L.orc_mul_mat_block_dots.restype = None
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def row_size(qtype: int, k: int) -> int:
    return int(lib().orc_row_size(qtype, k))


def quantize_weights(qtype: int, w: np.ndarray) -> np.ndarray:
    """ggml_quantize_chunk over rows of a float32 [N, K] matrix -> uint8 [N, row_size]."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    out = np.empty((n, row_size(qtype, k)), dtype=np.uint8)
    r = lib().orc_quantize_chunk(qtype, _ptr(w), _ptr(out), n, k)
    if r < 0:
        raise ValueError(f"unsupported quant type {qtype}")
    return out


def quantize_activations(vtype: int, x: np.ndarray) -> np.ndarray:
    """ggml-cpu activation quantiser (x86 rule) over rows of float32 [M, K]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    m, k = x.shape
    out = np.empty((m, row_size(vtype, k)), dtype=np.uint8)
    fn = {Q8_0: lib().orc_quantize_q8_0_act, Q8_1: lib().orc_quantize_q8_1_act}[vtype]
    for i in range(m):
        fn(x[i].ctypes.data, out[i].ctypes.data, k)
    return out


def dequantize(qtype: int, q: np.ndarray, k: int) -> np.ndarray:
    q = np.ascontiguousarray(q)
    rows = q.shape[0] if q.ndim == 2 else 1
    out = np.empty((rows, k), dtype=np.float32)
    rs = row_size(qtype, k)
    base = q.reshape(rows, -1)
    for i in range(rows):
        lib().orc_dequantize_row(qtype, base[i].ctypes.data, out[i].ctypes.data, k)
    return out


def mul_mat(qtype: int, wq: np.ndarray, K: int, N: int, x: np.ndarray, n_threads: int = 0) -> np.ndarray:
    """ggml_mul_mat(w, x): returns float32 [M, N] (ggml dst [N, M])."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    M = x.shape[0]
    assert x.shape[1] == K
    wq = np.ascontiguousarray(wq)
    y = np.empty((M, N), dtype=np.float32)
    n_threads = n_threads or (os.cpu_count() or 1)
    lib().orc_mul_mat(qtype, _ptr(wq), K, N, _ptr(x), K, M, _ptr(y), N, n_threads)
    return y


def mul_mat_dq16(qtype: int, wq: np.ndarray, K: int, N: int, x: np.ndarray) -> np.ndarray:
    """The library's DQ16 MUL_MAT arithmetic restated (checker only): x quantised to Q8_0 with the ggml-cpu
    rule, every activation code and every weight element dequantised (q * d, exact in float32) and rounded
    once to fp16, the products summed in float64 -- the tensor cores sum in fp32 in an unspecified order, so
    float64 is the reference that bounds them.  Returns float32 [M, N]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    a16 = dequantize(Q8_0, quantize_activations(Q8_0, x), K).astype(np.float16)
    w16 = dequantize(qtype, np.ascontiguousarray(wq), K).astype(np.float16)
    return (a16.astype(np.float64) @ w16.astype(np.float64).T).astype(np.float32)


def block_dots(qtype: int, wq: np.ndarray, K: int, N: int, x: np.ndarray, n_threads: int = 0) -> np.ndarray:
    """Per-(m, n, block) int32 dots of the integer codes: int32 [M, N, K/32]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    M = x.shape[0]
    out = np.empty((M, N, K // QK), dtype=np.int32)
    n_threads = n_threads or (os.cpu_count() or 1)
    lib().orc_mul_mat_block_dots(qtype, _ptr(np.ascontiguousarray(wq)), K, N, _ptr(x), M, _ptr(out), n_threads)
    return out


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, batch: int, N: int, heads: int, scale: float,
              n_threads: int = 0) -> np.ndarray:
    """ggml_flash_attn_ext in f32 (vit_oracle.c orc_attention): q, k, v [batch*heads][N][64] (ggml
    [64, N, heads, batch]) -> [batch*N][heads*64] (ggml [64, heads, N, batch])."""
    q, k, v = (np.ascontiguousarray(a, dtype=np.float32) for a in (q, k, v))
    out = np.empty((batch * N, heads * 64), np.float32)
    _vit_lib().orc_attention(q.ctypes.data, k.ctypes.data, v.ctypes.data, batch, N, heads, scale, out.ctypes.data,
                             n_threads or (os.cpu_count() or 1))
    return out


def attention_general(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float,
                      mask: np.ndarray | None = None, dtype=np.float64) -> np.ndarray:
    """ggml_flash_attn_ext with max_bias 0 and no softcap, in float64: q [B][H][NQ][D], k, v
    [B][H][NKV][D], mask f32 [NQ][NKV] (or None) added to the scaled scores; a key whose mask is -inf
    is skipped and a row with every key skipped gives zeros.  Returns f32 [B][NQ][H][D] (ggml dst
    [D, H, NQ, B])."""
    s = np.einsum("bhqd,bhkd->bhqk", q.astype(dtype), k.astype(dtype)) * dtype(scale)
    if mask is not None:
        s = s + mask.astype(dtype)[None, None]
    mx = np.max(s, axis=-1, keepdims=True)
    dead = ~np.isfinite(mx)
    p = np.exp(s - np.where(dead, 0.0, mx))
    p = np.where(np.isfinite(s), p, 0.0)
    den = p.sum(-1, keepdims=True)
    o = np.einsum("bhqk,bhkd->bhqd", p, v.astype(dtype)) / np.where(den > 0, den, dtype(1.0))
    return o.transpose(0, 2, 1, 3).astype(np.float32)


def conv_transpose_2d(w: np.ndarray, x: np.ndarray, stride: int) -> np.ndarray:
    """ggml_conv_transpose_2d_p0 (sam3.cpp:3884; ggml op GGML_OP_CONV_TRANSPOSE_2D) in float64.

    w: fp16 [ic][oc][kh][kw] (ggml [KW, KH, OC, IC]); x: f32 [ic][ih][iw].  As ggml's CPU path, the
    input is rounded to fp16 before the products; out[oc][oy][ox] sums x[ic][iy][ix] * w[ic][oc][ky][kx]
    over oy = stride*iy + ky, ox = stride*ix + kx (no padding).  Returns f32 [oc][oh][ow]."""
    ic, oc, kh, kw = w.shape
    _, ih, iw = x.shape
    xs = x.astype(np.float16).astype(np.float64).reshape(ic, ih * iw)
    wd = w.astype(np.float64)
    oh, ow = (ih - 1) * stride + kh, (iw - 1) * stride + kw
    out = np.zeros((oc, oh, ow), np.float64)
    for ky in range(kh):
        for kx in range(kw):
            t = (wd[:, :, ky, kx].T @ xs).reshape(oc, ih, iw)
            out[:, ky:ky + stride * (ih - 1) + 1:stride, kx:kx + stride * (iw - 1) + 1:stride] += t
    return out.astype(np.float32)


def conv_2d(w: np.ndarray, x: np.ndarray, s0: int, s1: int, p0: int, p1: int, d0: int = 1, d1: int = 1,
            f16: bool = True) -> np.ndarray:
    """ggml_conv_2d (sam3.cpp:3819, 3891, 4474; ggml im2col + mul_mat) in float64.

    w: fp16 [oc][ic][kh][kw] (ggml [KW, KH, IC, OC]); x: f32 [ic][ih][iw], rounded to fp16 as ggml's
    im2col does for an F16 kernel; zero padding p0/p1, strides s0/s1, dilations d0/d1 (x then y).
    Returns f32 [oc][oh][ow].  f16=False: an F32 kernel (ggml's f32 im2col path, no rounding)."""
    oc, ic, kh, kw = w.shape
    _, ih, iw = x.shape
    ow = (iw + 2 * p0 - d0 * (kw - 1) - 1) // s0 + 1
    oh = (ih + 2 * p1 - d1 * (kh - 1) - 1) // s1 + 1
    xp = np.zeros((ic, ih + 2 * p1 + s1 * oh, iw + 2 * p0 + s0 * ow), np.float64)
    xp[:, p1:p1 + ih, p0:p0 + iw] = (x.astype(np.float16) if f16 else x).astype(np.float64)
    wd = w.astype(np.float64)
    out = np.zeros((oc, oh * ow), np.float64)
    for ky in range(kh):
        for kx in range(kw):
            y0, x0 = ky * d1, kx * d0
            patch = xp[:, y0:y0 + s1 * oh:s1, x0:x0 + s0 * ow:s0].reshape(ic, oh * ow)
            out += wd[:, :, ky, kx] @ patch
    return out.reshape(oc, oh, ow).astype(np.float32)


def get_rows(qtype: int, rows: np.ndarray, ncols: int, idx: np.ndarray) -> np.ndarray:
    """ggml_get_rows: dequantise the selected rows (ggml dequantize_row_* rules) -> f32 [n][ncols]."""
    if qtype == F32:
        return np.ascontiguousarray(rows.view(np.float32).reshape(-1, ncols)[idx])
    if qtype == F16:
        return rows.view(np.float16).reshape(-1, ncols)[idx].astype(np.float32)
    return dequantize(qtype, np.ascontiguousarray(rows.reshape(rows.shape[0], -1)[idx]), ncols)


def preprocess_sam2(rgb: np.ndarray, img: int) -> np.ndarray:
    """sam2_preprocess_image (sam3.cpp:3522-3548): uint8 HxWx3 -> ImageNet-normalised f32 [3][img][img]."""
    rgb = np.ascontiguousarray(rgb, dtype=np.uint8)
    out = np.empty((3, img, img), np.float32)
    _vit_lib().orc_preprocess_sam2(rgb.ctypes.data, rgb.shape[1], rgb.shape[0], img, out.ctypes.data)
    return out


# ---- SAM3 visual encoder restatement (vit_oracle.h) ------------------------

class _Hp(ctypes.Structure):
    _fields_ = [("img", ctypes.c_int), ("patch", ctypes.c_int), ("E", ctypes.c_int), ("depth", ctypes.c_int),
                ("heads", ctypes.c_int), ("mlp", ctypes.c_int), ("window", ctypes.c_int),
                ("n_global", ctypes.c_int), ("global_idx", ctypes.c_int * 4), ("pos_grid", ctypes.c_int),
                ("neck_dim", ctypes.c_int), ("wtype", ctypes.c_int)]


class _BlockW(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("norm1_w", "norm1_b", "norm2_w", "norm2_b", "qkv_w", "qkv_b",
                                               "proj_w", "proj_b", "fc1_w", "fc1_b", "fc2_w", "fc2_b", "freqs")]


class _NeckW(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("dc1_w", "dc1_b", "dc2_w", "dc2_b", "c1_w", "c1_b", "c3_w", "c3_b")]


class _VitW(ctypes.Structure):
    _fields_ = [("patch_w", ctypes.c_void_p), ("pos_embed", ctypes.c_void_p), ("ln_pre_w", ctypes.c_void_p),
                ("ln_pre_b", ctypes.c_void_p), ("blocks", _BlockW * 64), ("neck", _NeckW * 4)]


def _vit_lib():
    L = lib()
    if not getattr(L, "_vit_sigs", False):
        vp, i32 = ctypes.c_void_p, ctypes.c_int
        L.orc_preprocess_sam3.argtypes = [vp, i32, i32, i32, vp]
        L.orc_preprocess_sam2.argtypes = [vp, i32, i32, i32, vp]
        L.orc_vit_prefix.argtypes = [vp, vp, vp, vp, i32]
        L.orc_vit_block.argtypes = [vp, vp, i32, vp, i32]
        L.orc_neck.argtypes = [vp, vp, vp, vp, i32]
        L.orc_layer_norm.argtypes = [vp, vp, ctypes.c_int64, i32, ctypes.c_float, vp, vp, i32]
        L.orc_attention.argtypes = [vp, vp, vp, i32, i32, i32, ctypes.c_float, vp, i32]
        L.orc_set_attention_f64.argtypes = [i32]
        L.orc_set_attention_f64.restype = None
        for f in ("orc_preprocess_sam3", "orc_preprocess_sam2", "orc_vit_prefix", "orc_vit_block", "orc_neck", "orc_layer_norm",
                  "orc_attention"):
            getattr(L, f).restype = None
        L._vit_sigs = True
    return L


class OracleVit:
    """CPU restatement of the SAM3 visual encoder over a tensor dict
    (name -> (ggml type, array, ne), as produced by model.random_vit_weights)."""

    def __init__(self, hp: dict, tensors: dict, n_threads: int = 0, neck_prefix: str = "neck.trk."):
        self.hp, self.t = dict(hp), tensors
        self.nt = n_threads or (os.cpu_count() or 1)
        self.G = hp["img"] // hp["patch"]
        self._keep = []
        h = _Hp()
        h.img, h.patch, h.E, h.depth, h.heads = hp["img"], hp["patch"], hp["embed"], hp["depth"], hp["heads"]
        h.mlp, h.window, h.pos_grid, h.neck_dim, h.wtype = hp["mlp"], hp["window"], hp["pos_grid"], \
            hp["neck_dim"], hp["wtype"]
        h.n_global = len(hp["global_idx"])
        for i, g in enumerate(hp["global_idx"]):
            h.global_idx[i] = g
        self.h = h
        w = _VitW()
        w.patch_w = self._p("vit.patch_embed.proj.weight")
        w.pos_embed = self._p("vit.pos_embed")
        w.ln_pre_w, w.ln_pre_b = self._p("vit.ln_pre.weight"), self._p("vit.ln_pre.bias")
        for i in range(hp["depth"]):
            b, pre = w.blocks[i], f"vit.blocks.{i}."
            b.norm1_w, b.norm1_b = self._p(pre + "norm1.weight"), self._p(pre + "norm1.bias")
            b.norm2_w, b.norm2_b = self._p(pre + "norm2.weight"), self._p(pre + "norm2.bias")
            b.qkv_w, b.qkv_b = self._p(pre + "attn.qkv.weight"), self._p(pre + "attn.qkv.bias")
            b.proj_w, b.proj_b = self._p(pre + "attn.proj.weight"), self._p(pre + "attn.proj.bias")
            b.fc1_w, b.fc1_b = self._p(pre + "mlp.lin1.weight"), self._p(pre + "mlp.lin1.bias")
            b.fc2_w, b.fc2_b = self._p(pre + "mlp.lin2.weight"), self._p(pre + "mlp.lin2.bias")
            b.freqs = self._p(pre + "attn.freqs_cis")
        pre = neck_prefix  # the tracker's neck, or "neck.det." for the detector's (same graph)
        names = {0: ("0.dconv_2x2_0", "0.dconv_2x2_1"), 1: ("1.dconv_2x2", None), 2: (None, None), 3: (None, None)}
        for s in range(4):
            nw = w.neck[s]
            d1, d2 = names[s]
            if d1:
                nw.dc1_w, nw.dc1_b = self._p(pre + d1 + ".weight"), self._p(pre + d1 + ".bias")
            if d2:
                nw.dc2_w, nw.dc2_b = self._p(pre + d2 + ".weight"), self._p(pre + d2 + ".bias")
            nw.c1_w, nw.c1_b = self._p(pre + f"{s}.conv_1x1.weight"), self._p(pre + f"{s}.conv_1x1.bias")
            nw.c3_w, nw.c3_b = self._p(pre + f"{s}.conv_3x3.weight"), self._p(pre + f"{s}.conv_3x3.bias")
        self.w = w

    def _p(self, name):
        arr = self.t[name][1]
        if self.t[name][0] == F32:
            arr = np.ascontiguousarray(arr, dtype=np.float32)
        else:
            arr = np.ascontiguousarray(arr)
        self._keep.append(arr)
        return arr.ctypes.data

    def preprocess(self, rgb: np.ndarray) -> np.ndarray:
        rgb = np.ascontiguousarray(rgb, dtype=np.uint8)
        S = self.hp["img"]
        out = np.empty((3, S, S), np.float32)
        _vit_lib().orc_preprocess_sam3(rgb.ctypes.data, rgb.shape[1], rgb.shape[0], S, out.ctypes.data)
        return out

    def preprocess_sam2(self, rgb: np.ndarray, img: int) -> np.ndarray:
        return preprocess_sam2(rgb, img)

    def prefix(self, img_chw: np.ndarray) -> np.ndarray:
        img_chw = np.ascontiguousarray(img_chw, dtype=np.float32)
        x = np.empty((self.G * self.G, self.hp["embed"]), np.float32)
        _vit_lib().orc_vit_prefix(ctypes.byref(self.h), ctypes.byref(self.w), img_chw.ctypes.data, x.ctypes.data,
                                  self.nt)
        return x

    def block(self, i: int, x: np.ndarray) -> np.ndarray:
        x = np.array(x, dtype=np.float32, copy=True, order="C")
        _vit_lib().orc_vit_block(ctypes.byref(self.h), ctypes.byref(self.w.blocks[i]), i, x.ctypes.data, self.nt)
        return x

    def neck(self, x: np.ndarray) -> list:
        x = np.ascontiguousarray(x, dtype=np.float32)
        D, G = self.hp["neck_dim"], self.G
        outs = [np.empty((s, s, D), np.float32) for s in (4 * G, 2 * G, G, G // 2)]
        ptrs = (ctypes.c_void_p * 4)(*[o.ctypes.data for o in outs])
        _vit_lib().orc_neck(ctypes.byref(self.h), ctypes.byref(self.w.neck), x.ctypes.data, ptrs, self.nt)
        return outs

    def encode(self, rgb: np.ndarray, depth: int | None = None, attn_f64: bool = False) -> tuple:
        """The whole encode.  attn_f64: attention in float64 instead of float32 -- a
        second, equally valid evaluation of the same graph (the tests measure the
        distance between the two)."""
        _vit_lib().orc_set_attention_f64(1 if attn_f64 else 0)
        try:
            x = self.prefix(self.preprocess(rgb))
            for i in range(self.hp["depth"] if depth is None else depth):
                x = self.block(i, x)
            return x, self.neck(x)
        finally:
            _vit_lib().orc_set_attention_f64(0)
