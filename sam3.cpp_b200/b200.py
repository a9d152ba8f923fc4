"""Python front end of libsam3_b200.so (the C ABI in include/sam3_b200.h).

Thin ctypes bindings plus numpy conveniences used by the tests and by
bench.py.  Every compute call goes to the CUDA library; there is no CPU
path here, and loading fails loudly when the library is missing.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "libsam3_b200.so")
HEADER = os.path.join(os.path.dirname(PKG_DIR), "include", "sam3_b200.h")

STATUS_ALLOC_FAILED, STATUS_FAILED, STATUS_SUCCESS, STATUS_ABORTED = -2, -1, 0, 1
TYPE_F32, TYPE_F16, TYPE_Q4_0, TYPE_Q4_1, TYPE_Q8_0 = 0, 1, 2, 3, 8
MMQ_AUTO, MMQ_TC, MMQ_SIMT = 0, 1, 2
ARITH_EXACT, ARITH_DQ16 = 0, 1
TYPE_I32 = 26
(OP_NONE, OP_VIEW, OP_MUL_MAT, OP_ADD, OP_FLASH_ATTN_EXT, OP_CONV_TRANSPOSE_2D, OP_CONV_2D, OP_GET_ROWS,
 OP_CONT, OP_MUL, OP_SCALE, OP_UNARY, OP_NORM, OP_SOFT_MAX, OP_WIN_PART, OP_WIN_UNPART, OP_SUB, OP_REPEAT,
 OP_CONCAT, OP_IM2COL, OP_POOL_2D, OP_PAD, OP_UPSCALE, OP_CONV_2D_DW, OP_GROUP_NORM) = range(25)
UNARY_RELU, UNARY_SIGMOID, UNARY_GELU_ERF, UNARY_GELU = 1, 2, 3, 4
TENSOR_FLAG_OUTPUT = 2

_lib = None


class GraphTensor(ctypes.Structure):
    """sam3b200_tensor (include/sam3_b200.h): one ggml graph node flattened to plain C."""


GraphTensor._fields_ = [
    ("type", ctypes.c_int32),
    ("op", ctypes.c_int32),
    ("ne", ctypes.c_int64 * 4),
    ("nb", ctypes.c_size_t * 4),
    ("op_params", ctypes.c_int32 * 16),
    ("flags", ctypes.c_int32),
    ("src", ctypes.POINTER(GraphTensor) * 4),
    ("data", ctypes.c_void_p),
    ("extra", ctypes.c_void_p),
]

# bytes per block and elements per block (ggml type traits)
_BLOCK = {TYPE_F32: (4, 1), TYPE_F16: (2, 1), TYPE_I32: (4, 1), TYPE_Q4_0: (18, 32), TYPE_Q4_1: (20, 32),
          TYPE_Q8_0: (34, 32)}


def graph_tensor(ttype: int, ne, op: int = OP_NONE, src=(), data: int | None = None, nb=None, op_params=(),
                 flags: int = 0, extra: int | None = None) -> GraphTensor:
    """A graph node with ggml's packed strides unless `nb` (bytes) is given.  The node keeps references to
    its sources so their structures stay alive as long as it does."""
    ne = list(ne) + [1] * (4 - len(ne))
    t = GraphTensor()
    t.type, t.op, t.flags = ttype, op, flags
    if nb is None:
        bb, be = _BLOCK[ttype]
        nb = [bb, bb * (ne[0] // be)]
        nb += [nb[1] * ne[1], nb[1] * ne[1] * ne[2]]
    for d in range(4):
        t.ne[d], t.nb[d] = ne[d], nb[d]
    for i, v in enumerate(op_params):
        t.op_params[i] = v
    for i, s in enumerate(src):
        if s is not None:
            t.src[i] = ctypes.pointer(s)
    t.data, t.extra = data, extra
    t._keep = list(src)
    return t


def f32_bits(x: float) -> int:
    """An f32 op parameter as the int32 word ggml stores it in op_params."""
    return int(np.array([x], np.float32).view(np.int32)[0])


def supports_op(node: GraphTensor) -> bool:
    """sam3b200_supports_op: whether the backend executes this node (host-only check)."""
    return bool(lib().sam3b200_supports_op(node))


class MemPromptHparams(ctypes.Structure):
    """sam3b200_mem_prompt_hparams (include/sam3_b200.h)."""
    _fields_ = [("d_model", ctypes.c_int32), ("mem_dim", ctypes.c_int32), ("num_maskmem", ctypes.c_int32),
                ("max_obj_ptrs", ctypes.c_int32)]


def select_memory_frames(bank_size: int, max_slots: int) -> list[int]:
    """sam3b200_select_memory_frames: the memory-bank slots one propagated frame attends to."""
    cap = max(bank_size, max_slots, 2)
    out = (ctypes.c_int32 * cap)()
    n = lib().sam3b200_select_memory_frames(bank_size, max_slots, out, cap)
    if n < 0:
        raise B200Error(f"select_memory_frames failed: {last_error()}")
    return list(out[:n])


def build_mem_prompt(hp: dict, slot_feats, slot_pes, slot_is_cond, obj_ptrs, ptr_frames, cur_frame: int,
                     tpos_enc=None, tpos_proj_w=None, tpos_proj_b=None):
    """sam3b200_build_mem_prompt on host arrays: returns (prompt [M][MD], prompt_pos [M][MD],
    n_ptr_tokens), the inputs of MemAttention.run.  hp: d_model, mem_dim, num_maskmem, max_obj_ptrs."""
    h = MemPromptHparams(hp["d_model"], hp["mem_dim"], hp["num_maskmem"], hp["max_obj_ptrs"])
    f32 = lambda a: None if a is None else np.ascontiguousarray(a, dtype=np.float32)
    feats, pes, ptrs = [f32(a) for a in slot_feats], [f32(a) for a in slot_pes], [f32(a) for a in obj_ptrs]
    n_slots, n_ptrs = len(feats), len(ptrs)
    slot_tokens = feats[0].size // hp["mem_dim"] if n_slots else 0
    ptr_arr = lambda arrs: (ctypes.c_void_p * max(len(arrs), 1))(*[a.ctypes.data for a in arrs])
    cond = np.ascontiguousarray(slot_is_cond, dtype=np.int32).reshape(-1)
    frames = np.ascontiguousarray(ptr_frames, dtype=np.int32).reshape(-1)
    te, w, b = f32(tpos_enc), f32(tpos_proj_w), f32(tpos_proj_b)
    split = hp["d_model"] // hp["mem_dim"]
    cap = n_slots * slot_tokens + min(n_ptrs, hp["max_obj_ptrs"]) * split
    prompt = np.empty((max(cap, 1), hp["mem_dim"]), np.float32)
    pos = np.empty_like(prompt)
    n_ptr_tokens = ctypes.c_int32()
    data = lambda a: None if a is None else a.ctypes.data
    m = lib().sam3b200_build_mem_prompt(ctypes.byref(h), n_slots, slot_tokens, ptr_arr(feats), ptr_arr(pes),
                                        cond.ctypes.data, n_ptrs, ptr_arr(ptrs), frames.ctypes.data, cur_frame,
                                        data(te), data(w), data(b), prompt.ctypes.data, pos.ctypes.data, cap,
                                        ctypes.byref(n_ptr_tokens))
    if m < 0:
        raise B200Error(f"build_mem_prompt failed: {last_error()}")
    return prompt[:m], pos[:m], n_ptr_tokens.value


def extract_obj_ptr(sam_token, obj_score: float, w, b, no_obj_ptr, blend: bool = False) -> np.ndarray:
    """sam3b200_extract_obj_ptr: the object pointer of a decoded frame (w: three f32 [D][D] layers
    [out][in], b: three f32 [D])."""
    f32 = lambda a: np.ascontiguousarray(a, dtype=np.float32)
    tok, nop = f32(sam_token).reshape(-1), f32(no_obj_ptr).reshape(-1)
    ws, bs = [f32(x) for x in w], [f32(x) for x in b]
    arr = lambda arrs: (ctypes.c_void_p * 3)(*[a.ctypes.data for a in arrs])
    out = np.empty(tok.size, np.float32)
    _check(lib().sam3b200_extract_obj_ptr(tok.size, 1 if blend else 0, tok.ctypes.data, obj_score, arr(ws),
                                          arr(bs), nop.ctypes.data, out.ctypes.data), "extract_obj_ptr")
    return out


def axial_cis(dim: int, end_x: int, end_y: int, theta: float = 10000.0, scale_pos: float = 1.0) -> np.ndarray:
    """sam3b200_axial_cis: [end_x*end_y][dim/2][2] float32 (cos, sin)."""
    out = np.empty((end_x * end_y, dim // 2, 2), np.float32)
    _check(lib().sam3b200_axial_cis(dim, end_x, end_y, theta, scale_pos, out.ctypes.data), "axial_cis")
    return out


def sinusoidal_pe_2d(H: int, W: int, d_model: int) -> np.ndarray:
    """sam3b200_sinusoidal_pe_2d: [H][W][d_model] float32."""
    out = np.empty((H, W, d_model), np.float32)
    _check(lib().sam3b200_sinusoidal_pe_2d(H, W, d_model, out.ctypes.data), "sinusoidal_pe_2d")
    return out


class MemBank:
    """sam3b200_mem_bank: the host-side memory of one tracked object (slots + object pointers)."""

    def __init__(self, hp: dict, feat_size: int):
        self.hp, self.H = hp, feat_size
        h = MemPromptHparams(hp["d_model"], hp["mem_dim"], hp["num_maskmem"], hp["max_obj_ptrs"])
        self.h = lib().sam3b200_mem_bank_create(ctypes.byref(h), feat_size)
        if not self.h:
            raise B200Error(f"mem_bank_create failed: {last_error()}")

    def add_slot(self, feats: np.ndarray, frame: int, is_cond: bool) -> None:
        f = np.ascontiguousarray(feats, dtype=np.float32)
        assert f.size == self.H * self.H * self.hp["mem_dim"]
        _check(lib().sam3b200_mem_bank_add_slot(self.h, f.ctypes.data, frame, 1 if is_cond else 0), "add_slot")

    def add_ptr(self, ptr: np.ndarray, frame: int) -> None:
        p = np.ascontiguousarray(ptr, dtype=np.float32)
        assert p.size == self.hp["d_model"]
        _check(lib().sam3b200_mem_bank_add_ptr(self.h, p.ctypes.data, frame), "add_ptr")

    def state(self):
        """([(slot frame, is_cond)], [pointer frame])."""
        cap = self.hp["num_maskmem"] + self.hp["max_obj_ptrs"] + 2
        sf, sc, pf = (np.zeros(cap, np.int32) for _ in range(3))
        n_ptrs = ctypes.c_int32()
        ns = lib().sam3b200_mem_bank_state(self.h, sf.ctypes.data, sc.ctypes.data, cap, pf.ctypes.data, cap,
                                           ctypes.byref(n_ptrs))
        if ns < 0:
            raise B200Error(f"mem_bank_state failed: {last_error()}")
        return [(int(sf[i]), bool(sc[i])) for i in range(ns)], [int(x) for x in pf[:n_ptrs.value]]

    def prompt(self, cur_frame: int, tpos_enc=None, tpos_proj_w=None, tpos_proj_b=None):
        """(prompt [M][MD], prompt_pos [M][MD], n_ptr_tokens) for the frame cur_frame."""
        f32 = lambda a: None if a is None else np.ascontiguousarray(a, dtype=np.float32)
        te, w, b = f32(tpos_enc), f32(tpos_proj_w), f32(tpos_proj_b)
        cap = self.hp["num_maskmem"] * self.H * self.H + self.hp["max_obj_ptrs"] * (
            self.hp["d_model"] // self.hp["mem_dim"])
        prompt = np.empty((max(cap, 1), self.hp["mem_dim"]), np.float32)
        pos = np.empty_like(prompt)
        n = ctypes.c_int32()
        data = lambda a: None if a is None else a.ctypes.data
        m = lib().sam3b200_mem_bank_prompt(self.h, cur_frame, data(te), data(w), data(b), prompt.ctypes.data,
                                           pos.ctypes.data, cap, ctypes.byref(n))
        if m < 0:
            raise B200Error(f"mem_bank_prompt failed: {last_error()}")
        return prompt[:m], pos[:m], n.value

    def rope(self):
        """(rope_q [H*H][D/2][2], rope_k [slots*H*H][D/2][2] or None) for the bank's current prompt."""
        D, HH = self.hp["d_model"], self.H * self.H
        rq = np.empty((HH, D // 2, 2), np.float32)
        rk = np.empty((self.hp["num_maskmem"] * HH, D // 2, 2), np.float32)
        m = lib().sam3b200_mem_bank_rope(self.h, rq.ctypes.data, rk.ctypes.data, rk.shape[0])
        if m < 0:
            raise B200Error(f"mem_bank_rope failed: {last_error()}")
        return rq, (rk[:m] if m else None)

    def free(self) -> None:
        if self.h:
            lib().sam3b200_mem_bank_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def graph_compute_status(be_handle, nodes) -> int:
    """sam3b200_graph_compute on a list of GraphTensor nodes; returns the ggml_status."""
    arr = (ctypes.POINTER(GraphTensor) * max(len(nodes), 1))(*[ctypes.pointer(n) for n in nodes])
    return lib().sam3b200_graph_compute(be_handle, arr, len(nodes))


class B200Error(RuntimeError):
    pass


def build() -> None:
    """Compile libsam3_b200.so in-tree (nvcc, sm_100a)."""
    subprocess.run(["make", "-s", "-j8", "-C", PKG_DIR], check=True)


def exported_symbols() -> list[str]:
    """Function names declared in include/sam3_b200.h."""
    import re
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"\b(sam3b200_[a-z0-9_]+)\s*\(", txt)))


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise B200Error(f"{LIB_PATH} is missing: build it with `make -C {PKG_DIR}` (nvcc, sm_100a)")
    L = ctypes.CDLL(LIB_PATH)
    vp, i64, i32, sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t
    sig = {
        "sam3b200_backend_init": (vp, [i32]),
        "sam3b200_backend_free": (None, [vp]),
        "sam3b200_backend_name": (ctypes.c_char_p, [vp]),
        "sam3b200_backend_synchronize": (i32, [vp]),
        "sam3b200_backend_stream": (vp, [vp]),
        "sam3b200_debug_wait_timeout": (i32, [vp, ctypes.c_uint64]),
        "sam3b200_last_error": (ctypes.c_char_p, []),
        "sam3b200_buffer_alloc": (vp, [vp, sz]),
        "sam3b200_buffer_free": (None, [vp, vp]),
        "sam3b200_tensor_set": (i32, [vp, vp, vp, sz, sz]),
        "sam3b200_tensor_get": (i32, [vp, vp, vp, sz, sz]),
        "sam3b200_weight_upload": (vp, [vp, i32, vp, i64, i64]),
        "sam3b200_weight_free": (None, [vp, vp]),
        "sam3b200_mul_mat": (i32, [vp, vp, vp, i64, i64, vp, vp, i64]),
        "sam3b200_mul_mat_block_dots": (i32, [vp, vp, vp, i64, vp]),
        "sam3b200_mul_mat_noalloc": (i32, [vp, vp, vp, i64, i64, vp, vp, i64]),
        "sam3b200_set_mmq_impl": (i32, [vp, i32]),
        "sam3b200_set_arith": (i32, [vp, i32]),
        "sam3b200_mul_mat_dq16": (i32, [vp, vp, vp, i64, i64, vp, vp, i64]),
        "sam3b200_vit_create": (vp, [vp, vp]),
        "sam3b200_vit_free": (None, [vp]),
        "sam3b200_vit_set_tensor": (i32, [vp, ctypes.c_char_p, i32, vp, vp]),
        "sam3b200_vit_missing": (i32, [vp, ctypes.c_char_p, i32]),
        "sam3b200_encode_image": (i32, [vp, vp, i32, i32, vp]),
        "sam3b200_encode_image_device": (i32, [vp, vp, i32, i32]),
        "sam3b200_encode_images": (i32, [vp, i32, vp, i32, i32, vp]),
        "sam3b200_encode_images_device": (i32, [vp, i32, vp, i32, i32]),
        "sam3b200_vit_output": (i32, [vp, i32, ctypes.POINTER(ctypes.c_void_p), vp]),
        "sam3b200_vit_run_prefix": (i32, [vp, vp, vp]),
        "sam3b200_vit_run_block": (i32, [vp, i32, vp]),
        "sam3b200_vit_run_neck": (i32, [vp, vp]),
        "sam3b200_preprocess": (i32, [vp, vp, i32, i32, i32, vp]),
        "sam3b200_preprocess_sam2": (i32, [vp, vp, i32, i32, i32, vp]),
        "sam3b200_flash_attn_ext": (i32, [vp, vp, vp, vp, i64, i64, i64, i64, ctypes.c_float, vp]),
        "sam3b200_flash_attn_ext_view": (i32, [vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, i64, vp, vp, vp,
                                                ctypes.c_float, vp]),
        "sam3b200_conv_transpose_2d": (i32, [vp, vp, vp, i64, i64, i64, i64, i64, i64, i32, vp]),
        "sam3b200_conv_2d": (i32, [vp, vp, vp, i64, i64, i64, i64, i64, i64, i32, i32, i32, i32, i32, i32, vp]),
        "sam3b200_get_rows": (i32, [vp, i32, vp, i64, i64, vp, i64, vp]),
        "sam3b200_supports_op": (i32, [ctypes.POINTER(GraphTensor)]),
        "sam3b200_select_memory_frames": (i32, [i32, i32, vp, i32]),
        "sam3b200_extract_obj_ptr": (i32, [i32, i32, vp, ctypes.c_float, vp, vp, vp, vp]),
        "sam3b200_sinusoidal_pe_2d": (i32, [i32, i32, i32, vp]),
        "sam3b200_mem_bank_create": (vp, [vp, i32]),
        "sam3b200_mem_bank_free": (None, [vp]),
        "sam3b200_mem_bank_add_slot": (i32, [vp, vp, i32, i32]),
        "sam3b200_mem_bank_add_ptr": (i32, [vp, vp, i32]),
        "sam3b200_mem_bank_state": (i32, [vp, vp, vp, i32, vp, i32, vp]),
        "sam3b200_mem_bank_prompt": (i64, [vp, i32, vp, vp, vp, vp, vp, i64, vp]),
        "sam3b200_axial_cis": (i32, [i32, i32, i32, ctypes.c_float, ctypes.c_float, vp]),
        "sam3b200_mem_bank_rope": (i64, [vp, vp, vp, i64]),
        "sam3b200_build_mem_prompt": (i64, [vp, i32, i32, vp, vp, vp, i32, vp, vp, i32, vp, vp, vp, vp, vp, i64,
                                            vp]),
        "sam3b200_graph_compute": (i32, [vp, ctypes.POINTER(ctypes.POINTER(GraphTensor)), i32]),
        "sam3b200_sam_dec_create": (vp, [vp, vp]),
        "sam3b200_sam_dec_free": (None, [vp]),
        "sam3b200_sam_dec_set_tensor": (i32, [vp, ctypes.c_char_p, i32, vp, vp]),
        "sam3b200_sam_dec_missing": (i32, [vp, ctypes.c_char_p, i32]),
        "sam3b200_sam_dec_run": (i32, [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32]),
        "sam3b200_sam_dec_outputs": (i32, [vp, ctypes.POINTER(ctypes.c_void_p), vp, vp,
                                           ctypes.POINTER(ctypes.c_void_p)]),
        "sam3b200_sam_dec_mask": (i32, [vp, i32, i32, i32, vp]),
        "sam3b200_sam_dec_run_tracking": (i32, [vp, vp, vp, vp]),
        "sam3b200_sam_dec_mask_token": (i32, [vp, i32, ctypes.POINTER(ctypes.c_void_p)]),
        "sam3b200_tracker_create": (vp, [vp, vp, vp, vp, vp, vp]),
        "sam3b200_tracker_free": (None, [vp]),
        "sam3b200_tracker_set_tensor": (i32, [vp, ctypes.c_char_p, i32, vp, vp]),
        "sam3b200_tracker_encode": (i32, [vp, vp]),
        "sam3b200_tracker_add_instance": (i32, [vp, vp, vp, i32, i32, i32]),
        "sam3b200_tracker_propagate": (i32, [vp]),
        "sam3b200_tracker_encode_image": (i32, [vp, vp, i32, i32]),
        "sam3b200_tracker_reset": (None, [vp]),
        "sam3b200_tracker_frame_index": (i32, [vp]),
        "sam3b200_tracker_instances": (i32, [vp, vp, i32]),
        "sam3b200_tracker_instance": (i32, [vp, i32, ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p),
                                            vp, vp, vp]),
        "sam3b200_tracker_mask": (i32, [vp, i32, i32, i32, vp]),
        "sam3b200_tracker_bank": (i32, [vp, i32, vp, vp, vp, i32, vp, vp, i32, vp]),
        "sam3b200_tracker_prompt": (i32, [vp, ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p)]),
        "sam3b200_tensor_memset": (i32, [vp, vp, i32, ctypes.c_size_t, ctypes.c_size_t]),
        "sam3b200_device_memory": (i32, [i32, vp, vp]),
        "sam3b200_device_count": (i32, [vp]),
        "sam3b200_text_create": (vp, [vp, vp]),
        "sam3b200_text_free": (None, [vp]),
        "sam3b200_text_set_tensor": (i32, [vp, ctypes.c_char_p, i32, vp, vp]),
        "sam3b200_text_missing": (i32, [vp, ctypes.c_char_p, i32]),
        "sam3b200_text_encode": (i32, [vp, vp, i32]),
        "sam3b200_text_output": (i32, [vp, ctypes.POINTER(ctypes.c_void_p), vp]),
        "sam3b200_mem_attn_create": (vp, [vp, vp]),
        "sam3b200_mem_attn_free": (None, [vp]),
        "sam3b200_mem_attn_set_tensor": (i32, [vp, ctypes.c_char_p, i32, vp, vp]),
        "sam3b200_mem_attn_missing": (i32, [vp, ctypes.c_char_p, i32]),
        "sam3b200_mem_attn_run": (i32, [vp, vp, vp, vp, vp, vp, vp, i32, i32, i32]),
        "sam3b200_mem_attn_run_device": (i32, [vp, vp, vp, vp, vp, vp, vp, i32, i32, i32]),
        "sam3b200_mem_attn_output": (i32, [vp, ctypes.POINTER(ctypes.c_void_p)]),
        "sam3b200_mem_enc_create": (vp, [vp, vp]),
        "sam3b200_mem_enc_free": (None, [vp]),
        "sam3b200_mem_enc_set_tensor": (i32, [vp, ctypes.c_char_p, i32, vp, vp]),
        "sam3b200_mem_enc_missing": (i32, [vp, ctypes.c_char_p, i32]),
        "sam3b200_mem_enc_run": (i32, [vp, vp, i32, i32, vp, ctypes.c_float]),
        "sam3b200_mem_enc_run_device": (i32, [vp, vp, i32, i32, vp, ctypes.c_float]),
        "sam3b200_mem_enc_output": (i32, [vp, ctypes.POINTER(ctypes.c_void_p)]),
        "sam3b200_fenc_create": (vp, [vp, vp]),
        "sam3b200_fenc_free": (None, [vp]),
        "sam3b200_fenc_set_tensor": (i32, [vp, ctypes.c_char_p, i32, vp, vp]),
        "sam3b200_fenc_missing": (i32, [vp, ctypes.c_char_p, i32]),
        "sam3b200_fenc_run": (i32, [vp, vp, vp, vp, vp, i32, i32]),
        "sam3b200_fenc_run_device": (i32, [vp, vp, vp, vp, vp, i32, i32]),
        "sam3b200_fenc_output": (i32, [vp, ctypes.POINTER(ctypes.c_void_p)]),
        "sam3b200_ddec_create": (vp, [vp, vp]),
        "sam3b200_ddec_free": (None, [vp]),
        "sam3b200_ddec_set_tensor": (i32, [vp, ctypes.c_char_p, i32, vp, vp]),
        "sam3b200_ddec_missing": (i32, [vp, ctypes.c_char_p, i32]),
        "sam3b200_ddec_run": (i32, [vp, vp, vp, vp, vp, vp, i32]),
        "sam3b200_ddec_run_device": (i32, [vp, vp, vp, vp, vp, vp, i32]),
        "sam3b200_ddec_outputs": (i32, [vp] + [ctypes.POINTER(ctypes.c_void_p)] * 4),
        "sam3b200_seg_create": (vp, [vp, vp]),
        "sam3b200_seg_free": (None, [vp]),
        "sam3b200_seg_set_tensor": (i32, [vp, ctypes.c_char_p, i32, vp, vp]),
        "sam3b200_seg_missing": (i32, [vp, ctypes.c_char_p, i32]),
        "sam3b200_seg_run": (i32, [vp, vp, vp, vp, vp, i32, vp, vp, i32]),
        "sam3b200_seg_run_device": (i32, [vp, vp, vp, vp, vp, i32, vp, vp, i32]),
        "sam3b200_seg_output": (i32, [vp, ctypes.POINTER(ctypes.c_void_p)]),
        "sam3b200_geom_create": (vp, [vp, vp]),
        "sam3b200_geom_free": (None, [vp]),
        "sam3b200_geom_set_tensor": (i32, [vp, ctypes.c_char_p, i32, vp, vp]),
        "sam3b200_geom_missing": (i32, [vp, ctypes.c_char_p, i32]),
        "sam3b200_geom_run": (i32, [vp, vp, i32, vp, vp, i32]),
        "sam3b200_geom_run_device": (i32, [vp, vp, i32, vp, vp, i32]),
        "sam3b200_geom_output": (i32, [vp, ctypes.POINTER(ctypes.c_void_p)]),
        "sam3b200_vit_output_det": (i32, [vp, i32, ctypes.POINTER(ctypes.c_void_p), vp]),
        "sam3b200_file_open": (vp, [ctypes.c_char_p]),
        "sam3b200_file_close": (None, [vp]),
        "sam3b200_file_info": (i32, [vp, vp, vp, vp, vp]),
        "sam3b200_file_hparams": (i32, [vp, vp, i32]),
        "sam3b200_file_tensor": (i32, [vp, i32, ctypes.c_char_p, i32, vp, vp, vp, vp]),
        "sam3b200_file_vit_hparams": (i32, [vp, vp]),
        "sam3b200_file_text_hparams": (i32, [vp, vp]),
        "sam3b200_file_hiera_hparams": (i32, [vp, vp]),
        "sam3b200_file_load": (i32, [vp, vp, vp, vp, vp]),
        "sam3b200_file_skipped": (i32, [vp, ctypes.c_char_p, i32]),
        "sam3b200_hiera_create": (vp, [vp, vp]),
        "sam3b200_hiera_free": (None, [vp]),
        "sam3b200_hiera_set_tensor": (i32, [vp, ctypes.c_char_p, i32, vp, vp]),
        "sam3b200_hiera_missing": (i32, [vp, ctypes.c_char_p, i32]),
        "sam3b200_hiera_block_info": (i32, [vp, i32, vp]),
        "sam3b200_hiera_run_prefix": (i32, [vp, vp, vp]),
        "sam3b200_hiera_run_block": (i32, [vp, i32, vp, i32, i32, vp]),
        "sam3b200_hiera_encode_device": (i32, [vp, vp]),
        "sam3b200_hiera_output": (i32, [vp, i32, ctypes.POINTER(ctypes.c_void_p), vp]),
        "sam3b200_backend_launch_count": (ctypes.c_longlong, [vp]),
        "sam3b200_backend_profile": (i32, [vp, i32]),
        "sam3b200_backend_profile_read": (i32, [vp, i32, ctypes.POINTER(ctypes.c_double),
                                                ctypes.POINTER(ctypes.c_int)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def last_error() -> str:
    return lib().sam3b200_last_error().decode()


def _check(status: int, what: str) -> None:
    if status != STATUS_SUCCESS:
        raise B200Error(f"{what} failed (status {status}): {last_error()}")


class DeviceBuffer:
    """Device allocation owned by a Backend."""

    def __init__(self, be: "Backend", nbytes: int):
        self.be, self.nbytes = be, int(nbytes)
        self.ptr = lib().sam3b200_buffer_alloc(be.h, self.nbytes)
        if not self.ptr:
            raise B200Error(f"buffer_alloc({nbytes}) failed: {last_error()}")

    def set(self, arr: np.ndarray, offset: int = 0) -> None:
        arr = np.ascontiguousarray(arr)
        assert offset + arr.nbytes <= self.nbytes
        _check(lib().sam3b200_tensor_set(self.be.h, self.ptr, arr.ctypes.data, offset, arr.nbytes), "tensor_set")

    def get(self, shape, dtype, offset: int = 0) -> np.ndarray:
        out = np.empty(shape, dtype=dtype)
        assert offset + out.nbytes <= self.nbytes
        _check(lib().sam3b200_tensor_get(self.be.h, self.ptr, out.ctypes.data, offset, out.nbytes), "tensor_get")
        return out

    def free(self) -> None:
        if self.ptr:
            lib().sam3b200_buffer_free(self.be.h, self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Weight:
    def __init__(self, be: "Backend", qtype: int, blocks: np.ndarray, K: int, N: int):
        blocks = np.ascontiguousarray(blocks)
        self.be, self.qtype, self.K, self.N = be, qtype, K, N
        self.h = lib().sam3b200_weight_upload(be.h, qtype, blocks.ctypes.data, K, N)
        if not self.h:
            raise B200Error(f"weight_upload failed: {last_error()}")

    def free(self) -> None:
        if self.h:
            lib().sam3b200_weight_free(self.be.h, self.h)
            self.h = None


class VitHparams(ctypes.Structure):
    """sam3b200_vit_hparams (include/sam3_b200.h)."""
    _fields_ = [("img", ctypes.c_int), ("patch", ctypes.c_int), ("embed", ctypes.c_int), ("depth", ctypes.c_int),
                ("heads", ctypes.c_int), ("mlp", ctypes.c_int), ("window", ctypes.c_int),
                ("n_global", ctypes.c_int), ("global_idx", ctypes.c_int * 4), ("pos_grid", ctypes.c_int),
                ("neck_dim", ctypes.c_int), ("wtype", ctypes.c_int)]

    @classmethod
    def from_dict(cls, d: dict) -> "VitHparams":
        h = cls()
        for k in ("img", "patch", "embed", "depth", "heads", "mlp", "window", "pos_grid", "neck_dim", "wtype"):
            setattr(h, k, int(d[k]))
        g = list(d["global_idx"])
        h.n_global = len(g)
        for i, v in enumerate(g):
            h.global_idx[i] = int(v)
        return h

    def to_dict(self) -> dict:
        d = {k: getattr(self, k) for k in ("img", "patch", "embed", "depth", "heads", "mlp", "window", "pos_grid",
                                           "neck_dim", "wtype")}
        d["global_idx"] = tuple(self.global_idx[:self.n_global])
        return d


class Vit:
    """The visual encoder (sam3b200_vit) on a backend."""

    def __init__(self, be: "Backend", hp: dict):
        self.be, self.hp = be, dict(hp)
        self._chp = VitHparams.from_dict(hp)
        self.h = lib().sam3b200_vit_create(be.h, ctypes.byref(self._chp))
        if not self.h:
            raise B200Error(f"vit_create failed: {last_error()}")
        self.G = hp["img"] // hp["patch"]

    def set_tensor(self, name: str, ttype: int, data: np.ndarray, ne) -> None:
        data = np.ascontiguousarray(data)
        ne4 = (ctypes.c_int64 * 4)(*(list(ne) + [1] * (4 - len(ne))))
        _check(lib().sam3b200_vit_set_tensor(self.h, name.encode(), ttype, data.ctypes.data, ne4), f"set {name}")

    def load(self, tensors: dict) -> None:
        """tensors: name -> (ggml type, array, ne)"""
        for name, (t, arr, ne) in tensors.items():
            self.set_tensor(name, t, arr, ne)
        buf = ctypes.create_string_buffer(1 << 16)
        n = lib().sam3b200_vit_missing(self.h, buf, len(buf))
        if n:
            raise B200Error(f"{n} encoder tensors missing: {buf.value.decode()[:200]}")

    def encode(self, rgb: np.ndarray) -> list:
        """sam3b200_encode_image: host uint8 HxWx3 -> four f32 [side, side, neck_dim] maps."""
        rgb = np.ascontiguousarray(rgb, dtype=np.uint8)
        h, w = rgb.shape[:2]
        D = self.hp["neck_dim"]
        outs = [np.empty((s, s, D), np.float32) for s in (4 * self.G, 2 * self.G, self.G, self.G // 2)]
        ptrs = (ctypes.c_void_p * 4)(*[o.ctypes.data for o in outs])
        _check(lib().sam3b200_encode_image(self.h, rgb.ctypes.data, w, h, ptrs), "encode_image")
        return outs

    def encode_device(self, rgb_dev: "DeviceBuffer", w: int, h: int) -> None:
        _check(lib().sam3b200_encode_image_device(self.h, rgb_dev.ptr, w, h), "encode_image_device")

    def encode_batch(self, rgbs) -> list:
        """sam3b200_encode_images: n host uint8 HxWx3 images (same size) -> per image four neck maps."""
        rgbs = [np.ascontiguousarray(r, dtype=np.uint8) for r in rgbs]
        h, w = rgbs[0].shape[:2]
        D = self.hp["neck_dim"]
        outs = [[np.empty((s, s, D), np.float32) for s in (4 * self.G, 2 * self.G, self.G, self.G // 2)]
                for _ in rgbs]
        srcs = (ctypes.c_void_p * len(rgbs))(*[r.ctypes.data for r in rgbs])
        ptrs = (ctypes.c_void_p * (4 * len(rgbs)))(*[o.ctypes.data for os_ in outs for o in os_])
        _check(lib().sam3b200_encode_images(self.h, len(rgbs), srcs, w, h, ptrs), "encode_images")
        return outs

    def encode_batch_device(self, rgb_devs, w: int, h: int) -> None:
        """sam3b200_encode_images_device: n device images, one batched pass through the blocks."""
        srcs = (ctypes.c_void_p * len(rgb_devs))(*[d.ptr for d in rgb_devs])
        _check(lib().sam3b200_encode_images_device(self.h, len(rgb_devs), srcs, w, h), "encode_images_device")

    def output(self, i: int):
        p = ctypes.c_void_p()
        ne = (ctypes.c_int64 * 4)()
        _check(lib().sam3b200_vit_output(self.h, i, ctypes.byref(p), ne), "vit_output")
        return p.value, tuple(ne)

    def output_host(self, i: int) -> np.ndarray:
        ptr, ne = self.output(i)
        self.be.synchronize()
        out = np.empty((ne[2], ne[1], ne[0]), np.float32)
        _check(lib().sam3b200_tensor_get(self.be.h, ptr, out.ctypes.data, 0, out.nbytes), "tensor_get")
        return out

    def output_det_host(self, i: int) -> np.ndarray:
        """Detector-neck level i (full SAM3 models): f32 [side, side, neck_dim]."""
        p = ctypes.c_void_p()
        ne = (ctypes.c_int64 * 4)()
        _check(lib().sam3b200_vit_output_det(self.h, i, ctypes.byref(p), ne), "vit_output_det")
        self.be.synchronize()
        out = np.empty((ne[2], ne[1], ne[0]), np.float32)
        _check(lib().sam3b200_tensor_get(self.be.h, p.value, out.ctypes.data, 0, out.nbytes), "tensor_get")
        return out

    def run_prefix(self, img_chw: "DeviceBuffer", x: "DeviceBuffer") -> None:
        _check(lib().sam3b200_vit_run_prefix(self.h, img_chw.ptr, x.ptr), "run_prefix")

    def run_block(self, idx: int, x: "DeviceBuffer") -> None:
        _check(lib().sam3b200_vit_run_block(self.h, idx, x.ptr), "run_block")

    def run_neck(self, x: "DeviceBuffer") -> None:
        _check(lib().sam3b200_vit_run_neck(self.h, x.ptr), "run_neck")

    def free(self) -> None:
        if self.h:
            lib().sam3b200_vit_free(self.h)
            self.h = None


class HieraHparams(ctypes.Structure):
    """sam3b200_hiera_hparams (include/sam3_b200.h)."""
    _fields_ = [("img", ctypes.c_int32), ("embed", ctypes.c_int32), ("heads", ctypes.c_int32),
                ("stages", ctypes.c_int32 * 4), ("q_pool", ctypes.c_int32), ("window_spec", ctypes.c_int32 * 4),
                ("n_global", ctypes.c_int32), ("global_idx", ctypes.c_int32 * 8), ("bkg_h", ctypes.c_int32),
                ("bkg_w", ctypes.c_int32), ("neck_dim", ctypes.c_int32), ("fpn_top_down_n", ctypes.c_int32),
                ("fpn_top_down_levels", ctypes.c_int32 * 4), ("scalp", ctypes.c_int32)]

    @classmethod
    def from_dict(cls, d: dict) -> "HieraHparams":
        h = cls()
        for k in ("img", "embed", "heads", "q_pool", "bkg_h", "bkg_w", "neck_dim", "scalp"):
            setattr(h, k, int(d[k]))
        for k in ("stages", "window_spec"):
            for i, v in enumerate(d[k]):
                getattr(h, k)[i] = int(v)
        h.n_global = len(d["global_idx"])
        for i, v in enumerate(d["global_idx"]):
            h.global_idx[i] = int(v)
        h.fpn_top_down_n = len(d["fpn_top_down_levels"])
        for i, v in enumerate(d["fpn_top_down_levels"]):
            h.fpn_top_down_levels[i] = int(v)
        return h


class Hiera:
    """The SAM2 Hiera image encoder (sam3b200_hiera) on a backend."""

    def __init__(self, be: "Backend", hp: dict):
        self.be, self.hp = be, dict(hp)
        self._chp = HieraHparams.from_dict(hp)
        self.h = lib().sam3b200_hiera_create(be.h, ctypes.byref(self._chp))
        if not self.h:
            raise B200Error(f"hiera_create failed: {last_error()}")

    def set_tensor(self, name: str, ttype: int, data: np.ndarray, ne) -> None:
        data = np.ascontiguousarray(data)
        ne4 = (ctypes.c_int64 * 4)(*(list(ne) + [1] * (4 - len(ne))))
        _check(lib().sam3b200_hiera_set_tensor(self.h, name.encode(), ttype, data.ctypes.data, ne4), f"set {name}")

    def load(self, tensors: dict) -> None:
        """tensors: name -> (ggml type, array, ne)"""
        for name, (t, arr, ne) in tensors.items():
            self.set_tensor(name, t, arr, ne)
        buf = ctypes.create_string_buffer(1 << 16)
        n = lib().sam3b200_hiera_missing(self.h, buf, len(buf))
        if n:
            raise B200Error(f"{n} hiera tensors missing: {buf.value.decode()[:200]}")

    def block_info(self, i: int) -> tuple:
        info = (ctypes.c_int32 * 5)()
        _check(lib().sam3b200_hiera_block_info(self.h, i, info), "hiera_block_info")
        return tuple(info)

    def run_prefix(self, img_chw: "DeviceBuffer", x: "DeviceBuffer") -> None:
        _check(lib().sam3b200_hiera_run_prefix(self.h, img_chw.ptr, x.ptr), "hiera_run_prefix")

    def run_block(self, i: int, x: "DeviceBuffer", H: int, W: int, out: "DeviceBuffer") -> None:
        _check(lib().sam3b200_hiera_run_block(self.h, i, x.ptr, H, W, out.ptr), "hiera_run_block")

    def encode_device(self, img_chw: "DeviceBuffer") -> None:
        _check(lib().sam3b200_hiera_encode_device(self.h, img_chw.ptr), "hiera_encode_device")

    def output_ptr(self, i: int) -> int:
        """Device address of output i (0..3 FPN levels, 4..7 stage outputs)."""
        p = ctypes.c_void_p()
        ne = (ctypes.c_int64 * 4)()
        _check(lib().sam3b200_hiera_output(self.h, i, ctypes.byref(p), ne), "hiera_output")
        return p.value

    def output_host(self, i: int) -> np.ndarray:
        """i = 0..3 FPN levels, 4..7 stage outputs: f32 [H, W, C]."""
        p = ctypes.c_void_p()
        ne = (ctypes.c_int64 * 4)()
        _check(lib().sam3b200_hiera_output(self.h, i, ctypes.byref(p), ne), "hiera_output")
        self.be.synchronize()
        out = np.empty((ne[2], ne[1], ne[0]), np.float32)
        _check(lib().sam3b200_tensor_get(self.be.h, p.value, out.ctypes.data, 0, out.nbytes), "tensor_get")
        return out

    def free(self) -> None:
        if self.h:
            lib().sam3b200_hiera_free(self.h)
            self.h = None


class SamDecHparams(ctypes.Structure):
    """sam3b200_sam_dec_hparams (include/sam3_b200.h)."""
    _fields_ = [(k, ctypes.c_int32) for k in ("feat_size", "embed", "depth", "heads", "mlp_dim", "n_multimask",
                                              "pred_obj_scores", "max_points")]


class SamDecoder:
    """SAM prompt encoder + mask decoder (sam3b200_sam_dec) on a backend."""

    def __init__(self, be: "Backend", hp: dict):
        self.be, self.hp = be, dict(hp)
        self._chp = SamDecHparams(*[int(hp[k]) for k, _ in SamDecHparams._fields_])
        self.h = lib().sam3b200_sam_dec_create(be.h, ctypes.byref(self._chp))
        if not self.h:
            raise B200Error(f"sam_dec_create failed: {last_error()}")

    def set_tensor(self, name: str, ttype: int, data: np.ndarray, ne) -> None:
        data = np.ascontiguousarray(data)
        ne4 = (ctypes.c_int64 * 4)(*(list(ne) + [1] * (4 - len(ne))))
        _check(lib().sam3b200_sam_dec_set_tensor(self.h, name.encode(), ttype, data.ctypes.data, ne4), f"set {name}")

    def load(self, tensors: dict) -> None:
        for name, (t, arr, ne) in tensors.items():
            self.set_tensor(name, t, arr, ne)
        buf = ctypes.create_string_buffer(1 << 16)
        n = lib().sam3b200_sam_dec_missing(self.h, buf, len(buf))
        if n:
            raise B200Error(f"{n} decoder tensors missing: {buf.value.decode()[:300]}")

    def run(self, img_feats: int, feat_s0: int, feat_s1: int, coords, labels, orig_w: int, orig_h: int,
            img_size: int) -> None:
        """Device addresses of the three feature maps; prompts in original-image pixels."""
        c = np.ascontiguousarray(coords, np.float32).reshape(-1)
        lab = np.ascontiguousarray(labels, np.int32)
        _check(lib().sam3b200_sam_dec_run(self.h, img_feats, feat_s0, feat_s1, c.ctypes.data, lab.ctypes.data,
                                          lab.size, orig_w, orig_h, img_size), "sam_dec_run")

    def outputs(self) -> tuple:
        """(mask logits [n][4H][4H], iou [4], obj logit, sam token [256]) on the host."""
        mp, tp = ctypes.c_void_p(), ctypes.c_void_p()
        iou = (ctypes.c_float * 4)()
        obj = ctypes.c_float()
        _check(lib().sam3b200_sam_dec_outputs(self.h, ctypes.byref(mp), iou, ctypes.byref(obj), ctypes.byref(tp)),
               "sam_dec_outputs")
        S, n = 4 * self.hp["feat_size"], self.hp["n_multimask"] + 1
        masks = np.empty((n, S, S), np.float32)
        tok = np.empty(self.hp["embed"], np.float32)
        _check(lib().sam3b200_tensor_get(self.be.h, mp.value, masks.ctypes.data, 0, masks.nbytes), "tensor_get")
        _check(lib().sam3b200_tensor_get(self.be.h, tp.value, tok.ctypes.data, 0, tok.nbytes), "tensor_get")
        return masks, np.array(iou[:n], np.float32), obj.value, tok

    def run_tracking(self, cond_feats: int, feat_s0: int, feat_s1: int) -> None:
        """A propagated frame's decode: memory-conditioned features, no prompt, no no_mem_embed."""
        _check(lib().sam3b200_sam_dec_run_tracking(self.h, cond_feats, feat_s0, feat_s1), "sam_dec_run_tracking")

    def mask_token(self, m: int) -> np.ndarray:
        p = ctypes.c_void_p()
        _check(lib().sam3b200_sam_dec_mask_token(self.h, m, ctypes.byref(p)), "sam_dec_mask_token")
        tok = np.empty(self.hp["embed"], np.float32)
        _check(lib().sam3b200_tensor_get(self.be.h, p.value, tok.ctypes.data, 0, tok.nbytes), "tensor_get")
        return tok

    def mask(self, m: int, out_w: int, out_h: int) -> np.ndarray:
        buf = DeviceBuffer(self.be, out_w * out_h)
        _check(lib().sam3b200_sam_dec_mask(self.h, m, out_w, out_h, buf.ptr), "sam_dec_mask")
        self.be.synchronize()
        return buf.get((out_h, out_w), np.uint8)

    def free(self) -> None:
        if self.h:
            lib().sam3b200_sam_dec_free(self.h)
            self.h = None


class TextEncoder:
    """The SAM3 text encoder (sam3b200_text) on a backend."""

    FIELDS = ("width", "heads", "layers", "ctx_len", "vocab", "out_dim")

    def __init__(self, be: "Backend", hp: dict):
        self.be, self.hp = be, dict(hp)
        self._chp = (ctypes.c_int32 * 6)(*[int(hp[k]) for k in self.FIELDS])
        self.h = lib().sam3b200_text_create(be.h, ctypes.byref(self._chp))
        if not self.h:
            raise B200Error(f"text_create failed: {last_error()}")

    def load(self, tensors: dict) -> None:
        for name, (t, arr, ne) in tensors.items():
            arr = np.ascontiguousarray(arr)
            ne4 = (ctypes.c_int64 * 4)(*(list(ne) + [1] * (4 - len(ne))))
            _check(lib().sam3b200_text_set_tensor(self.h, name.encode(), t, arr.ctypes.data, ne4), f"set {name}")
        buf = ctypes.create_string_buffer(1 << 16)
        n = lib().sam3b200_text_missing(self.h, buf, len(buf))
        if n:
            raise B200Error(f"{n} text tensors missing: {buf.value.decode()[:300]}")

    def encode(self, ids) -> np.ndarray:
        """Token ids -> f32 [ctx_len][out_dim] text features (host)."""
        ids = np.ascontiguousarray(ids, np.int32)
        _check(lib().sam3b200_text_encode(self.h, ids.ctypes.data, ids.size), "text_encode")
        p = ctypes.c_void_p()
        ne = (ctypes.c_int64 * 2)()
        _check(lib().sam3b200_text_output(self.h, ctypes.byref(p), ne), "text_output")
        self.be.synchronize()
        out = np.empty((ne[1], ne[0]), np.float32)
        _check(lib().sam3b200_tensor_get(self.be.h, p.value, out.ctypes.data, 0, out.nbytes), "tensor_get")
        return out

    def free(self) -> None:
        if self.h:
            lib().sam3b200_text_free(self.h)
            self.h = None


class MemAttention:
    """The tracker's memory attention (sam3b200_mem_attn) on a backend."""

    FIELDS = ("d_model", "mem_dim", "layers", "ffn_dim", "max_tokens", "max_mem_tokens")

    def __init__(self, be: "Backend", hp: dict):
        self.be, self.hp = be, dict(hp)
        self._chp = (ctypes.c_int32 * 6)(*[int(hp[k]) for k in self.FIELDS])
        self.h = lib().sam3b200_mem_attn_create(be.h, ctypes.byref(self._chp))
        if not self.h:
            raise B200Error(f"mem_attn_create failed: {last_error()}")

    def load(self, tensors: dict) -> None:
        """tensors: name -> (ggml type, array, ne)"""
        for name, (t, arr, ne) in tensors.items():
            arr = np.ascontiguousarray(arr)
            ne4 = (ctypes.c_int64 * 4)(*(list(ne) + [1] * (4 - len(ne))))
            _check(lib().sam3b200_mem_attn_set_tensor(self.h, name.encode(), t, arr.ctypes.data, ne4), f"set {name}")
        buf = ctypes.create_string_buffer(1 << 16)
        n = lib().sam3b200_mem_attn_missing(self.h, buf, len(buf))
        if n:
            raise B200Error(f"{n} mem_attn tensors missing: {buf.value.decode()[:300]}")

    def run(self, curr, src_pos, prompt, prompt_pos, rope_q, rope_k, n_obj_ptr_tokens: int) -> np.ndarray:
        """Host f32 inputs (token-major: curr/src_pos [N][D], prompt/prompt_pos [M][MD], rope_q [N][D/2][2],
        rope_k [M - n_obj_ptr_tokens][D/2][2] or None) -> conditioned tokens [N][D] (host)."""
        a = [np.ascontiguousarray(x, np.float32) for x in (curr, src_pos, prompt, prompt_pos, rope_q)]
        rk = None if rope_k is None else np.ascontiguousarray(rope_k, np.float32)
        N, M = a[0].shape[0], a[2].shape[0]
        _check(lib().sam3b200_mem_attn_run(self.h, *[x.ctypes.data for x in a], None if rk is None else rk.ctypes.data,
                                           N, M, n_obj_ptr_tokens), "mem_attn_run")
        p = ctypes.c_void_p()
        _check(lib().sam3b200_mem_attn_output(self.h, ctypes.byref(p)), "mem_attn_output")
        self.be.synchronize()
        out = np.empty((N, self.hp["d_model"]), np.float32)
        _check(lib().sam3b200_tensor_get(self.be.h, p.value, out.ctypes.data, 0, out.nbytes), "tensor_get")
        return out

    def output_host(self, n_tokens: int) -> np.ndarray:
        """The last run's conditioned tokens [n_tokens][d_model] (a run through the device entry included)."""
        p = ctypes.c_void_p()
        _check(lib().sam3b200_mem_attn_output(self.h, ctypes.byref(p)), "mem_attn_output")
        self.be.synchronize()
        out = np.empty((n_tokens, self.hp["d_model"]), np.float32)
        _check(lib().sam3b200_tensor_get(self.be.h, p.value, out.ctypes.data, 0, out.nbytes), "tensor_get")
        return out

    def free(self) -> None:
        if self.h:
            lib().sam3b200_mem_attn_free(self.h)
            self.h = None


class MemEncHparams(ctypes.Structure):
    _fields_ = [("feat", ctypes.c_int32), ("img", ctypes.c_int32), ("d_model", ctypes.c_int32),
                ("mem_dim", ctypes.c_int32), ("fuser_layers", ctypes.c_int32), ("fuser_dim", ctypes.c_int32),
                ("sigmoid_scale", ctypes.c_float), ("sigmoid_bias", ctypes.c_float), ("max_mask", ctypes.c_int32)]


class MemEncoder:
    """The tracker's memory encoder (sam3b200_mem_enc) on a backend."""

    def __init__(self, be: "Backend", hp: dict):
        self.be, self.hp = be, dict(hp)
        self._chp = MemEncHparams(**{k: hp[k] for k, _ in MemEncHparams._fields_})
        self.h = lib().sam3b200_mem_enc_create(be.h, ctypes.byref(self._chp))
        if not self.h:
            raise B200Error(f"mem_enc_create failed: {last_error()}")

    def load(self, tensors: dict) -> None:
        """tensors: name -> (ggml type, array, ne)"""
        for name, (t, arr, ne) in tensors.items():
            arr = np.ascontiguousarray(arr)
            ne4 = (ctypes.c_int64 * 4)(*(list(ne) + [1] * (4 - len(ne))))
            _check(lib().sam3b200_mem_enc_set_tensor(self.h, name.encode(), t, arr.ctypes.data, ne4), f"set {name}")
        buf = ctypes.create_string_buffer(1 << 16)
        n = lib().sam3b200_mem_enc_missing(self.h, buf, len(buf))
        if n:
            raise B200Error(f"{n} mem_enc tensors missing: {buf.value.decode()[:300]}")

    def run(self, mask_logits: np.ndarray, pix_feat: np.ndarray, obj_score: float = 1.0) -> np.ndarray:
        """Host mask logits [mh][mw] and pixel features [H*H][d_model] -> memory features [H*H][mem_dim]."""
        ml = np.ascontiguousarray(mask_logits, np.float32)
        pf = np.ascontiguousarray(pix_feat, np.float32)
        _check(lib().sam3b200_mem_enc_run(self.h, ml.ctypes.data, ml.shape[1], ml.shape[0], pf.ctypes.data,
                                          float(obj_score)), "mem_enc_run")
        p = ctypes.c_void_p()
        _check(lib().sam3b200_mem_enc_output(self.h, ctypes.byref(p)), "mem_enc_output")
        self.be.synchronize()
        H = self.hp["feat"]
        out = np.empty((H * H, self.hp["mem_dim"]), np.float32)
        _check(lib().sam3b200_tensor_get(self.be.h, p.value, out.ctypes.data, 0, out.nbytes), "tensor_get")
        return out

    def free(self) -> None:
        if self.h:
            lib().sam3b200_mem_enc_free(self.h)
            self.h = None


class Tracker:
    """The video tracker's frame loop (sam3b200_tracker) over a Hiera encoder, a SAM decoder, a memory
    attention and a memory encoder of one backend."""

    FIELDS = ("feat", "img", "d_model", "mem_dim", "num_maskmem", "max_obj_ptrs", "multimask_in_sam",
              "multimask_token_for_obj_ptr", "fixed_no_obj_ptr", "max_instances", "max_keep_alive")

    def __init__(self, be: "Backend", hp: dict, enc: "Hiera", dec: "SamDecoder", attn: "MemAttention",
                 menc: "MemEncoder"):
        self.be, self.hp = be, dict(hp)
        self._chp = (ctypes.c_int32 * len(self.FIELDS))(*[int(hp[k]) for k in self.FIELDS])
        self._parts = (enc, dec, attn, menc)
        self.h = lib().sam3b200_tracker_create(be.h, ctypes.byref(self._chp), enc.h, dec.h, attn.h, menc.h)
        if not self.h:
            raise B200Error(f"tracker_create failed: {last_error()}")

    def load(self, tensors: dict) -> None:
        for name, (t, arr, ne) in tensors.items():
            arr = np.ascontiguousarray(arr)
            ne4 = (ctypes.c_int64 * 4)(*(list(ne) + [1] * (4 - len(ne))))
            _check(lib().sam3b200_tracker_set_tensor(self.h, name.encode(), t, arr.ctypes.data, ne4), f"set {name}")

    def encode(self, img_chw: "DeviceBuffer") -> None:
        _check(lib().sam3b200_tracker_encode(self.h, img_chw.ptr), "tracker_encode")

    def add_instance(self, coords, labels, orig_w: int, orig_h: int) -> int:
        c = np.ascontiguousarray(coords, np.float32).reshape(-1)
        lab = np.ascontiguousarray(labels, np.int32)
        i = lib().sam3b200_tracker_add_instance(self.h, c.ctypes.data, lab.ctypes.data, lab.size, orig_w, orig_h)
        if i < 0:
            raise B200Error(f"tracker_add_instance: {last_error()}")
        return i

    def propagate(self) -> None:
        _check(lib().sam3b200_tracker_propagate(self.h), "tracker_propagate")

    def encode_image(self, rgb_ptr: int, w: int, h: int) -> None:
        """Host uint8 [h][w][3] frame at rgb_ptr: upload, SAM2 preprocessing, encode."""
        _check(lib().sam3b200_tracker_encode_image(self.h, ctypes.c_void_p(rgb_ptr), w, h), "tracker_encode_image")

    def reset(self) -> None:
        lib().sam3b200_tracker_reset(self.h)

    @property
    def frame_index(self) -> int:
        return lib().sam3b200_tracker_frame_index(self.h)

    def instances(self) -> list:
        ids = (ctypes.c_int32 * 64)()
        n = lib().sam3b200_tracker_instances(self.h, ids, 64)
        return list(ids[:n])

    def instance(self, iid: int) -> dict:
        """The instance's last kept mask logits [4H][4H], token [d_model], IoU, object score, last frame."""
        mp, tp = ctypes.c_void_p(), ctypes.c_void_p()
        iou, obj, seen = ctypes.c_float(), ctypes.c_float(), ctypes.c_int32()
        _check(lib().sam3b200_tracker_instance(self.h, iid, ctypes.byref(mp), ctypes.byref(tp), ctypes.byref(iou),
                                               ctypes.byref(obj), ctypes.byref(seen)), "tracker_instance")
        S, D = 4 * self.hp["feat"], self.hp["d_model"]
        mask, tok = np.empty((S, S), np.float32), np.empty(D, np.float32)
        _check(lib().sam3b200_tensor_get(self.be.h, mp.value, mask.ctypes.data, 0, mask.nbytes), "tensor_get")
        _check(lib().sam3b200_tensor_get(self.be.h, tp.value, tok.ctypes.data, 0, tok.nbytes), "tensor_get")
        return dict(mask=mask, token=tok, iou=iou.value, obj=obj.value, last_seen=seen.value)

    def mask(self, iid: int, out_w: int, out_h: int) -> np.ndarray:
        buf = DeviceBuffer(self.be, out_w * out_h)
        _check(lib().sam3b200_tracker_mask(self.h, iid, out_w, out_h, buf.ptr), "tracker_mask")
        self.be.synchronize()
        return buf.get((out_h, out_w), np.uint8)

    def bank(self, iid: int) -> tuple:
        """([(frame, is_cond, features [H*H][mem_dim])], [(frame, pointer [d_model])])"""
        cap = 256
        sf, sc, pf = (ctypes.c_int32 * cap)(), (ctypes.c_int32 * cap)(), (ctypes.c_int32 * cap)()
        sp, pp = (ctypes.c_void_p * cap)(), (ctypes.c_void_p * cap)()
        npt = ctypes.c_int32()
        ns = lib().sam3b200_tracker_bank(self.h, iid, sf, sc, sp, cap, pf, pp, cap, ctypes.byref(npt))
        if ns < 0:
            raise B200Error(f"tracker_bank: {last_error()}")
        N, MD, D = self.hp["feat"] ** 2, self.hp["mem_dim"], self.hp["d_model"]
        slots, ptrs = [], []
        for i in range(ns):
            a = np.empty((N, MD), np.float32)
            _check(lib().sam3b200_tensor_get(self.be.h, sp[i], a.ctypes.data, 0, a.nbytes), "tensor_get")
            slots.append((sf[i], bool(sc[i]), a))
        for i in range(npt.value):
            a = np.empty(D, np.float32)
            _check(lib().sam3b200_tensor_get(self.be.h, pp[i], a.ctypes.data, 0, a.nbytes), "tensor_get")
            ptrs.append((pf[i], a))
        return slots, ptrs

    def prompt(self, m_total: int) -> tuple:
        """The last propagated instance's prompt and prompt_pos, [m_total][mem_dim]."""
        p, q = ctypes.c_void_p(), ctypes.c_void_p()
        _check(lib().sam3b200_tracker_prompt(self.h, ctypes.byref(p), ctypes.byref(q)), "tracker_prompt")
        MD = self.hp["mem_dim"]
        a, b = np.empty((m_total, MD), np.float32), np.empty((m_total, MD), np.float32)
        _check(lib().sam3b200_tensor_get(self.be.h, p.value, a.ctypes.data, 0, a.nbytes), "tensor_get")
        _check(lib().sam3b200_tensor_get(self.be.h, q.value, b.ctypes.data, 0, b.nbytes), "tensor_get")
        return a, b

    def free(self) -> None:
        if self.h:
            lib().sam3b200_tracker_free(self.h)
            self.h = None


class FusionEncoder:
    """The detector's fusion encoder (sam3b200_fenc) on a backend."""

    FIELDS = ("d_model", "heads", "layers", "ffn_dim", "max_tokens", "max_prompt")

    def __init__(self, be: "Backend", hp: dict):
        self.be, self.hp = be, dict(hp)
        self._chp = (ctypes.c_int32 * 6)(*[int(hp[k]) for k in self.FIELDS])
        self.h = lib().sam3b200_fenc_create(be.h, ctypes.byref(self._chp))
        if not self.h:
            raise B200Error(f"fenc_create failed: {last_error()}")

    def load(self, tensors: dict) -> None:
        """tensors: name -> (ggml type, array, ne)"""
        for name, (t, arr, ne) in tensors.items():
            arr = np.ascontiguousarray(arr)
            ne4 = (ctypes.c_int64 * 4)(*(list(ne) + [1] * (4 - len(ne))))
            _check(lib().sam3b200_fenc_set_tensor(self.h, name.encode(), t, arr.ctypes.data, ne4), f"set {name}")
        buf = ctypes.create_string_buffer(1 << 16)
        n = lib().sam3b200_fenc_missing(self.h, buf, len(buf))
        if n:
            raise B200Error(f"{n} fenc tensors missing: {buf.value.decode()[:300]}")

    def run(self, image_feats, prompt, pos, prompt_bias=None) -> np.ndarray:
        """Host f32 token-major inputs (image_feats/pos [N][D], prompt [T][D], prompt_bias [T] or None)
        -> conditioned tokens [N][D]."""
        img, pr, ps = (np.ascontiguousarray(a, np.float32) for a in (image_feats, prompt, pos))
        pb = None if prompt_bias is None else np.ascontiguousarray(prompt_bias, np.float32)
        _check(lib().sam3b200_fenc_run(self.h, img.ctypes.data, pr.ctypes.data, ps.ctypes.data,
                                       None if pb is None else pb.ctypes.data, img.shape[0], pr.shape[0]), "fenc_run")
        p = ctypes.c_void_p()
        _check(lib().sam3b200_fenc_output(self.h, ctypes.byref(p)), "fenc_output")
        self.be.synchronize()
        out = np.empty(img.shape, np.float32)
        _check(lib().sam3b200_tensor_get(self.be.h, p.value, out.ctypes.data, 0, out.nbytes), "tensor_get")
        return out

    def free(self) -> None:
        if self.h:
            lib().sam3b200_fenc_free(self.h)
            self.h = None


class DetrDecoder:
    """The detector's DETR decoder with scoring and presence head (sam3b200_ddec) on a backend."""

    FIELDS = ("d_model", "heads", "layers", "ffn_dim", "num_queries", "feat", "max_prompt")

    def __init__(self, be: "Backend", hp: dict):
        self.be, self.hp = be, dict(hp)
        self._chp = (ctypes.c_int32 * 7)(*[int(hp[k]) for k in self.FIELDS])
        self.h = lib().sam3b200_ddec_create(be.h, ctypes.byref(self._chp))
        if not self.h:
            raise B200Error(f"ddec_create failed: {last_error()}")

    def load(self, tensors: dict) -> None:
        """tensors: name -> (ggml type, array, ne)"""
        for name, (t, arr, ne) in tensors.items():
            arr = np.ascontiguousarray(arr)
            ne4 = (ctypes.c_int64 * 4)(*(list(ne) + [1] * (4 - len(ne))))
            _check(lib().sam3b200_ddec_set_tensor(self.h, name.encode(), t, arr.ctypes.data, ne4), f"set {name}")
        buf = ctypes.create_string_buffer(1 << 16)
        n = lib().sam3b200_ddec_missing(self.h, buf, len(buf))
        if n:
            raise B200Error(f"{n} ddec tensors missing: {buf.value.decode()[:300]}")

    def run(self, enc, enc_pos, text, text_bias=None, text_valid=None) -> dict:
        """Host f32 token-major inputs -> dict of host outputs: queries [1+NQ][D], boxes [NQ][4],
        scores [NQ], presence (float)."""
        e, ep, tx = (np.ascontiguousarray(a, np.float32) for a in (enc, enc_pos, text))
        tb = None if text_bias is None else np.ascontiguousarray(text_bias, np.float32)
        tv = None if text_valid is None else np.ascontiguousarray(text_valid, np.float32)
        _check(lib().sam3b200_ddec_run(self.h, e.ctypes.data, ep.ctypes.data, tx.ctypes.data,
                                       None if tb is None else tb.ctypes.data, None if tv is None else tv.ctypes.data,
                                       tx.shape[0]), "ddec_run")
        ptr = [ctypes.c_void_p() for _ in range(4)]
        _check(lib().sam3b200_ddec_outputs(self.h, *[ctypes.byref(x) for x in ptr]), "ddec_outputs")
        self.be.synchronize()
        NQ, D = self.hp["num_queries"], self.hp["d_model"]
        outs = [np.empty((NQ + 1, D), np.float32), np.empty((NQ, 4), np.float32), np.empty(NQ, np.float32),
                np.empty(1, np.float32)]
        for p, o in zip(ptr, outs):
            _check(lib().sam3b200_tensor_get(self.be.h, p.value, o.ctypes.data, 0, o.nbytes), "tensor_get")
        return dict(queries=outs[0], boxes=outs[1], scores=outs[2], presence=float(outs[3][0]))

    def free(self) -> None:
        if self.h:
            lib().sam3b200_ddec_free(self.h)
            self.h = None


class SegHead:
    """The detector's segmentation head (sam3b200_seg) on a backend."""

    FIELDS = ("d_model", "heads", "feat", "max_queries", "max_prompt")

    def __init__(self, be: "Backend", hp: dict):
        self.be, self.hp = be, dict(hp)
        self._chp = (ctypes.c_int32 * 5)(*[int(hp[k]) for k in self.FIELDS])
        self.h = lib().sam3b200_seg_create(be.h, ctypes.byref(self._chp))
        if not self.h:
            raise B200Error(f"seg_create failed: {last_error()}")

    def load(self, tensors: dict) -> None:
        """tensors: name -> (ggml type, array, ne)"""
        for name, (t, arr, ne) in tensors.items():
            arr = np.ascontiguousarray(arr)
            ne4 = (ctypes.c_int64 * 4)(*(list(ne) + [1] * (4 - len(ne))))
            _check(lib().sam3b200_seg_set_tensor(self.h, name.encode(), t, arr.ctypes.data, ne4), f"set {name}")
        buf = ctypes.create_string_buffer(1 << 16)
        n = lib().sam3b200_seg_missing(self.h, buf, len(buf))
        if n:
            raise B200Error(f"{n} seg tensors missing: {buf.value.decode()[:300]}")

    def run(self, enc, fpn0, fpn1, queries, text, text_bias=None) -> np.ndarray:
        """Host f32 token-major inputs -> mask logits [n_queries][(4 feat)^2]."""
        e, f0, f1, q, tx = (np.ascontiguousarray(a, np.float32) for a in (enc, fpn0, fpn1, queries, text))
        tb = None if text_bias is None else np.ascontiguousarray(text_bias, np.float32)
        _check(lib().sam3b200_seg_run(self.h, e.ctypes.data, f0.ctypes.data, f1.ctypes.data, q.ctypes.data, q.shape[0],
                                      tx.ctypes.data, None if tb is None else tb.ctypes.data, tx.shape[0]), "seg_run")
        p = ctypes.c_void_p()
        _check(lib().sam3b200_seg_output(self.h, ctypes.byref(p)), "seg_output")
        self.be.synchronize()
        out = np.empty((q.shape[0], 16 * self.hp["feat"] ** 2), np.float32)
        _check(lib().sam3b200_tensor_get(self.be.h, p.value, out.ctypes.data, 0, out.nbytes), "tensor_get")
        return out

    def free(self) -> None:
        if self.h:
            lib().sam3b200_seg_free(self.h)
            self.h = None


class GeometryEncoder:
    """The detector's geometry (exemplar-prompt) encoder transformer (sam3b200_geom) on a backend."""

    FIELDS = ("d_model", "heads", "layers", "ffn_dim", "max_tokens", "max_image_tokens")

    def __init__(self, be: "Backend", hp: dict):
        self.be, self.hp = be, dict(hp)
        self._chp = (ctypes.c_int32 * 6)(*[int(hp[k]) for k in self.FIELDS])
        self.h = lib().sam3b200_geom_create(be.h, ctypes.byref(self._chp))
        if not self.h:
            raise B200Error(f"geom_create failed: {last_error()}")

    def load(self, tensors: dict) -> None:
        for name, (t, arr, ne) in tensors.items():
            arr = np.ascontiguousarray(arr)
            ne4 = (ctypes.c_int64 * 4)(*(list(ne) + [1] * (4 - len(ne))))
            _check(lib().sam3b200_geom_set_tensor(self.h, name.encode(), t, arr.ctypes.data, ne4), f"set {name}")
        buf = ctypes.create_string_buffer(1 << 16)
        n = lib().sam3b200_geom_missing(self.h, buf, len(buf))
        if n:
            raise B200Error(f"{n} geom tensors missing: {buf.value.decode()[:300]}")

    def run(self, tokens, img_feats, img_pe) -> np.ndarray:
        """Host f32 token-major tokens [S][D], img_feats / img_pe [N][D] -> encoded tokens [S][D]."""
        x, im, pe = (np.ascontiguousarray(a, np.float32) for a in (tokens, img_feats, img_pe))
        _check(lib().sam3b200_geom_run(self.h, x.ctypes.data, x.shape[0], im.ctypes.data, pe.ctypes.data, im.shape[0]),
               "geom_run")
        p = ctypes.c_void_p()
        _check(lib().sam3b200_geom_output(self.h, ctypes.byref(p)), "geom_output")
        self.be.synchronize()
        out = np.empty(x.shape, np.float32)
        _check(lib().sam3b200_tensor_get(self.be.h, p.value, out.ctypes.data, 0, out.nbytes), "tensor_get")
        return out

    def free(self) -> None:
        if self.h:
            lib().sam3b200_geom_free(self.h)
            self.h = None


class WeightFile:
    """A sam3.cpp weight file opened by the native reader (sam3b200_file_*); opening reads the header,
    hyper-parameters and tensor directory only."""

    PART_NAMES = ("vit", "hiera", "text", "sam_dec", "mem_attn", "mem_enc", "fenc", "ddec", "seg", "geom")

    def __init__(self, path: str):
        self.h = lib().sam3b200_file_open(str(path).encode())
        if not self.h:
            raise B200Error(f"file_open failed: {last_error()}")

    def info(self) -> dict:
        m, v, f, n = ctypes.c_uint32(), ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
        _check(lib().sam3b200_file_info(self.h, ctypes.byref(m), ctypes.byref(v), ctypes.byref(f), ctypes.byref(n)),
               "file_info")
        return dict(magic=m.value, version=v.value, ftype=f.value, n_tensors=n.value)

    def hparams(self) -> list[int]:
        n = lib().sam3b200_file_hparams(self.h, None, 0)
        words = (ctypes.c_int32 * max(n, 1))()
        lib().sam3b200_file_hparams(self.h, words, n)
        return list(words)[:n]

    def tensors(self) -> list[dict]:
        out = []
        for i in range(self.info()["n_tensors"]):
            name = ctypes.create_string_buffer(4097)
            t, ne, off, nb = ctypes.c_int32(), (ctypes.c_int64 * 4)(), ctypes.c_int64(), ctypes.c_int64()
            _check(lib().sam3b200_file_tensor(self.h, i, name, 4097, ctypes.byref(t), ne, ctypes.byref(off),
                                              ctypes.byref(nb)), "file_tensor")
            out.append(dict(name=name.value.decode(), type=t.value, ne=tuple(ne), offset=off.value, bytes=nb.value))
        return out

    def vit_hparams(self) -> "VitHparams":
        h = VitHparams()
        _check(lib().sam3b200_file_vit_hparams(self.h, ctypes.byref(h)), "file_vit_hparams")
        return h

    def text_hparams(self) -> dict:
        h = (ctypes.c_int32 * 6)()
        _check(lib().sam3b200_file_text_hparams(self.h, h), "file_text_hparams")
        return dict(zip(TextEncoder.FIELDS, list(h)))

    def hiera_hparams(self) -> "HieraHparams":
        h = HieraHparams()
        _check(lib().sam3b200_file_hiera_hparams(self.h, ctypes.byref(h)), "file_hiera_hparams")
        return h

    def load(self, backend: "Backend", **parts) -> tuple[int, int]:
        """Stream the tensors to the given runners (keyword per PART_NAMES, e.g. vit=Vit(...));
        returns (loaded, skipped)."""
        ptrs = (ctypes.c_void_p * len(self.PART_NAMES))(*[parts[k].h if k in parts else None for k in self.PART_NAMES])
        loaded, skipped = ctypes.c_int64(), ctypes.c_int64()
        _check(lib().sam3b200_file_load(self.h, backend.h, ptrs, ctypes.byref(loaded), ctypes.byref(skipped)),
               "file_load")
        return loaded.value, skipped.value

    def skipped(self) -> list[str]:
        buf = ctypes.create_string_buffer(1 << 20)
        lib().sam3b200_file_skipped(self.h, buf, len(buf))
        return [s for s in buf.value.decode().split("\n") if s]

    def close(self) -> None:
        if self.h:
            lib().sam3b200_file_close(self.h)
            self.h = None


class Backend:
    def __init__(self, device: int = 0):
        self.h = lib().sam3b200_backend_init(device)
        if not self.h:
            raise B200Error(f"backend_init({device}) failed: {last_error()}")

    @property
    def name(self) -> str:
        return lib().sam3b200_backend_name(self.h).decode()

    @property
    def stream(self) -> int:
        return lib().sam3b200_backend_stream(self.h)

    def synchronize(self) -> None:
        _check(lib().sam3b200_backend_synchronize(self.h), "synchronize")

    def debug_wait_timeout(self, limit_ns: int) -> None:
        """sam3b200_debug_wait_timeout: queue a bounded wait that runs out (failure-path test)."""
        _check(lib().sam3b200_debug_wait_timeout(self.h, limit_ns), "debug_wait_timeout")

    def alloc(self, nbytes: int) -> DeviceBuffer:
        return DeviceBuffer(self, nbytes)

    def upload(self, arr: np.ndarray) -> DeviceBuffer:
        arr = np.ascontiguousarray(arr)
        buf = DeviceBuffer(self, arr.nbytes)
        buf.set(arr)
        return buf

    def weight(self, qtype: int, blocks: np.ndarray, K: int, N: int) -> Weight:
        return Weight(self, qtype, blocks, K, N)

    def set_mmq_impl(self, impl: int) -> int:
        return lib().sam3b200_set_mmq_impl(self.h, impl)

    def set_arith(self, arith: int) -> int:
        """sam3b200_set_arith: ARITH_EXACT or ARITH_DQ16 for the encoder runners; returns the previous one."""
        return lib().sam3b200_set_arith(self.h, arith)

    def mul_mat(self, w: Weight, x: DeviceBuffer, M: int, y: DeviceBuffer, bias: DeviceBuffer | None = None,
                ldx: int | None = None, ldy: int | None = None) -> None:
        st = lib().sam3b200_mul_mat(self.h, w.h, x.ptr, ldx or w.K, M, bias.ptr if bias else None, y.ptr,
                                    ldy or w.N)
        _check(st, "mul_mat")

    def mul_mat_dq16(self, w: Weight, x: DeviceBuffer, M: int, y: DeviceBuffer, bias: DeviceBuffer | None = None,
                     ldx: int | None = None, ldy: int | None = None) -> None:
        """sam3b200_mul_mat_dq16: the MUL_MAT in the DQ16 arithmetic (fp16 tensor cores on dequantised Q8_0)."""
        st = lib().sam3b200_mul_mat_dq16(self.h, w.h, x.ptr, ldx or w.K, M, bias.ptr if bias else None, y.ptr,
                                         ldy or w.N)
        _check(st, "mul_mat_dq16")

    def mul_mat_noalloc(self, w: Weight, x: DeviceBuffer, M: int, y: DeviceBuffer,
                        bias: DeviceBuffer | None = None) -> None:
        """sam3b200_mul_mat_noalloc: the MUL_MAT with its activation scratch in
        the library's fixed device array (for callers that cannot allocate)."""
        st = lib().sam3b200_mul_mat_noalloc(self.h, w.h, x.ptr, w.K, M, bias.ptr if bias else None, y.ptr, w.N)
        _check(st, "mul_mat_noalloc")

    def mul_mat_block_dots(self, w: Weight, x: DeviceBuffer, M: int) -> np.ndarray:
        nb = w.K // 32
        out = self.alloc(M * w.N * nb * 4)
        _check(lib().sam3b200_mul_mat_block_dots(self.h, w.h, x.ptr, M, out.ptr), "mul_mat_block_dots")
        return out.get((M, w.N, nb), np.int32)

    def preprocess(self, rgb_dev: DeviceBuffer, w: int, h: int, img: int, out: DeviceBuffer) -> None:
        _check(lib().sam3b200_preprocess(self.h, rgb_dev.ptr, w, h, img, out.ptr), "preprocess")

    def flash_attn_ext(self, q: DeviceBuffer, k: DeviceBuffer, v: DeviceBuffer, D: int, N: int, heads: int,
                       batch: int, scale: float, dst: DeviceBuffer) -> None:
        """GGML_OP_FLASH_ATTN_EXT (sam3.cpp:3778): f32 [D, N, heads, batch] in, [D, heads, N, batch] out."""
        _check(lib().sam3b200_flash_attn_ext(self.h, q.ptr, k.ptr, v.ptr, D, N, heads, batch, scale, dst.ptr),
               "flash_attn_ext")

    def flash_attn_ext_view(self, q: int, k: int, v: int, mask: int | None, mask_nb1: int, D: int, NQ: int,
                            NKV: int, heads: int, batch: int, q_nb, k_nb, v_nb, scale: float, dst: DeviceBuffer) -> None:
        """General GGML_OP_FLASH_ATTN_EXT: q, k, v, mask are device addresses (views allowed); *_nb are the
        element strides (token, head, batch); dst f32 [D, heads, NQ, batch]."""
        arr = lambda nb: (ctypes.c_int64 * 3)(*[int(x) for x in nb])
        _check(lib().sam3b200_flash_attn_ext_view(self.h, q, k, v, mask, mask_nb1, D, NQ, NKV, heads, batch,
                                                  arr(q_nb), arr(k_nb), arr(v_nb), scale, dst.ptr),
               "flash_attn_ext_view")

    def conv_transpose_2d(self, w: DeviceBuffer, x: DeviceBuffer, iw: int, ih: int, ic: int, oc: int, kw: int,
                          kh: int, stride: int, dst: DeviceBuffer) -> None:
        """GGML_OP_CONV_TRANSPOSE_2D (ggml_conv_transpose_2d_p0): F16 kernel [kw, kh, oc, ic], f32 input
        [iw, ih, ic] -> f32 [(iw-1)*stride+kw, (ih-1)*stride+kh, oc]."""
        _check(lib().sam3b200_conv_transpose_2d(self.h, w.ptr, x.ptr, iw, ih, ic, oc, kw, kh, stride, dst.ptr),
               "conv_transpose_2d")

    def conv_2d(self, w: DeviceBuffer, x: DeviceBuffer, iw: int, ih: int, ic: int, oc: int, kw: int, kh: int,
                s0: int, s1: int, p0: int, p1: int, d0: int, d1: int, dst: DeviceBuffer) -> None:
        """GGML_OP_CONV_2D (ggml_conv_2d): F16 kernel [kw, kh, ic, oc], f32 input [iw, ih, ic] -> f32 [ow, oh, oc]."""
        _check(lib().sam3b200_conv_2d(self.h, w.ptr, x.ptr, iw, ih, ic, oc, kw, kh, s0, s1, p0, p1, d0, d1, dst.ptr),
               "conv_2d")

    def get_rows(self, qtype: int, src: DeviceBuffer, ncols: int, nrows: int, idx: DeviceBuffer, n: int,
                 dst: DeviceBuffer) -> None:
        """GGML_OP_GET_ROWS: dst[i] = dequantised row idx[i] of src (F32, F16, Q4_0, Q4_1, Q8_0)."""
        _check(lib().sam3b200_get_rows(self.h, qtype, src.ptr, ncols, nrows, idx.ptr, n, dst.ptr), "get_rows")

    def graph_compute(self, nodes) -> None:
        """sam3b200_graph_compute: run GraphTensor nodes in order and wait for them (ggml graph_compute)."""
        _check(graph_compute_status(self.h, nodes), "graph_compute")

    def preprocess_sam2(self, rgb_dev: DeviceBuffer, w: int, h: int, img: int, out: DeviceBuffer) -> None:
        """sam2_preprocess_image: ImageNet-normalised CHW (sam3.cpp:3522-3548)."""
        _check(lib().sam3b200_preprocess_sam2(self.h, rgb_dev.ptr, w, h, img, out.ptr), "preprocess_sam2")

    @property
    def launches(self) -> int:
        return int(lib().sam3b200_backend_launch_count(self.h))

    def profile(self, enable: bool) -> None:
        _check(lib().sam3b200_backend_profile(self.h, 1 if enable else 0), "profile")

    def profile_read(self, cls: int = 0):
        """(total ms, launch count) of the timed kernel class since profiling was enabled."""
        t, n = ctypes.c_double(), ctypes.c_int()
        _check(lib().sam3b200_backend_profile_read(self.h, cls, ctypes.byref(t), ctypes.byref(n)), "profile_read")
        return t.value, n.value

    def vit(self, hp: dict) -> Vit:
        return Vit(self, hp)

    def hiera(self, hp: dict) -> Hiera:
        return Hiera(self, hp)

    def sam_decoder(self, hp: dict) -> SamDecoder:
        return SamDecoder(self, hp)

    def text_encoder(self, hp: dict) -> TextEncoder:
        return TextEncoder(self, hp)

    def mem_attention(self, hp: dict) -> MemAttention:
        return MemAttention(self, hp)

    def mem_encoder(self, hp: dict) -> MemEncoder:
        return MemEncoder(self, hp)

    def tracker(self, hp: dict, enc: "Hiera", dec: "SamDecoder", attn: "MemAttention",
                menc: "MemEncoder") -> Tracker:
        return Tracker(self, hp, enc, dec, attn, menc)

    def fusion_encoder(self, hp: dict) -> FusionEncoder:
        return FusionEncoder(self, hp)

    def detr_decoder(self, hp: dict) -> DetrDecoder:
        return DetrDecoder(self, hp)

    def seg_head(self, hp: dict) -> SegHead:
        return SegHead(self, hp)

    def geometry_encoder(self, hp: dict) -> GeometryEncoder:
        return GeometryEncoder(self, hp)

    def free(self) -> None:
        if self.h:
            lib().sam3b200_backend_free(self.h)
            self.h = None
