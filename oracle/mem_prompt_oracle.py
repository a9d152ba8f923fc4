"""CPU restatement of the tracker's memory prompt preparation (TEST INFRASTRUCTURE ONLY).

Only tests/ import this module, as the checker of sam3b200_select_memory_frames and
sam3b200_build_mem_prompt.  It restates, in plain Python / numpy:
  - sam3_select_memory_frames (sam3.cpp:9427-9451): every slot when the bank holds at most
    max_slots, else slot 0, the newest slot and max_slots - 2 evenly spaced ones between them
    (float step (bank - 2) / (remaining + 1), truncated, clamped to bank - 2), sorted, unique;
  - the temporal positions of sam3_propagate_single (sam3.cpp:11196-11233): t = 0 for a
    conditioning slot, n_sel - s otherwise; pointer distance max(1, |frame - pointer frame|) for the
    first min(n, max_obj_ptrs) pointers;
  - sam3_build_prompt_and_pos (sam3.cpp:9126-9217): spatial tokens with pos + tpos_enc[num_maskmem
    - t - 1] when 0 <= t < num_maskmem; each pointer split into D / MD tokens whose positional
    code is obj_ptr_tpos_proj(sine_1d(distance / 15)) (sam3_get_1d_sine_pe, sam3.cpp:3641-3651).
  - sam3_extract_obj_ptr_cpu (sam3.cpp:9347-9420): the SAM token through three D x D layers (ReLU
    after the first two), or no_obj_ptr for a non-positive object score (SAM3), or the SAM2 blend
    l * mlp + (1 - l) * no_obj_ptr, l = [score > 0].
  - sam3_sinusoidal_pe_2d (sam3.cpp:3601-3637) and the memory-bank eviction of sam3_encode_memory
    (:11700-11711: beyond num_maskmem slots drop the oldest non-conditioning slot, else slot 1) and
    sam3_store_obj_ptr (:11716-11734: keep the newest max_obj_ptrs pointers).
Token rows are [tokens][MD] float32.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


def select_memory_frames(bank_size: int, max_slots: int) -> list[int]:
    if bank_size <= max_slots:
        return list(range(bank_size))
    sel = [0, bank_size - 1]
    remaining = max_slots - 2
    if remaining > 0:
        step = F32(bank_size - 2) / F32(remaining + 1)
        for i in range(remaining):
            idx = 1 + int(F32(i + 1) * step)
            sel.append(min(idx, bank_size - 2))
    return sorted(set(sel))


def sine_pe_1d(pos: float, dim: int, temperature: float = 10000.0) -> np.ndarray:
    half = dim // 2
    i = np.arange(half)
    paired = (i & ~1).astype(F32)
    dim_t = np.power(F32(temperature), paired / F32(half)).astype(F32)
    val = (F32(pos) / dim_t).astype(F32)
    return np.concatenate([np.sin(val), np.cos(val)]).astype(F32)


def build_mem_prompt(d_model: int, mem_dim: int, num_maskmem: int, max_obj_ptrs: int, slot_feats, slot_pes,
                     slot_is_cond, obj_ptrs, ptr_frames, cur_frame: int, tpos_enc=None, tpos_proj_w=None,
                     tpos_proj_b=None):
    """Returns (prompt [M_total][MD], prompt_pos [M_total][MD], n_ptr_tokens).  tpos_enc
    [num_maskmem][MD]; tpos_proj_w [MD][D] (ggml [D, MD]); tpos_proj_b [MD]; None = zeros."""
    MD, D = mem_dim, d_model
    split = D // MD
    n_sel = len(slot_feats)
    if tpos_enc is None:
        tpos_enc = np.zeros((num_maskmem, MD), F32)
    prompt, pos = [], []
    for s in range(n_sel):
        t = 0 if slot_is_cond[s] else n_sel - s
        f = np.asarray(slot_feats[s], F32).reshape(-1, MD)
        p = np.asarray(slot_pes[s], F32).reshape(-1, MD).copy()
        if 0 <= t < num_maskmem:
            p = (p + tpos_enc[num_maskmem - t - 1][None, :]).astype(F32)
        prompt.append(f)
        pos.append(p)
    n_ptr_tokens = 0
    w = np.zeros((MD, D), F32) if tpos_proj_w is None else np.asarray(tpos_proj_w, F32).reshape(MD, D)
    b = np.zeros(MD, F32) if tpos_proj_b is None else np.asarray(tpos_proj_b, F32)
    for p in range(min(len(obj_ptrs), max_obj_ptrs)):
        rel = max(1, abs(cur_frame - ptr_frames[p]))
        sine = sine_pe_1d(F32(rel) / F32(15.0), D).astype(np.float64)
        proj = (b.astype(np.float64) + w.astype(np.float64) @ sine).astype(F32)
        ptr = np.asarray(obj_ptrs[p], F32).reshape(split, MD)
        prompt.append(ptr)
        pos.append(np.repeat(proj[None, :], split, axis=0))
        n_ptr_tokens += split
    if not prompt:
        return np.zeros((0, MD), F32), np.zeros((0, MD), F32), 0
    return np.concatenate(prompt).astype(F32), np.concatenate(pos).astype(F32), n_ptr_tokens


def extract_obj_ptr(sam_token, obj_score: float, w, b, no_obj_ptr, blend: bool = False) -> np.ndarray:
    """w[j]: [out][in] float32; accumulation in float64 (the C code sums in f32 order)."""
    nop = np.asarray(no_obj_ptr, F32).reshape(-1)
    if not blend and obj_score <= 0.0:
        return nop.copy()
    h = np.asarray(sam_token, F32).astype(np.float64)
    for j in range(3):
        h = np.asarray(b[j], np.float64) + np.asarray(w[j], np.float64) @ h
        if j < 2:
            h = np.maximum(h, 0.0)
        h = h.astype(F32).astype(np.float64)
    h = h.astype(F32)
    if blend:
        lam = F32(1.0) if obj_score > 0.0 else F32(0.0)
        return (lam * h + (F32(1.0) - lam) * nop).astype(F32)
    return h


def sinusoidal_pe_2d(H: int, W: int, d_model: int) -> np.ndarray:
    """[H][W][d_model] float32; channels [0, d/2) from y, [d/2, d) from x; sin on even, cos on odd."""
    half = d_model // 2
    i = np.arange(half)
    dim_t = np.power(F32(10000.0), (i & ~1).astype(F32) / F32(half)).astype(F32)
    scale = F32(2.0 * np.pi)
    py = ((np.arange(H, dtype=F32) + F32(1)) / F32(H) * scale).astype(F32)
    px = ((np.arange(W, dtype=F32) + F32(1)) / F32(W) * scale).astype(F32)
    vy = (py[:, None] / dim_t[None, :]).astype(F32)
    vx = (px[:, None] / dim_t[None, :]).astype(F32)
    ey = np.where(i % 2 == 0, np.sin(vy), np.cos(vy)).astype(F32)  # [H][half]
    ex = np.where(i % 2 == 0, np.sin(vx), np.cos(vx)).astype(F32)  # [W][half]
    out = np.empty((H, W, d_model), F32)
    out[:, :, :half] = ey[:, None, :]
    out[:, :, half:] = ex[None, :, :]
    return out


class MemBank:
    """The bank's bookkeeping: slots [(frame, is_cond, feats)], pointers [(frame, ptr)]."""

    def __init__(self, num_maskmem: int, max_obj_ptrs: int):
        self.num_maskmem, self.max_obj_ptrs = num_maskmem, max_obj_ptrs
        self.slots, self.ptrs = [], []

    def add_slot(self, feats, frame: int, is_cond: bool) -> None:
        self.slots.append((frame, bool(is_cond), np.asarray(feats, F32)))
        while len(self.slots) > self.num_maskmem:
            for k, sl in enumerate(self.slots):
                if not sl[1]:
                    del self.slots[k]
                    break
            else:
                del self.slots[1]

    def add_ptr(self, ptr, frame: int) -> None:
        self.ptrs.append((frame, np.asarray(ptr, F32)))
        while len(self.ptrs) > self.max_obj_ptrs:
            del self.ptrs[0]
