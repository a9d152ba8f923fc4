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


def block_dots(qtype: int, wq: np.ndarray, K: int, N: int, x: np.ndarray, n_threads: int = 0) -> np.ndarray:
    """Per-(m, n, block) int32 dots of the integer codes: int32 [M, N, K/32]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    M = x.shape[0]
    out = np.empty((M, N, K // QK), dtype=np.int32)
    n_threads = n_threads or (os.cpu_count() or 1)
    lib().orc_mul_mat_block_dots(qtype, _ptr(np.ascontiguousarray(wq)), K, N, _ptr(x), M, _ptr(out), n_threads)
    return out
