"""tensor_core operators on host arrays, run by the CUDA kernels.

Same argument meaning and error behaviour as crates/tensor_core
(``gemv_bf16``, ``rmsnorm_bf16_weight``, ``gqa_attn_f32``,
``swiglu_mul_f32``, ``rope_f32``): each returns ``(status, result)`` with
status 0 on success and the reference's error variant otherwise.
"""
from __future__ import annotations

import numpy as np

from . import _lib


def _f(a):
    return np.ascontiguousarray(a, np.float32)


def gemv_bf16(w: np.ndarray, x, m: int, k: int):
    L = _lib.load()
    x = _f(x)
    w = np.ascontiguousarray(w, np.uint8)
    y = np.zeros(m, np.float32)
    st = L.myos_gemv_bf16(y.ctypes.data_as(_lib._f32p), y.size, w.ctypes.data_as(_lib._u8p), w.size,
                          x.ctypes.data_as(_lib._f32p), x.size, m, k)
    return st, y


def rmsnorm_bf16_weight(w: np.ndarray, x, eps: float):
    L = _lib.load()
    x = _f(x)
    w = np.ascontiguousarray(w, np.uint8)
    y = np.zeros(x.size, np.float32)
    st = L.myos_rmsnorm_bf16_weight(y.ctypes.data_as(_lib._f32p), y.size,
                                    w.ctypes.data_as(_lib._u8p), w.size,
                                    x.ctypes.data_as(_lib._f32p), x.size, eps)
    return st, y


def gqa_attn_f32(q, k, v, hq, hkv, d, seq, causal_pos=None):
    L = _lib.load()
    q, k, v = _f(q), _f(k), _f(v)
    y = np.zeros(hq * d, np.float32)
    mk, qp = (0, 0) if causal_pos is None else (1, causal_pos)
    st = L.myos_gqa_attn_f32(y.ctypes.data_as(_lib._f32p), y.size, q.ctypes.data_as(_lib._f32p),
                             q.size, k.ctypes.data_as(_lib._f32p), k.size,
                             v.ctypes.data_as(_lib._f32p), v.size, hq, hkv, d, seq, mk, qp)
    return st, y


def swiglu_mul_f32(gate, up):
    L = _lib.load()
    gate, up = _f(gate), _f(up)
    h = np.zeros(gate.size, np.float32)
    st = L.myos_swiglu_mul_f32(h.ctypes.data_as(_lib._f32p), h.size,
                               gate.ctypes.data_as(_lib._f32p), gate.size,
                               up.ctypes.data_as(_lib._f32p), up.size)
    return st, h


def rope_f32(x, position: int, head_dim: int, theta: float):
    L = _lib.load()
    x = _f(x)
    y = np.zeros(x.size, np.float32)
    st = L.myos_rope_f32(y.ctypes.data_as(_lib._f32p), y.size, x.ctypes.data_as(_lib._f32p),
                         x.size, position, head_dim, theta)
    return st, y
