"""CPU ORACLE bindings — test infrastructure only.

ctypes access to ``liboracle.so`` (a C++ restatement of the MyOS reference's
CPU numerics; see ``myos_oracle.h``). Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s ``cpu_baseline`` /
``--impl reference`` legs import this module, always as the checker or the
timed CPU baseline, never as the product path.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

OK, SHAPE, TOKEN, ROW_OOB, POSITION, CACHE_FULL, CACHE_RANGE = 0, 1, 2, 3, 4, 5, 6
W_MISSING, W_DTYPE, W_SHAPE, W_LENGTH, DUPLICATE, EMPTY_NAME = 7, 8, 9, 10, 11, 12
F32, F16, BF16 = 0, 1, 2

_f32p = C.POINTER(C.c_float)
_u8p = C.POINTER(C.c_uint8)
_u32p = C.POINTER(C.c_uint32)
_szp = C.POINTER(C.c_size_t)


class OrcShape(C.Structure):
    _fields_ = [
        ("hidden", C.c_size_t),
        ("num_q_heads", C.c_size_t),
        ("num_kv_heads", C.c_size_t),
        ("head_dim", C.c_size_t),
        ("rope_theta", C.c_float),
        ("intermediate", C.c_size_t),
        ("vocab", C.c_size_t),
        ("num_layers", C.c_size_t),
        ("rms_eps", C.c_float),
        ("tied_head", C.c_int),
    ]


def build() -> str:
    """Compile liboracle.so with its Makefile (g++ only)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        L.orc_bf16_le_to_f32.restype = C.c_float
        L.orc_silu_f32.restype = C.c_float
        L.orc_silu_f32.argtypes = [C.c_float]
        L.orc_greedy_token.restype = C.c_uint32
        L.orc_greedy_token.argtypes = [_f32p, C.c_size_t]
        L.orc_gemv_row_spans.restype = C.c_size_t
        L.orc_gemv_row_spans.argtypes = [C.c_size_t, C.c_size_t, _szp]
        L.orc_map_new.restype = C.c_void_p
        L.orc_map_free.argtypes = [C.c_void_p]
        L.orc_map_len.restype = C.c_size_t
        L.orc_map_len.argtypes = [C.c_void_p]
        L.orc_map_insert.argtypes = [C.c_void_p, C.c_char_p, C.c_int, _szp, C.c_size_t,
                                     C.c_void_p, C.c_size_t, C.c_int]
        L.orc_model_new.restype = C.c_void_p
        L.orc_model_new.argtypes = [C.POINTER(OrcShape), C.c_size_t, C.POINTER(C.c_int)]
        L.orc_model_free.argtypes = [C.c_void_p]
        L.orc_forward_token.argtypes = [C.c_void_p, C.c_void_p, C.c_uint32, C.c_size_t]
        L.orc_prefill.argtypes = [C.c_void_p, C.c_void_p, _u32p, C.c_size_t]
        L.orc_greedy_decode.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, _u32p, _f32p, _f32p]
        L.orc_forced_decode.argtypes = [C.c_void_p, C.c_void_p, _u32p, C.c_size_t, _u32p, _f32p,
                                        _f32p]
        L.orc_model_logits.restype = _f32p
        L.orc_model_logits.argtypes = [C.c_void_p]
        L.orc_model_residual.restype = _f32p
        L.orc_model_residual.argtypes = [C.c_void_p]
        L.orc_kv_len.restype = C.c_size_t
        L.orc_kv_len.argtypes = [C.c_void_p]
        L.orc_kv_clear.argtypes = [C.c_void_p]
        L.orc_kv_head.argtypes = [C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t, _f32p, _f32p]
        L.orc_set_threads.argtypes = [C.c_int]
        L.orc_get_threads.restype = C.c_int
        sz = C.c_size_t
        L.orc_bf16_le_to_f32.argtypes = [_u8p]
        L.orc_gemv_bf16.argtypes = [_f32p, sz, _u8p, sz, _f32p, sz, sz, sz, C.c_int]
        L.orc_gemm_bf16.argtypes = [_f32p, sz, _u8p, sz, _f32p, sz, sz, sz, sz, C.c_int]
        L.orc_add_bf16_bias.argtypes = [_f32p, sz, _u8p, sz]
        L.orc_embed_gather_bf16.argtypes = [_f32p, sz, _u8p, sz, _szp, sz, C.c_uint32]
        L.orc_rmsnorm_f32.argtypes = [_f32p, sz, _f32p, sz, _f32p, sz, C.c_float]
        L.orc_rmsnorm_bf16_weight.argtypes = [_f32p, sz, _u8p, sz, _f32p, sz, C.c_float]
        L.orc_attn_scale_f32.argtypes = [sz, _f32p]
        L.orc_gqa_attn_f32.argtypes = [_f32p, sz, _f32p, sz, _f32p, sz, _f32p, sz, _f32p, sz, sz,
                                       sz, sz, sz, C.c_int, sz]
        L.orc_rope_inv_freqs.argtypes = [_f32p, sz, sz, C.c_float]
        L.orc_rope_f32.argtypes = [_f32p, sz, _f32p, sz, C.c_uint32, sz, C.c_float]
        L.orc_rope_f32_inplace.argtypes = [_f32p, sz, C.c_uint32, sz, C.c_float]
        L.orc_swiglu_mul_f32.argtypes = [_f32p, sz, _f32p, sz, _f32p, sz]
        L.orc_swiglu_bf16.argtypes = [_f32p, sz, _f32p, sz, _u8p, sz, _u8p, sz, _u8p, sz, _f32p,
                                      sz, _f32p, sz, _f32p, sz, sz, sz]
        _lib = L
    return _lib


# ------------------------------------------------------------------ helpers
def f32p(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_f32p)


def u8p(a: np.ndarray):
    assert a.dtype == np.uint8 and a.flags.c_contiguous
    return a.ctypes.data_as(_u8p)


def pack_bf16(values) -> np.ndarray:
    """Exact BF16 little-endian bytes of f32 values whose low 16 bits are zero."""
    a = np.asarray(values, dtype=np.float32)
    bits = a.view(np.uint32)
    assert np.all(bits & 0xFFFF == 0), "value is not exact in bf16"
    return (bits >> 16).astype("<u2").view(np.uint8).copy()


def f32_bits(a) -> list:
    return [int(b) for b in np.asarray(a, dtype=np.float32).view(np.uint32)]


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def gemv_bf16(w: np.ndarray, x: np.ndarray, m: int, k: int, threads: int = 0, y=None):
    y = np.zeros(m, np.float32) if y is None else y
    x = np.ascontiguousarray(x, np.float32)
    st = lib().orc_gemv_bf16(f32p(y), y.size, u8p(w), w.size, f32p(x), x.size, m, k, threads)
    return st, y


def gemm_bf16(w, x, batch, m, k, threads=0):
    y = np.zeros(batch * m, np.float32)
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    st = lib().orc_gemm_bf16(f32p(y), y.size, u8p(w), w.size, f32p(x), x.size, batch, m, k,
                             threads)
    return st, y


def rmsnorm_bf16_weight(w_bytes, x, eps, y=None):
    x = np.ascontiguousarray(x, np.float32)
    y = np.zeros(x.size, np.float32) if y is None else y
    st = lib().orc_rmsnorm_bf16_weight(f32p(y), y.size, u8p(w_bytes), w_bytes.size, f32p(x),
                                       x.size, C.c_float(eps))
    return st, y


def rmsnorm_f32(w, x, eps, y=None):
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    y = np.zeros(x.size, np.float32) if y is None else y
    st = lib().orc_rmsnorm_f32(f32p(y), y.size, f32p(w), w.size, f32p(x), x.size, C.c_float(eps))
    return st, y


def add_bf16_bias(y, bias_bytes):
    return lib().orc_add_bf16_bias(f32p(y), y.size, u8p(bias_bytes), bias_bytes.size)


def embed_gather_bf16(table, shape, token, out):
    sh = (C.c_size_t * len(shape))(*shape)
    return lib().orc_embed_gather_bf16(f32p(out), out.size, u8p(table), table.size, sh,
                                       len(shape), C.c_uint32(token))


def attn_scale_f32(head_dim):
    out = np.zeros(1, np.float32)
    st = lib().orc_attn_scale_f32(head_dim, f32p(out))
    return st, out[0]


def gqa_attn_f32(q, k, v, hq, hkv, d, seq, causal_pos=None, y=None, probs=None):
    q = np.ascontiguousarray(q, np.float32)
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    y = np.zeros(hq * d, np.float32) if y is None else y
    probs = np.zeros(seq, np.float32) if probs is None else probs
    mk, qp = (0, 0) if causal_pos is None else (1, causal_pos)
    st = lib().orc_gqa_attn_f32(f32p(y), y.size, f32p(q), q.size, f32p(k), k.size, f32p(v),
                                v.size, f32p(probs), probs.size, C.c_size_t(hq),
                                C.c_size_t(hkv), C.c_size_t(d), C.c_size_t(seq), mk,
                                C.c_size_t(qp))
    return st, y, probs


def rope_inv_freqs(head_dim, theta, n=None):
    n = head_dim // 2 if n is None else n
    out = np.zeros(max(n, 1), np.float32)
    st = lib().orc_rope_inv_freqs(f32p(out), C.c_size_t(n), C.c_size_t(head_dim),
                                  C.c_float(theta))
    return st, out[:n]


def rope_f32(x, position, head_dim, theta, y=None):
    x = np.ascontiguousarray(x, np.float32)
    y = np.zeros_like(x) if y is None else y
    st = lib().orc_rope_f32(f32p(y), y.size, f32p(x), x.size, C.c_uint32(position),
                            C.c_size_t(head_dim), C.c_float(theta))
    return st, y


def rope_f32_inplace(x, position, head_dim, theta):
    return lib().orc_rope_f32_inplace(f32p(x), x.size, C.c_uint32(position), C.c_size_t(head_dim),
                                      C.c_float(theta))


def silu_f32(z):
    return lib().orc_silu_f32(C.c_float(z))


def swiglu_mul_f32(gate, up, h=None):
    gate = np.ascontiguousarray(gate, np.float32)
    up = np.ascontiguousarray(up, np.float32)
    h = np.zeros(gate.size, np.float32) if h is None else h
    st = lib().orc_swiglu_mul_f32(f32p(h), h.size, f32p(gate), gate.size, f32p(up), up.size)
    return st, h


def swiglu_bf16(x, gate_w, up_w, down_w, hidden, inter):
    x = np.ascontiguousarray(x, np.float32)
    y = np.zeros(hidden, np.float32)
    g = np.zeros(inter, np.float32)
    u = np.zeros(inter, np.float32)
    h = np.zeros(inter, np.float32)
    st = lib().orc_swiglu_bf16(f32p(y), y.size, f32p(x), x.size, u8p(gate_w), gate_w.size,
                               u8p(up_w), up_w.size, u8p(down_w), down_w.size, f32p(g), g.size,
                               f32p(u), u.size, f32p(h), h.size, hidden, inter)
    return st, y, g, u, h


def greedy_token(logits) -> int:
    a = np.ascontiguousarray(logits, np.float32)
    return int(lib().orc_greedy_token(f32p(a), a.size))


def gemv_row_spans(m, threads):
    buf = (C.c_size_t * 128)()
    n = lib().orc_gemv_row_spans(m, threads, buf)
    return [(buf[2 * i], buf[2 * i + 1]) for i in range(n)]


# ------------------------------------------------------------------ model
@dataclass
class Shape:
    hidden: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    rope_theta: float
    intermediate: int
    vocab: int
    num_layers: int
    rms_eps: float
    tied_head: bool = True

    def c(self) -> OrcShape:
        return OrcShape(self.hidden, self.num_q_heads, self.num_kv_heads, self.head_dim,
                        self.rope_theta, self.intermediate, self.vocab, self.num_layers,
                        self.rms_eps, 1 if self.tied_head else 0)


class WeightMap:
    """Named-tensor table (MmapWeights). Borrows the byte arrays it is given."""

    def __init__(self):
        self.h = lib().orc_map_new()
        self._keep = []

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_map_free(self.h)
            self.h = None

    def insert(self, name: str, dtype: int, shape, data: np.ndarray) -> int:
        data = np.ascontiguousarray(data)
        self._keep.append(data)
        sh = (C.c_size_t * max(len(shape), 1))(*shape)
        return lib().orc_map_insert(self.h, name.encode(), dtype, sh, len(shape),
                                    data.ctypes.data_as(C.c_void_p), data.nbytes, 0)

    def insert_bf16(self, name, shape, data: np.ndarray) -> int:
        return self.insert(name, BF16, shape, data)

    def __len__(self):
        return int(lib().orc_map_len(self.h))


class Model:
    """KvCache + BlockWorkspace + forward/prefill/greedy_decode over a WeightMap."""

    def __init__(self, shape: Shape, max_seq: int):
        st = C.c_int()
        cs = shape.c()
        self.h = lib().orc_model_new(C.byref(cs), max_seq, C.byref(st))
        self.status = st.value
        self.shape = shape
        self.max_seq = max_seq

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_model_free(self.h)
            self.h = None

    def forward_token(self, wmap: WeightMap, token: int, pos: int) -> int:
        return lib().orc_forward_token(self.h, wmap.h, C.c_uint32(token), C.c_size_t(pos))

    def prefill(self, wmap: WeightMap, tokens) -> int:
        t = np.ascontiguousarray(tokens, np.uint32)
        return lib().orc_prefill(self.h, wmap.h, t.ctypes.data_as(_u32p), t.size)

    def greedy_decode(self, wmap: WeightMap, steps: int, dump_logits=False):
        out = np.zeros(steps, np.uint32)
        gap = np.zeros(steps, np.float32)
        dump = np.zeros(steps * self.shape.vocab, np.float32) if dump_logits else None
        st = lib().orc_greedy_decode(self.h, wmap.h, steps, out.ctypes.data_as(_u32p),
                                     f32p(dump) if dump is not None else None, f32p(gap))
        return st, out, gap, dump

    def forced_decode(self, wmap: WeightMap, feed, dump_logits=False):
        feed = np.ascontiguousarray(feed, np.uint32)
        steps = feed.size
        am = np.zeros(steps, np.uint32)
        gap = np.zeros(steps, np.float32)
        dump = np.zeros(steps * self.shape.vocab, np.float32) if dump_logits else None
        st = lib().orc_forced_decode(self.h, wmap.h, feed.ctypes.data_as(_u32p), steps,
                                     am.ctypes.data_as(_u32p), f32p(gap),
                                     f32p(dump) if dump is not None else None)
        return st, am, gap, dump

    def logits(self) -> np.ndarray:
        p = lib().orc_model_logits(self.h)
        return np.ctypeslib.as_array(p, shape=(self.shape.vocab,)).copy()

    def residual(self) -> np.ndarray:
        p = lib().orc_model_residual(self.h)
        return np.ctypeslib.as_array(p, shape=(self.shape.hidden,)).copy()

    def kv_len(self) -> int:
        return int(lib().orc_kv_len(self.h))

    def kv_clear(self):
        lib().orc_kv_clear(self.h)

    def kv_head(self, layer, head, pos):
        k = np.zeros(self.shape.head_dim, np.float32)
        v = np.zeros(self.shape.head_dim, np.float32)
        st = lib().orc_kv_head(self.h, layer, head, pos, f32p(k), f32p(v))
        return st, k, v
