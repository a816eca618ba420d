"""Host-side mirror of the reference's model_core API over the CUDA engine.

``Engine`` owns one device context (weights, KV cache and workspace in HBM).
Its methods keep the reference's names and semantics:

  reference (crates/model_core)                      here
  -------------------------------------------------  ---------------------------
  KvCache::new / len / clear / key_head / value_head  Engine(...), kv_len, reset, kv_head
  BlockWorkspace::logits                              logits()
  forward_token(token, pos, map, shape, cache, work)  forward_token(token, pos)
  prefill(tokens, map, shape, cache, work)            prefill(tokens)
  greedy_decode(steps, map, shape, cache, work, out)  greedy_decode(steps)

Errors raise :class:`MyosError` whose ``code`` names the reference enum
variant (Shape, Position, Token, CacheFull, WeightMissing, ...). As in the
reference, a failed call leaves the KV cursor and the logits unchanged.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from ._lib import MyosError


def shape_from_dict(d: dict) -> _lib.Shape:
    return _lib.Shape(int(d["hidden"]), int(d["num_q_heads"]), int(d["num_kv_heads"]),
                      int(d["head_dim"]), float(d["rope_theta"]), int(d["intermediate"]),
                      int(d["vocab"]), int(d["num_layers"]), float(d["rms_eps"]),
                      1 if d.get("tied_head", True) else 0)


def tp_unique_id() -> bytes:
    """A fresh rendezvous token for a tensor-parallel group (myos_tp_unique_id);
    made on one rank and handed to every rank's Engine(tp=(size, rank, id))."""
    L = _lib.load()
    buf = (C.c_uint8 * 128)()
    st = L.myos_tp_unique_id(buf)
    if st != 0:
        raise MyosError(st, "myos_tp_unique_id failed")
    return bytes(buf)


class Engine:
    def __init__(self, shape: dict, max_seq: int, device: int = 0, kv_dtype: str = "f32",
                 use_graphs: bool = True, tp=None):
        """tp = (size, rank, unique_id): this process is one rank of a
        tensor-parallel group (one process per GPU; every rank makes the same
        calls in the same order). Weights are passed whole on every rank."""
        self.L = _lib.load()
        self.shape = dict(shape)
        self.max_seq = int(max_seq)
        self.kv_dtype = kv_dtype
        s = shape_from_dict(shape)
        o = _lib.Opts(int(device), int(max_seq), _lib.KV_BF16 if kv_dtype == "bf16" else _lib.KV_F32,
                      1 if use_graphs else 0)
        h = C.c_void_p()
        if tp is None:
            st = self.L.myos_ctx_create(C.byref(s), C.byref(o), C.byref(h))
        else:
            size, rank, uid = tp
            t = _lib.TP(int(size), int(rank))
            C.memmove(t.unique_id, bytes(uid), 128)
            st = self.L.myos_ctx_create_tp(C.byref(s), C.byref(o), C.byref(t), C.byref(h))
        if st != 0:
            raise MyosError(st, "myos_ctx_create failed")
        self.h = h

    # ---------------------------------------------------------------- lifetime
    def close(self):
        if getattr(self, "h", None):
            self.L.myos_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _check(self, st: int):
        if st != 0:
            raise MyosError(st, self.L.myos_last_error(self.h).decode(errors="replace"))

    def last_error(self) -> str:
        return self.L.myos_last_error(self.h).decode(errors="replace")

    # ---------------------------------------------------------------- weights
    def load_tensor(self, name: str, dims, data: np.ndarray, dtype: int = _lib.BF16) -> None:
        data = np.ascontiguousarray(data)
        shape = (C.c_int64 * max(len(dims), 1))(*[int(x) for x in dims])
        self._check(self.L.myos_load_tensor(self.h, name.encode(), dtype, shape, len(dims),
                                            data.ctypes.data_as(C.c_void_p), data.nbytes))

    def load_table(self, table: dict) -> None:
        """{name: (dims, bf16 bytes)} — e.g. myos.synth.weights(...) or a fixture."""
        for name, (dims, data) in table.items():
            self.load_tensor(name, dims, data)

    def load_safetensors(self, path: str) -> None:
        self._check(self.L.myos_load_safetensors(self.h, path.encode()))

    def weights_ready(self) -> bool:
        return bool(self.L.myos_weights_ready(self.h))

    # ---------------------------------------------------------------- token loop
    def forward_token(self, token: int, pos: int, want_logits: bool = True):
        out = np.empty(self.shape["vocab"], np.float32) if want_logits else None
        self._check(self.L.myos_forward_token(
            self.h, C.c_uint32(token), pos,
            out.ctypes.data_as(_lib._f32p) if out is not None else None))
        return out

    def prefill(self, tokens, want_logits: bool = True):
        t = np.ascontiguousarray(tokens, np.uint32)
        out = np.empty(self.shape["vocab"], np.float32) if want_logits else None
        self._check(self.L.myos_prefill(self.h, t.ctypes.data_as(_lib._u32p), t.size,
                                        out.ctypes.data_as(_lib._f32p) if out is not None else None))
        return out

    def greedy_decode(self, steps: int) -> np.ndarray:
        out = np.zeros(max(steps, 1), np.uint32)
        self._check(self.L.myos_greedy_decode(self.h, steps, out.ctypes.data_as(_lib._u32p)))
        return out[:steps]

    def batch_generate(self, prompts, steps: int) -> np.ndarray:
        """Greedy ids [len(prompts), steps] for independent prompts decoded
        together (myos_batch_generate); the context's own cache is untouched."""
        lens = np.array([len(p) for p in prompts], np.uint32)
        ids = np.ascontiguousarray(np.concatenate([np.asarray(p, np.uint32) for p in prompts]),
                                   np.uint32)
        out = np.zeros(max(len(prompts) * steps, 1), np.uint32)
        self._check(self.L.myos_batch_generate(self.h, len(prompts), ids.ctypes.data_as(_lib._u32p),
                                               lens.ctypes.data_as(_lib._u32p), steps,
                                               out.ctypes.data_as(_lib._u32p)))
        return out[:len(prompts) * steps].reshape(len(prompts), steps)

    def batch_forced(self, prompts, feed, want_logits: bool = False):
        """Teacher-forced batched decode (myos_batch_forced_decode): feed is
        [len(prompts), steps]; returns (argmax [len(prompts), steps], final
        logits [len(prompts), vocab] or None)."""
        lens = np.array([len(p) for p in prompts], np.uint32)
        ids = np.ascontiguousarray(np.concatenate([np.asarray(p, np.uint32) for p in prompts]),
                                   np.uint32)
        feed = np.ascontiguousarray(feed, np.uint32).reshape(len(prompts), -1)
        steps = feed.shape[1]
        am = np.zeros(max(feed.size, 1), np.uint32)
        lg = np.zeros(len(prompts) * self.shape["vocab"], np.float32) if want_logits else None
        self._check(self.L.myos_batch_forced_decode(
            self.h, len(prompts), ids.ctypes.data_as(_lib._u32p), lens.ctypes.data_as(_lib._u32p),
            steps, feed.ctypes.data_as(_lib._u32p), am.ctypes.data_as(_lib._u32p),
            lg.ctypes.data_as(_lib._f32p) if lg is not None else None))
        am = am[:feed.size].reshape(len(prompts), steps)
        return am, (lg.reshape(len(prompts), -1) if lg is not None else None)

    def forced_decode(self, ids) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.uint32)
        am = np.zeros(max(ids.size, 1), np.uint32)
        self._check(self.L.myos_forced_decode(self.h, ids.ctypes.data_as(_lib._u32p), ids.size,
                                              am.ctypes.data_as(_lib._u32p)))
        return am[:ids.size]

    def logits(self) -> np.ndarray:
        out = np.empty(self.shape["vocab"], np.float32)
        self._check(self.L.myos_logits(self.h, out.ctypes.data_as(_lib._f32p)))
        return out

    def kv_len(self) -> int:
        n = C.c_size_t()
        self._check(self.L.myos_kv_len(self.h, C.byref(n)))
        return n.value

    def reset(self) -> None:
        self._check(self.L.myos_reset(self.h))

    def kv_head(self, layer: int, head: int, pos: int):
        d = self.shape["head_dim"]
        k = np.empty(d, np.float32)
        v = np.empty(d, np.float32)
        self._check(self.L.myos_kv_head(self.h, layer, head, pos, k.ctypes.data_as(_lib._f32p),
                                        v.ctypes.data_as(_lib._f32p)))
        return k, v

    KERNEL_KINDS = ("qkv", "attention", "o_proj", "gate_up", "down", "head")

    def profile_kernels(self, iters: int = 3) -> dict:
        """{kind: (mean ms per launch, algorithmic bytes per launch)}."""
        ms = (C.c_float * 6)()
        by = (C.c_double * 6)()
        self._check(self.L.myos_profile_kernels(self.h, iters, ms, by))
        return {k: (ms[i], by[i]) for i, k in enumerate(self.KERNEL_KINDS)}

    def last_timing(self):
        p = C.c_float()
        d = C.c_float()
        self._check(self.L.myos_last_timing(self.h, C.byref(p), C.byref(d)))
        return p.value, d.value

    def launch_count(self) -> int:
        """Kernel launches the library has enqueued in this process so far
        (graph replays count the kernels captured in them)."""
        n = C.c_uint64()
        self._check(self.L.myos_launch_count(C.byref(n)))
        return int(n.value)


def greedy_token(logits) -> int:
    """model_core::greedy_token (lib.rs:157-167) on the device."""
    L = _lib.load()
    a = np.ascontiguousarray(logits, np.float32)
    out = C.c_uint32()
    st = L.myos_greedy_token(a.ctypes.data_as(_lib._f32p), a.size, C.byref(out))
    if st != 0:
        raise MyosError(st)
    return int(out.value)


def check_safetensors(path: str) -> int:
    """SafeTensorsMmap::open + parse on the host; returns the tensor count."""
    L = _lib.load()
    n = C.c_size_t()
    err = C.create_string_buffer(512)
    st = L.myos_check_safetensors(path.encode(), C.byref(n), err, 512)
    if st != 0:
        raise MyosError(st, err.value.decode(errors="replace"))
    return n.value
