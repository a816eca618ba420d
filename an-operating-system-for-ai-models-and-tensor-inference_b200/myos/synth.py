"""Seeded synthetic Qwen2.5 weights and prompts (the BASELINE configs).

Weights follow the configs' recipe: linear, embedding and bias tensors
~N(0, 0.02); norm weights 1 + N(0, 0.01); f32 -> bf16 round-to-nearest-even.
Stream s of a tensor is its index in :func:`tensor_specs` (the SafeTensors
key order of ``qwen25_layout``: embed, then per layer the 12 suffixes in
LAYER_SUFFIXES order, then the final norm, then lm_head when untied), so
any subset of tensors can be regenerated independently.
"""
from __future__ import annotations

import ctypes as C
import json
import os
import struct

import numpy as np

from . import _lib

LAYER_SUFFIXES = [
    "input_layernorm.weight",
    "self_attn.q_proj.weight",
    "self_attn.q_proj.bias",
    "self_attn.k_proj.weight",
    "self_attn.k_proj.bias",
    "self_attn.v_proj.weight",
    "self_attn.v_proj.bias",
    "self_attn.o_proj.weight",
    "post_attention_layernorm.weight",
    "mlp.gate_proj.weight",
    "mlp.up_proj.weight",
    "mlp.down_proj.weight",
]
PROMPT_STREAM = 0x5052_4F4D_5054  # distinct from every tensor stream

_synth = None


def _lib_synth():
    global _synth
    if _synth is None:
        if not os.path.exists(_lib.SYNTH_LIB):
            raise RuntimeError(f"{_lib.SYNTH_LIB} is missing: build it with python build.py")
        L = C.CDLL(_lib.SYNTH_LIB)
        L.myos_synth_normal_bf16.argtypes = [C.c_uint64, C.c_uint64, C.c_float, C.c_float,
                                             C.c_void_p, C.c_size_t, C.c_int]
        L.myos_synth_normal_f32.argtypes = [C.c_uint64, C.c_uint64, C.c_float, C.c_float,
                                            C.c_void_p, C.c_size_t, C.c_int]
        L.myos_synth_uniform_u32.argtypes = [C.c_uint64, C.c_uint64, C.c_uint32, C.c_void_p,
                                             C.c_size_t]
        L.myos_synth_normal_bf16_block.argtypes = [C.c_uint64, C.c_uint64, C.c_float, C.c_float,
                                                   C.c_void_p] + [C.c_size_t] * 6 + [C.c_int]
        _synth = L
    return _synth


def shape_qwen25_1_5b() -> dict:
    return dict(hidden=1536, num_q_heads=12, num_kv_heads=2, head_dim=128, rope_theta=1e6,
                intermediate=8960, vocab=151936, num_layers=28, rms_eps=1e-6, tied_head=True)


def shape_qwen25_14b() -> dict:
    return dict(hidden=5120, num_q_heads=40, num_kv_heads=8, head_dim=128, rope_theta=1e6,
                intermediate=13824, vocab=152064, num_layers=48, rms_eps=1e-6, tied_head=False)


def tensor_specs(shape: dict):
    """[(name, dims, is_norm)] in stream order."""
    h = shape["hidden"]
    qd = shape["num_q_heads"] * shape["head_dim"]
    kvd = shape["num_kv_heads"] * shape["head_dim"]
    inter = shape["intermediate"]
    dims = {
        "input_layernorm.weight": [h],
        "self_attn.q_proj.weight": [qd, h],
        "self_attn.q_proj.bias": [qd],
        "self_attn.k_proj.weight": [kvd, h],
        "self_attn.k_proj.bias": [kvd],
        "self_attn.v_proj.weight": [kvd, h],
        "self_attn.v_proj.bias": [kvd],
        "self_attn.o_proj.weight": [h, qd],
        "post_attention_layernorm.weight": [h],
        "mlp.gate_proj.weight": [inter, h],
        "mlp.up_proj.weight": [inter, h],
        "mlp.down_proj.weight": [h, inter],
    }
    out = [("model.embed_tokens.weight", [shape["vocab"], h], False)]
    for layer in range(shape["num_layers"]):
        for suf in LAYER_SUFFIXES:
            out.append((f"model.layers.{layer}.{suf}", dims[suf], "layernorm" in suf))
    out.append(("model.norm.weight", [h], True))
    if not shape.get("tied_head", True):
        out.append(("lm_head.weight", [shape["vocab"], h], False))
    return out


def normal_bf16(seed: int, stream: int, n: int, mean: float, std: float,
                threads: int = 0) -> np.ndarray:
    out = np.empty(n, np.uint16)
    _lib_synth().myos_synth_normal_bf16(seed, stream, mean, std,
                                        out.ctypes.data_as(C.c_void_p), n, threads)
    return out


def normal_bf16_block(seed: int, stream: int, rows: int, cols: int, row0: int, nrows: int,
                      col0: int, ncols: int, mean: float, std: float,
                      threads: int = 0) -> np.ndarray:
    """A rows x cols buffer holding only block [row0, +nrows) x [col0, +ncols)
    of normal_bf16(seed, stream, rows * cols, ...) (same values); the rest
    is uninitialised."""
    out = np.empty(rows * cols, np.uint16)
    _lib_synth().myos_synth_normal_bf16_block(seed, stream, mean, std,
                                              out.ctypes.data_as(C.c_void_p), rows, cols, row0,
                                              nrows, col0, ncols, threads)
    return out


def normal_f32(seed: int, stream: int, n: int, mean: float = 0.0, std: float = 1.0,
               threads: int = 0) -> np.ndarray:
    out = np.empty(n, np.float32)
    _lib_synth().myos_synth_normal_f32(seed, stream, mean, std,
                                       out.ctypes.data_as(C.c_void_p), n, threads)
    return out


def prompt_ids(seed: int, n: int, vocab: int, stream: int = PROMPT_STREAM) -> np.ndarray:
    out = np.empty(n, np.uint32)
    _lib_synth().myos_synth_uniform_u32(seed, stream, vocab, out.ctypes.data_as(C.c_void_p), n)
    return out


def weights(shape: dict, seed: int, threads: int = 0) -> dict:
    """{name: (dims, little-endian bf16 bytes as uint8)} for the whole model."""
    table = {}
    for stream, (name, dims, is_norm) in enumerate(tensor_specs(shape)):
        n = int(np.prod(dims))
        if is_norm:
            data = normal_bf16(seed, stream, n, 1.0, 0.01, threads)
        else:
            data = normal_bf16(seed, stream, n, 0.0, 0.02, threads)
        table[name] = (tuple(dims), data.view(np.uint8))
    return table


def weight_bytes(shape: dict) -> int:
    return sum(2 * int(np.prod(d)) for _, d, _ in tensor_specs(shape))


def write_safetensors(path: str, tensors: dict, metadata: dict | None = None) -> None:
    """Write {name: (dims, bf16 bytes)} as a SafeTensors file (dtype BF16)."""
    header = {}
    off = 0
    names = list(tensors.keys())
    for name in names:
        dims, data = tensors[name]
        header[name] = {"dtype": "BF16", "shape": list(dims), "data_offsets": [off, off + data.nbytes]}
        off += data.nbytes
    if metadata:
        header["__metadata__"] = {k: str(v) for k, v in metadata.items()}
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for name in names:
            f.write(tensors[name][1].tobytes())
