"""ctypes binding of libmyos_cuda.so (the C ABI in include/myos_cuda.h).

The library is loaded from the package's lib/ directory; it is built by
``build.py``. There is no fallback: a missing library raises immediately.
"""
from __future__ import annotations

import ctypes as C
import os

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_DIR = os.path.join(PKG_DIR, "lib")
CUDA_LIB = os.path.join(LIB_DIR, "libmyos_cuda.so")
SYNTH_LIB = os.path.join(LIB_DIR, "libmyos_synth.so")

# enum myos_status
OK = 0
ERR_SHAPE, ERR_TOKEN, ERR_ROW_OOB, ERR_POSITION, ERR_CACHE_FULL, ERR_CACHE_RANGE = 1, 2, 3, 4, 5, 6
ERR_WEIGHT_MISSING, ERR_WEIGHT_DTYPE, ERR_WEIGHT_SHAPE, ERR_WEIGHT_LENGTH = 7, 8, 9, 10
ERR_DUPLICATE, ERR_EMPTY_NAME, ERR_PARSE, ERR_UNSUPPORTED, ERR_IO = 11, 12, 13, 14, 15
ERR_CUDA, ERR_NCCL, ERR_TIMEOUT, ERR_ARG, ERR_SCRATCH_LIMIT = 16, 17, 18, 19, 20
STATUS_NAMES = {
    0: "Ok", 1: "Shape", 2: "Token", 3: "RowOutOfBounds", 4: "Position", 5: "CacheFull",
    6: "CacheRange", 7: "WeightMissing", 8: "WeightDType", 9: "WeightShape", 10: "WeightLength",
    11: "Duplicate", 12: "EmptyName", 13: "Parse", 14: "UnsupportedDType", 15: "Io", 16: "Cuda",
    17: "Nccl", 18: "Timeout", 19: "Arg", 20: "ScratchLimit",
}
F32, F16, BF16 = 0, 1, 2
KV_F32, KV_BF16 = 0, 1

_f32p = C.POINTER(C.c_float)
_u8p = C.POINTER(C.c_uint8)
_u32p = C.POINTER(C.c_uint32)
_i64p = C.POINTER(C.c_int64)
_szp = C.POINTER(C.c_size_t)
sz = C.c_size_t


class Shape(C.Structure):
    """myos_shape: BlockShape + AttnShape (qwen25_block.rs:53-75, attn_wire.rs:44-63)."""
    _fields_ = [
        ("hidden", C.c_uint32),
        ("num_q_heads", C.c_uint32),
        ("num_kv_heads", C.c_uint32),
        ("head_dim", C.c_uint32),
        ("rope_theta", C.c_float),
        ("intermediate", C.c_uint32),
        ("vocab", C.c_uint32),
        ("num_layers", C.c_uint32),
        ("rms_eps", C.c_float),
        ("tied_head", C.c_uint32),
    ]

    def as_dict(self) -> dict:
        return {k: getattr(self, k) for k, _ in self._fields_}


class Opts(C.Structure):
    _fields_ = [
        ("device", C.c_int32),
        ("max_seq", C.c_uint32),
        ("kv_dtype", C.c_int32),
        ("use_graphs", C.c_int32),
    ]


class TP(C.Structure):
    """myos_tp: one rank of a tensor-parallel group."""
    _fields_ = [
        ("size", C.c_int32),
        ("rank", C.c_int32),
        ("unique_id", C.c_uint8 * 128),
    ]


class TPPart(C.Structure):
    """myos_tp_part: how a tensor-parallel rank holds one tensor."""
    _fields_ = [(n, C.c_uint64) for n in ("rows", "cols", "row0", "nrows", "col0", "ncols",
                                          "store_rows", "store_cols")] + [
        ("matrix", C.c_int32),
        ("kept", C.c_int32),
    ]


# Every symbol include/myos_cuda.h declares, with (restype, argtypes).
SIGNATURES = {
    "myos_version": (C.c_char_p, []),
    "myos_shape_qwen25_1_5b": (Shape, []),
    "myos_shape_qwen25_14b": (Shape, []),
    "myos_ctx_create": (C.c_int, [C.POINTER(Shape), C.POINTER(Opts), C.POINTER(C.c_void_p)]),
    "myos_ctx_create_tp": (C.c_int, [C.POINTER(Shape), C.POINTER(Opts), C.POINTER(TP),
                                      C.POINTER(C.c_void_p)]),
    "myos_tp_unique_id": (C.c_int, [_u8p]),
    "myos_tp_slice": (C.c_int, [C.POINTER(Shape), C.c_int32, C.c_int32, C.c_char_p,
                                C.POINTER(TPPart)]),
    "myos_tp_reduce_selftest": (C.c_int, [C.c_int32, C.c_uint32, C.c_uint32, C.c_int32,
                                          C.c_uint32, _f32p]),
    "myos_ctx_destroy": (None, [C.c_void_p]),
    "myos_last_error": (C.c_char_p, [C.c_void_p]),
    "myos_load_tensor": (C.c_int, [C.c_void_p, C.c_char_p, C.c_int32, _i64p, C.c_int32,
                                   C.c_void_p, sz]),
    "myos_load_safetensors": (C.c_int, [C.c_void_p, C.c_char_p]),
    "myos_check_safetensors": (C.c_int, [C.c_char_p, _szp, C.c_char_p, sz]),
    "myos_weights_ready": (C.c_int, [C.c_void_p]),
    "myos_prefill": (C.c_int, [C.c_void_p, _u32p, sz, _f32p]),
    "myos_forward_token": (C.c_int, [C.c_void_p, C.c_uint32, sz, _f32p]),
    "myos_greedy_decode": (C.c_int, [C.c_void_p, sz, _u32p]),
    "myos_forced_decode": (C.c_int, [C.c_void_p, _u32p, sz, _u32p]),
    "myos_kv_len": (C.c_int, [C.c_void_p, _szp]),
    "myos_reset": (C.c_int, [C.c_void_p]),
    "myos_kv_head": (C.c_int, [C.c_void_p, C.c_uint32, C.c_uint32, sz, _f32p, _f32p]),
    "myos_logits": (C.c_int, [C.c_void_p, _f32p]),
    "myos_last_timing": (C.c_int, [C.c_void_p, _f32p, _f32p]),
    "myos_launch_count": (C.c_int, [C.POINTER(C.c_uint64)]),
    "myos_profile_kernels": (C.c_int, [C.c_void_p, C.c_int, _f32p, C.POINTER(C.c_double)]),
    "myos_gemv_bf16": (C.c_int, [_f32p, sz, _u8p, sz, _f32p, sz, sz, sz]),
    "myos_rmsnorm_bf16_weight": (C.c_int, [_f32p, sz, _u8p, sz, _f32p, sz, C.c_float]),
    "myos_gqa_attn_f32": (C.c_int, [_f32p, sz, _f32p, sz, _f32p, sz, _f32p, sz, sz, sz, sz, sz,
                                    C.c_int32, sz]),
    "myos_swiglu_mul_f32": (C.c_int, [_f32p, sz, _f32p, sz, _f32p, sz]),
    "myos_rope_f32": (C.c_int, [_f32p, sz, _f32p, sz, C.c_uint32, sz, C.c_float]),
    "myos_greedy_token": (C.c_int, [_f32p, sz, _u32p]),
    "myos_dev_gemv_bf16": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, sz, sz, C.c_void_p]),
    "myos_batch_generate": (C.c_int, [C.c_void_p, sz, _u32p, _u32p, sz, _u32p]),
    "myos_batch_forced_decode": (C.c_int, [C.c_void_p, sz, _u32p, _u32p, sz, _u32p, _u32p, _f32p]),
    "myos_dev_gqa_attn_f32_noalloc": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                                sz, sz, sz, sz, C.c_int32, sz, C.c_void_p]),
}

_lib = None


def load():
    """Load libmyos_cuda.so. Raises if the library was not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(CUDA_LIB):
            raise RuntimeError(
                f"{CUDA_LIB} is missing: build it with python build.py (nvcc, sm_100a)")
        L = C.CDLL(CUDA_LIB)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def status_name(code: int) -> str:
    return STATUS_NAMES.get(code, f"status {code}")


class MyosError(RuntimeError):
    def __init__(self, code: int, msg: str = ""):
        super().__init__(f"{status_name(code)}: {msg}" if msg else status_name(code))
        self.code = code
