"""myos — B200 (sm_100a) Qwen2.5 BF16 token loop behind the MyOS C ABI.

The numeric path is libmyos_cuda.so (CUDA kernels); this package only
binds it with ctypes and mirrors the reference's crate APIs:

  myos.engine   model_core: Engine.prefill / forward_token / greedy_decode / KV access
  myos.ops      tensor_core operators on host arrays (run on the GPU)
  myos.synth    seeded synthetic weights and prompts for the benchmark configs
  myos.tp       tensor-parallel generation, one process per GPU (torchrun)
"""
from . import _lib
from ._lib import MyosError, status_name
from .engine import Engine, check_safetensors, greedy_token, shape_from_dict, tp_unique_id

__all__ = ["Engine", "MyosError", "check_safetensors", "greedy_token", "shape_from_dict",
           "status_name", "tp_unique_id", "_lib"]
