"""Fixed workloads of the tensor-core (GEMM) path for launch-list and ncu
captures, on seeded synthetic Qwen2.5-1.5B weights.

    python -m myos.profile_workloads decode NGEN
        S1: a 128-id prompt, one warm greedy decode of NGEN steps, then the
        measured one (token steps replayed from CUDA graphs)
    python -m myos.profile_workloads prefill
        three warm 128-id prefills, then the measured one
    python -m myos.profile_workloads batched NSEQ NPROMPT NGEN
        one warm batched call without decode steps, then the measured call
        (NSEQ prompts of NPROMPT ids, NGEN greedy steps)

Each prints `skip=S count=C ...`: S kernels were enqueued before the
measured part and C inside it (myos_launch_count; graph replays count their
kernels), the values for ncu's -s and -c. For `batched` the measured part is
the decode steps of the second call (its prompts are skipped too).
"""
from __future__ import annotations

import ctypes
import sys

from . import Engine, _lib, dp, synth


def _count() -> int:
    v = ctypes.c_uint64()
    _lib.load().myos_launch_count(ctypes.byref(v))
    return v.value


def prefill() -> None:
    shape = synth.shape_qwen25_1_5b()
    e = Engine(shape, 256)
    try:
        e.load_table(synth.weights(shape, 1234))
        prompt = synth.prompt_ids(1234, 128, shape["vocab"])
        for _ in range(3):
            e.reset()
            e.prefill(prompt, want_logits=False)
        c0 = _count()
        e.reset()
        e.prefill(prompt, want_logits=False)
        c1 = _count()
        print(f"skip={c0} count={c1 - c0} prefill_ms={e.last_timing()[0]:.3f}", flush=True)
    finally:
        e.close()


def decode(ngen: int) -> None:
    shape = synth.shape_qwen25_1_5b()
    e = Engine(shape, 128 + 2 * ngen)
    try:
        e.load_table(synth.weights(shape, 1234))
        prompt = synth.prompt_ids(1234, 128, shape["vocab"])
        e.reset()
        e.prefill(prompt, want_logits=False)
        e.greedy_decode(ngen)
        e.reset()
        e.prefill(prompt, want_logits=False)
        c0 = _count()
        e.greedy_decode(ngen)
        c1 = _count()
        _, d_ms = e.last_timing()
        print(f"skip={c0} count={c1 - c0} decode_ms_per_token={d_ms / max(ngen, 1):.4f}", flush=True)
    finally:
        e.close()


def batched(nseq: int, nprompt: int, ngen: int) -> None:
    shape = synth.shape_qwen25_1_5b()
    e = Engine(shape, max(256, nprompt + ngen))
    try:
        e.load_table(synth.weights(shape, 1234))
        prompts = dp.prompts_for(range(nseq), nprompt, shape["vocab"], 5000)
        c0 = _count()
        e.batch_generate(prompts, 0)  # prompts and the first head only
        c1 = _count()
        e.batch_generate(prompts, ngen)
        c2 = _count()
        per_call = c1 - c0
        _, d_ms = e.last_timing()
        print(f"skip={c1 + per_call} count={c2 - c1 - per_call} "
              f"decode_ms_per_step={d_ms / max(ngen, 1):.3f}", flush=True)
    finally:
        e.close()


def main(argv) -> int:
    if len(argv) == 2 and argv[0] == "decode":
        decode(int(argv[1]))
        return 0
    if len(argv) >= 1 and argv[0] == "prefill":
        prefill()
        return 0
    if len(argv) == 4 and argv[0] == "batched":
        batched(int(argv[1]), int(argv[2]), int(argv[3]))
        return 0
    sys.stderr.write(__doc__)
    return 2


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
