"""Per-kernel launch timeline of the token step (MYOS_KTRACE_FILE).

With ``MYOS_KTRACE_FILE=path`` set when a context is created, the per-kernel
step records %globaltimer stamps for every kernel of the last call: per
(step mod 64, slot) eight u64 fields, slot = 5 * layer + {qkv, attention,
o_proj, gate_up, down} and 5 * layers for the head; field 0 is the earliest
block start, 1 the earliest return from the programmatic-dependency wait,
2 the latest block end, 3..7 stage marks. Calls longer than 64 steps wrap
(step mod 64), so trace a call of at most 64 steps.

    python -m myos.ktrace trace.bin --layers 48

prints, per kernel kind, the mean over steps 8..55 of: the gap from the
previous kernel's last block end to this kernel's first return from its
wait (launch, dependency release and, under tensor parallelism, the
exchange between the two), the run time (first wait return to last end)
and the pre-wait prologue (first start to first wait return).
"""
from __future__ import annotations

import argparse
import json

import numpy as np

STEPS, WIDTH = 64, 8
KINDS = ["qkv", "attention", "o_proj", "gate_up", "down"]


def summarize(path: str, layers: int, first: int = 8, last: int = 56) -> dict:
    ns = 5 * layers + 1
    t = np.fromfile(path, dtype=np.uint64).reshape(STEPS, ns, WIDTH).astype(np.float64)
    agg = {k: np.zeros(3) for k in KINDS + ["head"]}
    for st in range(first, last):
        r = t[st]
        prev_end = None
        for sl in range(ns):
            k = KINDS[sl % 5] if sl < 5 * layers else "head"
            start, wait, end = r[sl, 0], r[sl, 1], r[sl, 2]
            if end == 0:  # no launch in this slot (down_proj inside the fused MLP)
                continue
            gap = wait - prev_end if prev_end is not None else 0.0
            agg[k] += [gap, end - wait, wait - start]
            prev_end = end
    n = last - first
    out = {"token_us": float(np.mean([t[s + 1, 0, 1] - t[s, 0, 1]
                                      for s in range(first, last)]) / 1e3)}
    for k, v in agg.items():
        if not v.any():
            continue
        per = n * (layers if k != "head" else 1)
        out[k] = {"gap_us": round(v[0] / per / 1e3, 2), "run_us": round(v[1] / per / 1e3, 2),
                  "prewait_us": round(v[2] / per / 1e3, 2)}
    return out


def main() -> None:
    ap = argparse.ArgumentParser(description="summarize a MYOS_KTRACE_FILE timeline")
    ap.add_argument("path")
    ap.add_argument("--layers", type=int, default=28)
    args = ap.parse_args()
    print(json.dumps(summarize(args.path, args.layers), indent=1))


if __name__ == "__main__":
    main()
