#!/usr/bin/env python3
"""Benchmark: MyOS Qwen2.5 BF16 token loop on B200 (sm_100a).

Workload ("S1"): Qwen2.5-1.5B architecture with seeded
random-init BF16 weights, a 128-id uniform prompt, 128 greedy decode steps,
batch 1. A step is one S1 request: reset, prefill the prompt, decode 128.
Headline metric: decode tok/s (T_decode = n_gen / t_decode,
crates/runtime/src/meter.rs:48-78), with prefill tok/s and the HBM
roofline fraction beside it.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--n-prompt P --n-gen G]   (smaller cases for profiler captures)

N>1 runs one independent S1 replica per GPU (the path has no exchange
step: independent sequences, weak scaling), timed as the max over ranks.
``--impl reference`` times the reference's CPU ``--threads`` path (the C++
restatement under oracle/, bit-identical to it on the reference's own
known-answer tests) on the host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "an-operating-system-for-ai-models-and-tensor-inference_b200")
sys.path.insert(0, PKG)
sys.path.insert(0, REPO)

SEED = 1234
N_PROMPT, N_GEN = 128, 128
METRIC = "decode tok/s Qwen2.5-1.5B bf16 b=1; % HBM roofline; prefill tok/s"
PUBLISHED_DECODE = 15.4880  # reference T_decode, knife 9, 8 threads (CPU)


def measured_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ---------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9 or parts[0] != str(self.idx):
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- distributed
def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    pg = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
        pg = dist
    return world, rank, local, pg


def barrier(pg):
    if pg is not None:
        pg.barrier()


def max_over_ranks(pg, value: float, local: int) -> float:
    """The slowest rank's value (NCCL on the rank's GPU; gloo on the host)."""
    if pg is None:
        return value
    import torch

    dev = f"cuda:{local}" if pg.get_backend() == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    pg.all_reduce(t, op=pg.ReduceOp.MAX)
    return float(t.item())


def aggregate_tok_s(world: int, tokens_per_rank_step: int, steps: int, max_ms: float) -> float:
    """Whole-job throughput: every rank's tokens over the slowest rank's time."""
    return world * tokens_per_rank_step * steps / (max_ms / 1000.0)


# ---------------------------------------------------------------- CPU baseline
def cpu_decode_sample(shape, table, prompt, n_decode: int, threads: int, max_seq: int):
    """Reference --threads path (oracle restatement): prefill + n_decode greedy."""
    from oracle import oracle as orc
    sys.path.insert(0, os.path.join(REPO, "tests"))
    import ref_fixtures as rf

    orc.build()
    orc.set_threads(threads)
    wm = rf.load_into_oracle(orc, table)
    md = orc.Model(rf.oracle_shape(orc, shape), max_seq)
    t0 = time.perf_counter()
    assert md.prefill(wm, prompt) == 0
    t1 = time.perf_counter()
    st, ids, _, _ = md.greedy_decode(wm, n_decode)
    t2 = time.perf_counter()
    assert st == 0
    return {"t_prefill": t1 - t0, "t_decode": t2 - t1, "ids": ids}


def host_threads() -> int:
    try:
        n = len(os.sched_getaffinity(0))
    except Exception:
        n = os.cpu_count() or 1
    return max(1, min(n, 64))  # GEMV_THREADS_MAX


# ---------------------------------------------------------------- arms
def run_reference(args, world, rank):
    if rank != 0:
        return 0
    from myos import synth
    shape = synth.shape_qwen25_1_5b()
    threads = host_threads()
    table = synth.weights(shape, SEED, threads=threads)
    prompt = synth.prompt_ids(SEED, N_PROMPT, shape["vocab"])
    n_dec = args.ref_decode
    for _ in range(args.warmup):
        cpu_decode_sample(shape, table, prompt, 1, threads, N_PROMPT + N_GEN)
    samples = [cpu_decode_sample(shape, table, prompt, n_dec, threads, N_PROMPT + N_GEN)
               for _ in range(args.steps)]
    t_dec = sum(s["t_decode"] for s in samples)
    t_pre = sum(s["t_prefill"] for s in samples)
    value = n_dec * len(samples) / t_dec
    sample = (f"per step: prefill {N_PROMPT} ids + {n_dec} greedy decode steps of S1 "
              f"(of {N_GEN}); {threads} threads")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1000 * (t_dec + t_pre) / len(samples), 3),
        "higher_is_better": True, "scaling": "weak",
        "vs_baseline": round(value / PUBLISHED_DECODE, 4), "dtype": "bf16 weights, f32 compute",
        "data": "synthetic (seeded random-init Qwen2.5-1.5B weights, uniform prompt ids)",
        "config": {"workload": "S1: Qwen2.5-1.5B, 128-id prompt + 128 greedy steps, batch 1",
                   "seed": SEED, "parallelism": "cpu row-split threads"},
        "prefill_tok_s": round(N_PROMPT * len(samples) / t_pre, 3),
        "cpu_baseline": {"value": round(value, 4), "unit": "tok/s", "cores": threads,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


def run_ours(args, world, rank, local, pg):
    import numpy as np

    import build as pkg_build
    import myos
    from myos import synth

    if rank == 0 or not os.path.exists(os.path.join(PKG, "lib", "libmyos_cuda.so")):
        pkg_build.build()
    barrier(pg)
    shape = synth.shape_qwen25_1_5b()
    threads = max(1, host_threads() // max(world, 1))
    table = synth.weights(shape, SEED, threads=threads)
    n_prompt, n_gen = args.n_prompt, args.n_gen
    prompt = synth.prompt_ids(SEED, n_prompt, shape["vocab"])
    eng = myos.Engine(shape, n_prompt + n_gen, device=local, kv_dtype=args.kv)
    eng.load_table(table)

    def one_step():
        eng.reset()
        eng.prefill(prompt, want_logits=False)
        p_ms, _ = eng.last_timing()
        ids = eng.greedy_decode(n_gen)
        _, d_ms = eng.last_timing()
        return p_ms, d_ms, ids

    for _ in range(max(args.warmup, 3)):
        one_step()
    # device-timed region (CUDA events inside the library's stream)
    barrier(pg)
    clocks = ClockSampler(local)
    clocks.start()
    pre_ms, dec_ms = [], []
    ids = None
    for _ in range(args.steps):
        p, d, ids = one_step()
        pre_ms.append(p)
        dec_ms.append(d)
    clk = clocks.stop()
    barrier(pg)
    tot_dec = max_over_ranks(pg, sum(dec_ms), local)
    tot_pre = max_over_ranks(pg, sum(pre_ms), local)
    value = aggregate_tok_s(world, n_gen, args.steps, tot_dec)
    prefill_tps = aggregate_tok_s(world, n_prompt, args.steps, tot_pre)

    # end to end through the C ABI with host buffers: prompt ids in, ids out
    barrier(pg)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        eng.reset()
        eng.prefill(prompt, want_logits=False)
        eng.greedy_decode(n_gen)
    wall = max_over_ranks(pg, time.perf_counter() - t0, local)
    e2e = world * n_gen * args.steps / wall

    # dominant kernel (gate/up GEMV: ~60% of the weight bytes) timed alone
    eng.reset()
    eng.prefill(prompt, want_logits=False)
    prof = eng.profile_kernels(iters=3)
    peak, peak_kind = measured_peaks()
    gu_ms, gu_bytes = prof["gate_up"]
    achieved = gu_bytes / (gu_ms / 1000.0) / 1e9
    traffic = None
    tp = os.path.join(REPO, "profiles", "traffic.json")
    if os.path.exists(tp):
        traffic = json.load(open(tp)).get("gate_up_bytes_per_launch")
    step_bytes = synth.weight_bytes(shape)
    step_gbs = step_bytes * n_gen * args.steps / (sum(dec_ms) / 1000.0) / 1e9

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        t = host_threads()
        smp = cpu_decode_sample(shape, table, prompt, args.cpu_decode, t, n_prompt + n_gen)
        cpu = {"value": round(args.cpu_decode / smp["t_decode"], 4), "unit": "tok/s", "cores": t,
               "kind": "port",
               "sample": f"prefill {n_prompt} ids + {args.cpu_decode} greedy steps of S1 on the "
                         f"reference's --threads path restated in C++ (oracle/), {t} threads",
               "prefill_tok_s": round(n_prompt / smp["t_prefill"], 3),
               "ids_match_gpu_prefix": bool(np.array_equal(smp["ids"], ids[:args.cpu_decode]))}

    if rank == 0:
        launches_per_token = 5 * shape["num_layers"] + 1
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3),
            "ms_per_step": round((tot_pre + tot_dec) / args.steps, 3),
            "higher_is_better": True, "scaling": "weak",
            "vs_baseline": round(value / PUBLISHED_DECODE, 2),
            "dtype": "bf16 weights, f32 activations/accumulate",
            "data": "synthetic (seeded random-init Qwen2.5-1.5B BF16 weights, uniform prompt ids)",
            "config": {"workload": f"S1: Qwen2.5-1.5B, {n_prompt}-id prompt + {n_gen} greedy "
                                   f"steps, batch 1",
                       "seed": SEED, "kv_dtype": args.kv,
                       "parallelism": f"replicas x{world} (independent sequences)",
                       "l2": "each decode step streams 3.09 GB of weights (> 126 MB L2); no flush"},
            "prefill_tok_s": round(prefill_tps, 1),
            "decode_ms_per_token": round(tot_dec / (args.steps * n_gen), 4),
            "step_hbm": {"bytes_per_token": step_bytes, "achieved_gbs": round(step_gbs, 1),
                         "frac_of_measured": round(step_gbs / peak, 4),
                         "frac_of_8tbs_nominal": round(step_gbs / 8000.0, 4)},
            "roofline": {"bound": "hbm", "kernel": "gate_up GEMV (RMSNorm+gate|up+SiLU*up)",
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "peak_source": peak_kind,
                         "bytes_per_launch": gu_bytes, "ms_per_launch": round(gu_ms, 5)},
            "kernels": {k: {"ms": round(v[0], 5), "gbs": round(v[1] / (v[0] / 1000) / 1e9, 1)}
                        for k, v in prof.items()},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": n_prompt * 4,
                    "d2h_bytes_per_step": n_gen * 4,
                    "note": "generated tokens / wall time of reset+prefill(host ids)+"
                            "greedy_decode(host ids) through the C ABI"},
            "gpu_launches": launches_per_token * (n_prompt + n_gen) * args.steps,
            "clocks": clk,
        }
        print(json.dumps(line))
    eng.close()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--kv", choices=["f32", "bf16"], default="f32")
    ap.add_argument("--cpu-decode", type=int, default=16)
    ap.add_argument("--ref-decode", type=int, default=8)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--n-prompt", type=int, default=N_PROMPT)
    ap.add_argument("--n-gen", type=int, default=N_GEN)
    args = ap.parse_args()
    world, rank, local, pg = dist_setup(args) if args.impl == "ours" else (
        int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), 0, None)
    try:
        if args.impl == "reference":
            return run_reference(args, world, rank)
        return run_ours(args, world, rank, local, pg)
    finally:
        if pg is not None:
            pg.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
