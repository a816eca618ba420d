"""Many independent sequences over several GPUs (data parallel): one process
per GPU, each rank decodes its share of the sequences with
``Engine.batch_generate`` (myos_batch_generate: tensor-core prefill into
per-sequence KV slabs, then all of its sequences' steps as GEMMs), and rank 0
gathers the ids in sequence order. Weights are replicated; nothing crosses
GPUs on the data path, only the ids at the end (host side, gloo).

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \\
        -m myos.dp --n-seq 64 --n-prompt 512 --n-gen 128

The reference decodes the sequences one after another
(crates/runtime/src/main.rs, batch 1); this is BASELINE's batched config
sharded by sequence. Prompt b is ``synth.prompt_ids(seed + b, n_prompt,
vocab)`` (seeded, uniform ids), so any sharding sees the same prompts.
"""
from __future__ import annotations

import argparse
import json
import os

import numpy as np

from . import synth


def shard(n_seq: int, world: int, rank: int) -> range:
    """Contiguous, balanced block of sequence indices for `rank` (sizes
    differ by at most one; the first n_seq % world ranks take one more)."""
    base, extra = divmod(n_seq, world)
    lo = rank * base + min(rank, extra)
    return range(lo, lo + base + (1 if rank < extra else 0))


def merge(parts, n_seq: int, n_gen: int) -> np.ndarray:
    """Rank-ordered [(first sequence index, ids[k, n_gen])] -> ids[n_seq, n_gen]."""
    out = np.zeros((n_seq, n_gen), np.uint32)
    seen = 0
    for first, ids in parts:
        ids = np.asarray(ids, np.uint32).reshape(-1, n_gen)
        out[first:first + len(ids)] = ids
        seen += len(ids)
    if seen != n_seq:
        raise ValueError("gathered %d sequences, expected %d" % (seen, n_seq))
    return out


def prompts_for(idx: range, n_prompt: int, vocab: int, seed: int):
    return [synth.prompt_ids(seed + b, n_prompt, vocab) for b in idx]


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--n-seq", type=int, default=64)
    ap.add_argument("--n-prompt", type=int, default=512)
    ap.add_argument("--n-gen", type=int, default=128)
    ap.add_argument("--seed", type=int, default=5000)
    ap.add_argument("--weight-seed", type=int, default=1234)
    ap.add_argument("--iters", type=int, default=2)
    args = ap.parse_args()

    from datetime import timedelta

    import torch
    import torch.distributed as dist

    from .engine import Engine
    from .tp import load_synth

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=900))
    shape = synth.shape_qwen25_1_5b()
    idx = shard(args.n_seq, world, rank)
    prompts = prompts_for(idx, args.n_prompt, shape["vocab"], args.seed)
    e = Engine(shape, args.n_prompt + args.n_gen, device=local)
    try:
        load_synth(e, shape, args.weight_seed, max(1, (os.cpu_count() or 2) // world))
        if len(idx):
            e.batch_generate(prompts[:1], 2)  # first-use allocations
        ms = []
        for _ in range(args.iters):
            dist.barrier()
            ids = e.batch_generate(prompts, args.n_gen) if len(idx) else \
                np.zeros((0, args.n_gen), np.uint32)
            ms.append(e.last_timing()[1] if len(idx) else 0.0)
    finally:
        e.close()
    t = torch.tensor([ms[-1]], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    parts = [None] * world
    dist.all_gather_object(parts, (idx.start, ids))
    if rank == 0:
        all_ids = merge(parts, args.n_seq, args.n_gen)
        worst = float(t[0])
        print(json.dumps({
            "model": "qwen2.5-1.5b", "gpus": world, "n_seq": args.n_seq,
            "n_prompt": args.n_prompt, "n_gen": args.n_gen,
            "generated_tok_s": round(args.n_seq * args.n_gen / (worst / 1e3), 1),
            "ms_slowest_rank": round(worst, 1),
            "ids_first": [int(x) for x in all_ids[0, :4]],
            "data": "synthetic seeded weights and prompts",
            "timing": "cuda events around each rank's batch call (prefill included), max over ranks"}),
            flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
