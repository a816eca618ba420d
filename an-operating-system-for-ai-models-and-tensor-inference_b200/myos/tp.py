"""Tensor-parallel generation: one process per GPU, each rank an
``Engine(tp=(size, rank, id))`` that holds its slice of the model.

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \\
        -m myos.tp --model 14b --n-prompt 512 --n-gen 128

Rank 0 makes the NCCL rendezvous id (myos_tp_unique_id) and hands it to the
other ranks through a host-side gloo group; every rank then streams the
seeded synthetic weights in whole, one tensor at a time, and the library
keeps that rank's slice. Rank 0 prints one JSON line: prefill and greedy
decode throughput timed on the device (CUDA events inside the library around
each call), the max over ranks, and the greedy ids' head.

The reference runs one process on one device (crates/runtime/src/main.rs);
this is the sharded form of its token loop for models whose weights and
step time want more than one GPU (Qwen2.5-14B).
"""
from __future__ import annotations

import argparse
import json
import os

import numpy as np

from . import synth
from .engine import Engine, tp_unique_id


def reduce_selftest(n: int, H: int, fill: bool, timeout_ms: int = 1000, device: int = 0):
    """myos_tp_reduce_selftest: (status, sums or None) of the exchange's
    reduce kernel over a host-filled (or never-written) inbox on one GPU."""
    from . import _lib
    import ctypes as C
    L = _lib.load()
    out = np.zeros(H, np.float32)
    st = L.myos_tp_reduce_selftest(int(device), int(n), int(H), 1 if fill else 0,
                                   int(timeout_ms), out.ctypes.data_as(C.POINTER(C.c_float)))
    return st, (out if fill else None)


def slice_of(shape: dict, size: int, rank: int, name: str):
    """myos_tp_slice: how rank `rank` of `size` holds tensor `name` (a
    myos_tp_part with rows, cols, row0, nrows, col0, ncols, store_rows,
    store_cols, matrix, kept)."""
    from . import _lib
    import ctypes as C
    L = _lib.load()
    part = _lib.TPPart()
    from .engine import shape_from_dict
    st = L.myos_tp_slice(C.byref(shape_from_dict(shape)), int(size), int(rank),
                         name.encode(), C.byref(part))
    if st != 0:
        raise ValueError("myos_tp_slice(%s, %d, %d) failed: %d" % (name, size, rank, st))
    return part


def load_synth(e: Engine, shape: dict, seed: int, threads: int = 0, size: int = 1,
               rank: int = 0) -> None:
    """The seeded weights of ``synth.weights`` one tensor at a time (host
    memory: the largest tensor, not the model). With size > 1 only the block
    of each tensor that this rank keeps (myos_tp_slice) is generated; the
    library reads nothing else of the buffer it is given."""
    for stream, (name, dims, is_norm) in enumerate(synth.tensor_specs(shape)):
        mean, std = (1.0, 0.01) if is_norm else (0.0, 0.02)
        if size > 1:
            p = slice_of(shape, size, rank, name)
            if not p.kept:
                continue
            data = synth.normal_bf16_block(seed, stream, p.rows, p.cols, p.row0, p.nrows,
                                           p.col0, p.ncols, mean, std, threads)
        else:
            data = synth.normal_bf16(seed, stream, int(np.prod(dims)), mean, std, threads)
        e.load_tensor(name, tuple(dims), data.view(np.uint8))


def run_rank(size: int, rank: int, uid: bytes, shape: dict, seed: int, n_prompt: int,
             n_gen: int, kv: str = "f32", forced=None, iters: int = 1, device: int | None = None,
             threads: int = 0) -> dict:
    """One rank's share of: prefill(prompt), greedy_decode(n_gen), logits;
    then (forced given) reset, prefill, forced_decode(forced), logits.
    Every rank must call this with the same arguments but its own rank."""
    prompt = synth.prompt_ids(seed, n_prompt, shape["vocab"])
    e = Engine(shape, n_prompt + n_gen, device=rank if device is None else device, kv_dtype=kv,
               tp=(size, rank, uid))
    try:
        load_synth(e, shape, seed, threads, size, rank)
        out = {"prefill_ms": [], "decode_ms": []}
        for it in range(iters):
            e.reset()
            pl = e.prefill(prompt)
            p_ms, _ = e.last_timing()
            ids = e.greedy_decode(n_gen)
            _, d_ms = e.last_timing()
            out["prefill_ms"].append(p_ms)
            out["decode_ms"].append(d_ms)
        out.update(prefill=pl, ids=ids, final=e.logits())
        if forced is not None:
            e.reset()
            e.prefill(prompt, want_logits=False)
            out["forced_argmax"] = e.forced_decode(np.asarray(forced, np.uint32))
            out["forced_final"] = e.logits()
        return out
    finally:
        e.close()


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--model", choices=["1.5b", "14b"], default="14b")
    ap.add_argument("--n-prompt", type=int, default=512)
    ap.add_argument("--n-gen", type=int, default=128)
    ap.add_argument("--kv", choices=["f32", "bf16"], default="f32")
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--ktrace", default="",
                    help="write each rank's launch timeline of the last call to PREFIX_r<rank>.bin "
                         "(MYOS_KTRACE_FILE; keep --n-gen <= 64, see myos.ktrace)")
    args = ap.parse_args()

    import torch.distributed as dist
    from datetime import timedelta

    rank = int(os.environ.get("RANK", "0"))
    size = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    if args.ktrace:
        os.environ["MYOS_KTRACE_FILE"] = "%s_r%d.bin" % (args.ktrace, rank)
    dist.init_process_group("gloo", rank=rank, world_size=size, timeout=timedelta(seconds=600))
    box = [tp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    shape = synth.shape_qwen25_14b() if args.model == "14b" else synth.shape_qwen25_1_5b()
    r = run_rank(size, rank, box[0], shape, args.seed, args.n_prompt, args.n_gen, args.kv,
                 iters=args.iters, device=local, threads=max(1, (os.cpu_count() or 2) // size))
    # the last iteration (graphs captured, caches warm), max over ranks
    import torch
    t = torch.tensor([r["prefill_ms"][-1], r["decode_ms"][-1]], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if rank == 0:
        p_ms, d_ms = float(t[0]), float(t[1])
        print(json.dumps({
            "model": "qwen2.5-" + args.model, "tp": size, "kv": args.kv,
            "n_prompt": args.n_prompt, "n_gen": args.n_gen,
            "prefill_tok_s": round(args.n_prompt / (p_ms / 1e3), 1),
            "decode_tok_s": round(args.n_gen / (d_ms / 1e3), 1),
            "decode_ms_per_token": round(d_ms / args.n_gen, 3),
            "decode_ms_all_iters": [round(x, 2) for x in r["decode_ms"]],
            "ids_head": [int(x) for x in r["ids"][:8]],
            "data": "synthetic seeded weights", "timing": "cuda events, max over ranks"}),
            flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
