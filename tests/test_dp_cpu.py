"""Data-parallel batched decode (myos.dp): the sequence sharding and the
rank-0 gather, on CPU with two gloo ranks (no GPU; the ids are stand-ins
built from the sequence index)."""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from myos import dp


def test_shards_are_contiguous_balanced_and_cover_every_sequence():
    for n, world in [(64, 1), (64, 2), (64, 3), (64, 8), (5, 8), (0, 2)]:
        parts = [dp.shard(n, world, r) for r in range(world)]
        assert [i for p in parts for i in p] == list(range(n))
        sizes = [len(p) for p in parts]
        assert max(sizes) - min(sizes) <= 1
        assert sizes == sorted(sizes, reverse=True)


def test_merge_rejects_a_missing_shard():
    with pytest.raises(ValueError):
        dp.merge([(0, np.zeros((3, 4), np.uint32))], 4, 4)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, n_seq, n_gen, q):
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        idx = dp.shard(n_seq, world, rank)
        ids = np.array([[1000 * b + s for s in range(n_gen)] for b in idx],
                       np.uint32).reshape(len(idx), n_gen)
        parts = [None] * world
        dist.all_gather_object(parts, (idx.start, ids))
        if rank == 0:
            q.put(dp.merge(parts, n_seq, n_gen))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n_seq", [64, 3])
def test_two_gloo_ranks_gather_ids_in_sequence_order(n_seq):
    n_gen = 5
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, n_seq, n_gen, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=120)
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    want = np.array([[1000 * b + s for s in range(n_gen)] for b in range(n_seq)], np.uint32)
    np.testing.assert_array_equal(got, want)
