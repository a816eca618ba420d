"""bench.py's multi-GPU host logic on CPU: two gloo ranks (world_size 2) time
different amounts of work; the reported figure uses the slowest rank's time
and every rank's tokens (weak scaling, one independent S1 replica per rank)."""
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    import datetime
    import sys
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, repo)
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        bench.barrier(dist)
        ms = 100.0 + 50.0 * rank  # rank 1 is the slow one
        worst = bench.max_over_ranks(dist, ms, 0)
        q.put((rank, worst, bench.aggregate_tok_s(world, 128, 5, worst)))
        bench.barrier(dist)
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_take_the_slowest_time():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    got = sorted(q.get(timeout=10) for _ in range(2))
    for rank, worst, agg in got:
        assert worst == 150.0
        assert agg == pytest.approx(2 * 128 * 5 / 0.150)
