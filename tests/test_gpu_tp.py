"""Tensor parallelism over two GPUs (one process per GPU): Qwen2.5-1.5B with
seeded random-init BF16 weights, a 136-id prompt (two tensor-core prefill
chunks, 128 + 8) and 24 greedy steps, against the oracle under the same pass
rule as the single-GPU test (greedy ids equal the oracle's before the first
step whose top-2 gap is below tolerance; teacher-forced argmax equal
wherever the gap is not; logits within 1e-2 absolute / 1e-3 relative, the
bf16 KV cache's wider bound for that cache). Both ranks must also return
identical ids and logits. Two exchange modes: peer-memory pushes (f32 KV)
and NCCL collectives (bf16 KV).

The split (heads, MLP columns padded 4480 -> 4608, vocabulary rows) sums
the projections' partial results across ranks, so the order of the f32
additions differs from one GPU's; the tolerance covers that.
"""
import multiprocessing as mp

import numpy as np
import pytest

from myos import synth

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

SEED = 1234
N_PROMPT, N_GEN = 136, 24
ATOL, RTOL = 1e-2, 1e-3
TOL = {"f32": (ATOL, RTOL), "bf16": (6e-2, 6e-3)}
TIMEOUT_S = 900


def _gpu_count() -> int:
    import torch
    return torch.cuda.device_count()


def _rank(q, idq, size, rank, shape, forced, comm, kv, n_prompt=N_PROMPT, n_gen=N_GEN):
    import os
    if comm:
        os.environ["MYOS_TP_COMM"] = comm
    from myos import tp
    try:
        # rank 0 makes the rendezvous id in its own process (its NCCL hosts
        # the bootstrap root) and hands it to the other ranks
        if rank == 0:
            uid = tp.tp_unique_id()
            for _ in range(size - 1):
                idq.put(uid)
        else:
            uid = idq.get(timeout=TIMEOUT_S)
        q.put((rank, tp.run_rank(size, rank, uid, shape, SEED, n_prompt, n_gen, kv=kv,
                                 forced=forced)))
    except Exception as ex:  # reported by the parent
        q.put((rank, repr(ex)))


@pytest.fixture(scope="module")
def golden(orc):
    if _gpu_count() < 2:
        pytest.skip("tensor parallelism needs two GPUs")
    import ref_fixtures as rf
    shape = synth.shape_qwen25_1_5b()
    table = synth.weights(shape, SEED)
    prompt = synth.prompt_ids(SEED, N_PROMPT, shape["vocab"])
    wm = rf.load_into_oracle(orc, table)
    md = orc.Model(rf.oracle_shape(orc, shape), N_PROMPT + N_GEN)
    assert md.prefill(wm, prompt) == 0
    pre = md.logits()
    st, ids, gap, _ = md.greedy_decode(wm, N_GEN)
    assert st == 0
    return shape, dict(prefill=pre, ids=np.asarray(ids), gap=np.asarray(gap), final=md.logits())


def _run_ranks(shape, forced, comm, kv, n_prompt, n_gen):
    ctx = mp.get_context("spawn")
    q, idq = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(q, idq, 2, r, shape, forced, comm, kv, n_prompt,
                                             n_gen)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in procs:
            rank, out = q.get(timeout=TIMEOUT_S)
            res[rank] = out
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in (0, 1):
        assert isinstance(res[r], dict), res[r]
    a, b = res[0], res[1]
    for k in ("prefill", "ids", "final", "forced_argmax", "forced_final"):
        np.testing.assert_array_equal(a[k], b[k], err_msg=k)
    return a


def _check(a, g, atol, rtol, n_gen):
    np.testing.assert_allclose(a["prefill"], g["prefill"], atol=atol, rtol=rtol)
    ref, gap = g["ids"], g["gap"]
    first_close = next((i for i in range(n_gen) if gap[i] < atol), n_gen)
    diverge = next((i for i in range(n_gen) if a["ids"][i] != ref[i]), n_gen)
    assert diverge >= first_close, (diverge, first_close)
    if diverge == n_gen:
        np.testing.assert_allclose(a["final"], g["final"], atol=atol, rtol=rtol)
    bad = [i for i in range(n_gen) if a["forced_argmax"][i] != ref[i] and gap[i] >= atol]
    assert not bad, bad
    np.testing.assert_allclose(a["forced_final"], g["final"], atol=atol, rtol=rtol)


@pytest.mark.parametrize("comm,kv", [("", "f32"), ("nccl", "bf16")])
def test_tp2_matches_oracle(golden, comm, kv):
    shape, g = golden
    atol, rtol = TOL[kv]
    a = _run_ranks(shape, g["ids"], comm, kv, N_PROMPT, N_GEN)
    _check(a, g, atol, rtol, N_GEN)


def test_tp2_padded_slices_match_oracle(orc):
    """A shape whose per-rank slices need the zero padding: 10 q heads over
    2 ranks is 5 x 128 = 640 o_proj input columns (padded to 768), and
    intermediate 3456 / 2 = 1728 MLP rows (padded to 1792); 14B at 8 ranks
    needs the same o_proj padding."""
    if _gpu_count() < 2:
        pytest.skip("tensor parallelism needs two GPUs")
    import ref_fixtures as rf
    shape = dict(hidden=1280, num_q_heads=10, num_kv_heads=2, head_dim=128, rope_theta=1e6,
                 intermediate=3456, vocab=32000, num_layers=4, rms_eps=1e-6, tied_head=True)
    n_prompt, n_gen = 40, 16
    table = synth.weights(shape, SEED)
    prompt = synth.prompt_ids(SEED, n_prompt, shape["vocab"])
    wm = rf.load_into_oracle(orc, table)
    md = orc.Model(rf.oracle_shape(orc, shape), n_prompt + n_gen)
    assert md.prefill(wm, prompt) == 0
    pre = md.logits()
    st, ids, gap, _ = md.greedy_decode(wm, n_gen)
    assert st == 0
    g = dict(prefill=pre, ids=np.asarray(ids), gap=np.asarray(gap), final=md.logits())
    a = _run_ranks(shape, g["ids"], "", "f32", n_prompt, n_gen)
    _check(a, g, ATOL, RTOL, n_gen)
