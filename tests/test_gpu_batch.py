"""Batched greedy decode (BASELINE config 4's per-GPU path): independent
prompts of different lengths prefilled into their own KV slabs and decoded
together with GEMM projections (myos_batch_generate), against each prompt
decoded alone through the single-sequence API, and four of the config's 64
sequences (512-id prompts, 128 steps) against the oracle's answers for the
same seeded inputs (computed once on the CPU and committed:
tests/golden/batch_512.npz, tests/golden/make_goldens.py): free-running ids
before the first near-tie, teacher-forced argmaxes at every other step
(myos_batch_forced_decode) and final logits at the fixture's indices."""
import numpy as np
import pytest

import myos
from myos import synth
from golden import make_goldens as mg

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

SEED = 1234


@pytest.fixture(scope="module")
def engine():
    shape = synth.shape_qwen25_1_5b()
    table = synth.weights(shape, SEED)
    e = myos.Engine(shape, 256)
    e.load_table(table)
    yield shape, e
    e.close()


def test_batch_matches_single_sequences(engine):
    shape, e = engine
    lens = [5, 17, 64, 130, 1, 40]
    prompts = [synth.prompt_ids(SEED + 10 + i, n, shape["vocab"]) for i, n in enumerate(lens)]
    steps = 8
    got = e.batch_generate(prompts, steps)
    assert e.kv_len() == 0  # the context's own cursor is untouched
    for p, row in zip(prompts, got):
        e.reset()
        e.prefill(p, want_logits=False)
        want = e.greedy_decode(steps)
        assert row.tolist() == want.tolist(), (len(p), row, want)
    # a second call reuses the slabs and gives the same ids
    again = e.batch_generate(prompts, steps)
    assert np.array_equal(again, got)


def test_batch_errors_leave_state(engine):
    shape, e = engine
    before = e.kv_len()
    with pytest.raises(myos.MyosError) as ex:
        e.batch_generate([[1, 2, 3]] * 2, 254)  # 3 + 254 > 256 slots
    assert ex.value.code == myos._lib.ERR_CACHE_FULL
    with pytest.raises(myos.MyosError) as ex:
        e.batch_generate([[1, shape["vocab"]]], 2)
    assert ex.value.code == myos._lib.ERR_TOKEN
    with pytest.raises(myos.MyosError) as ex:
        e.batch_generate([[]], 2)
    assert ex.value.code == myos._lib.ERR_SHAPE
    assert e.kv_len() == before


def test_batch_against_oracle_golden():
    ATOL, RTOL = 1e-2, 1e-3
    g = mg.load("batch")
    shape = synth.shape_qwen25_1_5b()
    n_prompt, n_gen = int(g["n_prompt"]), int(g["n_gen"])
    prompts = [synth.prompt_ids(int(s), n_prompt, shape["vocab"]) for s in g["prompt_seeds"]]
    e = myos.Engine(shape, n_prompt + n_gen)
    e.load_table(synth.weights(shape, int(g["weight_seed"])))
    got = e.batch_generate(prompts, n_gen)
    am, lg = e.batch_forced(prompts, g["ids"], want_logits=True)
    for b in range(len(prompts)):
        ref, gap = g["ids"][b], g["gap"][b]
        first_close = next((i for i in range(n_gen) if gap[i] < ATOL), n_gen)
        diverge = next((i for i in range(n_gen) if got[b, i] != ref[i]), n_gen)
        assert diverge >= first_close, (b, diverge, first_close)
        bad = [i for i in range(n_gen) if am[b, i] != ref[i] and gap[i] >= ATOL]
        assert not bad, (b, bad)
        fi, fv = mg.sampled(g, "final", b)
        np.testing.assert_allclose(lg[b, fi], fv, atol=ATOL, rtol=RTOL)
    e.close()


def _batch64(table, shape, prompts, feed, graphs=True, env=None):
    import os
    saved = {k: os.environ.get(k) for k in (env or {})}
    os.environ.update(env or {})
    try:
        e = myos.Engine(shape, 64, use_graphs=graphs)
    finally:
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    try:
        e.load_table(table)
        ids = e.batch_generate(prompts, feed.shape[1])
        am, lg = e.batch_forced(prompts, feed, want_logits=True)
        return ids, am, lg
    finally:
        e.close()


def test_batch64_paths_agree():
    """64 sequences: 3 x 64 = 192 GEMM rows, the shape that runs on 64-row
    tiles with K slices and replays each step from a CUDA graph. Without the
    graph the kernels and their order are the same: bit-identical. 64-row
    and 128-row tiles without K slices sum every output in the same k order:
    bit-identical. K slices change the summation order: logits within
    1e-2 / 1e-3, teacher-forced argmaxes equal wherever the top-2 gap of the
    reference run exceeds the tolerance."""
    ATOL, RTOL = 1e-2, 1e-3
    shape = synth.shape_qwen25_1_5b()
    table = synth.weights(shape, SEED)
    prompts = [synth.prompt_ids(SEED + 100 + i, 9 + (i % 7), shape["vocab"]) for i in range(64)]
    steps = 5
    feed = np.stack([synth.prompt_ids(SEED + 300 + i, steps, shape["vocab"]) for i in range(64)])
    ids, am, lg = _batch64(table, shape, prompts, feed)
    ids_ng, am_ng, lg_ng = _batch64(table, shape, prompts, feed, graphs=False)
    assert np.array_equal(ids, ids_ng) and np.array_equal(am, am_ng)
    assert np.array_equal(lg.view(np.uint32), lg_ng.view(np.uint32))
    _, am1, lg1 = _batch64(table, shape, prompts, feed, env={"MYOS_SPLITK": "0"})
    _, am2, lg2 = _batch64(table, shape, prompts, feed,
                           env={"MYOS_SPLITK": "0", "MYOS_GEMM_M64": "0"})
    assert np.array_equal(am1, am2)
    assert np.array_equal(lg1.view(np.uint32), lg2.view(np.uint32))
    np.testing.assert_allclose(lg, lg1, atol=ATOL, rtol=RTOL)
    top2 = np.sort(lg1, axis=1)[:, -2:]
    close = (top2[:, 1] - top2[:, 0]) < ATOL
    assert all(am[b, -1] == am1[b, -1] or close[b] for b in range(64))
