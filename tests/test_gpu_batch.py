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
