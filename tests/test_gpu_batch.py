"""Batched greedy decode (BASELINE config 4's per-GPU path): independent
prompts of different lengths prefilled into their own KV slabs and decoded
together with GEMM projections (myos_batch_generate), against each prompt
decoded alone through the single-sequence API."""
import numpy as np
import pytest

import myos
from myos import synth

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
