"""Qwen2.5-14B architecture on one B200 (tensor-parallel
size 1): seeded random-init BF16 weights with an untied lm_head, an 8-id
prompt through the GEMM prefill, 4 greedy steps, against the oracle.

The reference has no untied head (its forward_token always uses
embed_tokens, qwen25_block.rs:290-301); the oracle applies the same GEMV
semantics to lm_head.weight, so this comparison is parity-unpinned for the
head and pinned for everything before it."""
import numpy as np
import pytest

import myos
from myos import synth

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

SEED = 1234
ATOL, RTOL = 1e-2, 1e-3


def test_14b_tp1_greedy_and_logits(orc):
    import ref_fixtures as rf
    shape = synth.shape_qwen25_14b()
    table = synth.weights(shape, SEED)
    prompt = synth.prompt_ids(SEED, 8, shape["vocab"])
    n_gen = 4
    wm = rf.load_into_oracle(orc, table)
    md = orc.Model(rf.oracle_shape(orc, shape), len(prompt) + n_gen)
    assert md.prefill(wm, prompt) == 0
    pre = md.logits()
    st, ref, gap, _ = md.greedy_decode(wm, n_gen)
    assert st == 0
    final = md.logits()

    e = myos.Engine(shape, len(prompt) + n_gen)
    e.load_table(table)
    np.testing.assert_allclose(e.prefill(prompt), pre, atol=ATOL, rtol=RTOL)
    ids = e.greedy_decode(n_gen)
    first_close = next((i for i in range(n_gen) if gap[i] < ATOL), n_gen)
    diverge = next((i for i in range(n_gen) if ids[i] != ref[i]), n_gen)
    assert diverge >= first_close, (ids, ref)
    if diverge == n_gen:
        np.testing.assert_allclose(e.logits(), final, atol=ATOL, rtol=RTOL)
    e.close()
