"""Qwen2.5-14B architecture on one B200 (tensor-parallel
size 1): seeded random-init BF16 weights with an untied lm_head, a 512-id
prompt through the GEMM prefill, 16 greedy steps, against the oracle's
answers for the same seeded inputs (computed once on the CPU and committed:
tests/golden/q14b_512.npz, tests/golden/make_goldens.py).

The reference has no untied head (its forward_token always uses
embed_tokens, qwen25_block.rs:290-301); the oracle applies the same GEMV
semantics to lm_head.weight, so this comparison is parity-unpinned for the
head and pinned for everything before it."""
import numpy as np
import pytest

import myos
from myos import synth
from golden import make_goldens as mg

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

SEED = 1234
ATOL, RTOL = 1e-2, 1e-3


def test_14b_512_against_oracle_golden():
    g = mg.load("q14b")
    shape = synth.shape_qwen25_14b()
    table = synth.weights(shape, int(g["weight_seed"]))
    n_prompt, n_gen = int(g["n_prompt"]), int(g["n_gen"])
    prompt = synth.prompt_ids(int(g["prompt_seeds"][0]), n_prompt, shape["vocab"])
    ref, gap = g["ids"][0], g["gap"][0]
    e = myos.Engine(shape, n_prompt + n_gen)
    e.load_table(table)
    del table
    pi, pv = mg.sampled(g, "prefill", 0)
    np.testing.assert_allclose(e.prefill(prompt)[pi], pv, atol=ATOL, rtol=RTOL)
    ids = e.greedy_decode(n_gen)
    first_close = next((i for i in range(n_gen) if gap[i] < ATOL), n_gen)
    diverge = next((i for i in range(n_gen) if ids[i] != ref[i]), n_gen)
    assert diverge >= first_close, (ids, ref)
    e.reset()
    e.prefill(prompt, want_logits=False)
    am = e.forced_decode(ref)
    bad = [i for i in range(n_gen) if am[i] != ref[i] and gap[i] >= ATOL]
    assert not bad, bad
    fi, fv = mg.sampled(g, "final", 0)
    np.testing.assert_allclose(e.logits()[fi], fv, atol=ATOL, rtol=RTOL)
    e.close()
