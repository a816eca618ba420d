"""Long-context decode (a 4096-token prompt, then greedy
steps, KV cache over 4352 positions) on the seeded 1.5B model.

At 4352 slots the decode attention splits each KV head's keys 74 ways and
merges them in global memory (more splits than one thread-block cluster
holds), and the prompt runs as 32 tensor-core prefill chunks. Checks:
  * a 512-token prompt (17 splits, same merge path) against the oracle run
    live: the greedy ids except at near-ties, teacher-forced argmaxes, final
    logits;
  * the 4096-token prompt and 32 greedy steps against the oracle's answers
    for the same seeded inputs, computed once on the CPU and committed
    (tests/golden/s3_4096.npz, tests/golden/make_goldens.py): prompt and
    final logits at the fixture's indices, greedy ids before the first
    near-tie, teacher-forced argmaxes at every step that is not a near-tie.
The oracle's cache is f32; a bf16 cache rounds every cached element, so its
logits are held to the wider bf16 tolerance of tests/test_gpu_qwen.py.
"""
import numpy as np
import pytest

import myos
from myos import synth
from golden import make_goldens as mg

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

SEED = 1234
TOL = {"f32": (1e-2, 1e-3), "bf16": (6e-2, 6e-3)}


@pytest.fixture(scope="module")
def model():
    shape = synth.shape_qwen25_1_5b()
    return shape, synth.weights(shape, SEED)


def check_against(e, prompt, ref, gap, final_idx, final_val, pre_idx, pre_val, atol, rtol):
    n_gen = len(ref)
    pl = e.prefill(prompt)
    if pre_idx is not None:
        np.testing.assert_allclose(pl[pre_idx], pre_val, atol=atol, rtol=rtol)
    ids = e.greedy_decode(n_gen)
    first_close = next((i for i in range(n_gen) if gap[i] < atol), n_gen)
    diverge = next((i for i in range(n_gen) if ids[i] != ref[i]), n_gen)
    assert diverge >= first_close, (diverge, first_close)
    e.reset()
    e.prefill(prompt, want_logits=False)
    am = e.forced_decode(ref)
    bad = [i for i in range(n_gen) if am[i] != ref[i] and gap[i] >= atol]
    assert not bad, bad
    np.testing.assert_allclose(e.logits()[final_idx], final_val, atol=atol, rtol=rtol)


def test_512_context_bf16_kv_against_oracle(model, orc):
    import ref_fixtures as rf
    shape, table = model
    n_prompt, n_gen = 512, 16
    atol, rtol = TOL["bf16"]
    prompt = synth.prompt_ids(SEED + 3, n_prompt, shape["vocab"])
    wm = rf.load_into_oracle(orc, table)
    md = orc.Model(rf.oracle_shape(orc, shape), n_prompt + n_gen)
    assert md.prefill(wm, prompt) == 0
    st, ref, gap, _ = md.greedy_decode(wm, n_gen)
    assert st == 0
    final = md.logits()
    e = myos.Engine(shape, n_prompt + n_gen, kv_dtype="bf16")
    e.load_table(table)
    check_against(e, prompt, ref, gap, np.arange(final.size), final, None, None, atol, rtol)
    e.close()


@pytest.mark.parametrize("kv", ["f32", "bf16"])
def test_4096_context_against_oracle_golden(model, kv):
    shape, table = model
    g = mg.load("s3")
    n_prompt, n_gen = int(g["n_prompt"]), int(g["n_gen"])
    prompt = synth.prompt_ids(int(g["prompt_seeds"][0]), n_prompt, shape["vocab"])
    atol, rtol = TOL[kv]
    e = myos.Engine(shape, 4352, kv_dtype=kv)
    e.load_table(table)
    fi, fv = mg.sampled(g, "final", 0)
    pi, pv = mg.sampled(g, "prefill", 0)
    check_against(e, prompt, g["ids"][0], g["gap"][0], fi, fv, pi, pv, atol, rtol)
    assert e.kv_len() == n_prompt + n_gen
    e.close()
