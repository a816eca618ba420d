"""Long-context decode (a 4096-token prompt, then greedy
steps, bf16 KV cache over 4352 positions) on the seeded 1.5B model.

At 4352 slots the decode attention splits each KV head's keys 74 ways and
merges them in global memory (more splits than one thread-block cluster
holds), and the prompt runs as 32 tensor-core prefill chunks. Checks:
  * a 512-token prompt (17 splits, same merge path) against the oracle: the
    greedy ids except at near-ties, teacher-forced argmaxes, final logits;
  * the 4096-token prompt through the GEMM prefill against the same prompt
    as single-token steps: logits and the greedy continuation.
The bf16 cache rounds every cached element (the reference's cache is f32),
so logits are held to the bf16 tolerance of tests/test_gpu_qwen.py.
"""
import numpy as np
import pytest

import myos
from myos import synth

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

SEED = 1234
ATOL, RTOL = 6e-2, 6e-3


@pytest.fixture(scope="module")
def model():
    shape = synth.shape_qwen25_1_5b()
    return shape, synth.weights(shape, SEED)


def test_512_context_bf16_kv_against_oracle(model, orc):
    import ref_fixtures as rf
    shape, table = model
    n_prompt, n_gen = 512, 16
    prompt = synth.prompt_ids(SEED + 3, n_prompt, shape["vocab"])
    wm = rf.load_into_oracle(orc, table)
    md = orc.Model(rf.oracle_shape(orc, shape), n_prompt + n_gen)
    assert md.prefill(wm, prompt) == 0
    st, ref, gap, _ = md.greedy_decode(wm, n_gen)
    assert st == 0
    final = md.logits()

    e = myos.Engine(shape, n_prompt + n_gen, kv_dtype="bf16")
    e.load_table(table)
    e.prefill(prompt, want_logits=False)
    ids = e.greedy_decode(n_gen)
    first_close = next((i for i in range(n_gen) if gap[i] < ATOL), n_gen)
    diverge = next((i for i in range(n_gen) if ids[i] != ref[i]), n_gen)
    assert diverge >= first_close, (diverge, first_close)
    e.reset()
    e.prefill(prompt, want_logits=False)
    am = e.forced_decode(ref)
    bad = [i for i in range(n_gen) if am[i] != ref[i] and gap[i] >= ATOL]
    assert not bad, bad
    np.testing.assert_allclose(e.logits(), final, atol=ATOL, rtol=RTOL)
    e.close()


def test_4096_context_gemm_prefill_against_token_steps(model, monkeypatch):
    shape, table = model
    n_prompt, n_gen, max_seq = 4096, 16, 4352
    prompt = synth.prompt_ids(SEED + 4, n_prompt, shape["vocab"])
    out = {}
    for mode in ("gemm", "steps"):
        monkeypatch.setenv("MYOS_PREFILL", mode)
        e = myos.Engine(shape, max_seq, kv_dtype="bf16")
        e.load_table(table)
        logits = e.prefill(prompt)
        ids = e.greedy_decode(n_gen)
        out[mode] = (logits, ids, e.logits())
        assert e.kv_len() == n_prompt + n_gen
        e.close()
    np.testing.assert_allclose(out["gemm"][0], out["steps"][0], atol=ATOL, rtol=RTOL)
    g, s_ = out["gemm"][1].tolist(), out["steps"][1].tolist()
    # the continuations agree until a near-tie of the step path's logits
    agree = next((i for i in range(n_gen) if g[i] != s_[i]), n_gen)
    assert agree >= 4, (g, s_)
    if agree == n_gen:
        np.testing.assert_allclose(out["gemm"][2], out["steps"][2], atol=ATOL, rtol=RTOL)
