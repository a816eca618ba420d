"""Qwen2.5-1.5B S1 parity: seeded random-init BF16
weights, a 128-id uniform prompt, 128 greedy steps.

Pass rule: the GPU's greedy ids equal the oracle's at
every step, except where the oracle's top-1/top-2 logit gap is below the
logit tolerance; to keep every step comparable after such a divergence the
GPU is also run teacher-forced on the oracle's ids. Final-step logits agree
within 1e-2 absolute / 1e-3 relative.
"""
import numpy as np
import pytest

import myos
from myos import synth

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

SEED = 1234
N_PROMPT, N_GEN = 128, 128
ATOL, RTOL = 1e-2, 1e-3
# A bf16 KV cache rounds every cached K and V element to 8 mantissa bits
# (relative 2^-9), which the reference's f32 cache never does; its logits
# are held to this wider bound instead.
TOL = {"f32": (ATOL, RTOL), "bf16": (6e-2, 6e-3)}


@pytest.fixture(scope="module")
def model():
    shape = synth.shape_qwen25_1_5b()
    table = synth.weights(shape, SEED)
    prompt = synth.prompt_ids(SEED, N_PROMPT, shape["vocab"])
    return shape, table, prompt


@pytest.fixture(scope="module")
def golden(model, orc):
    import ref_fixtures as rf
    shape, table, prompt = model
    wm = rf.load_into_oracle(orc, table)
    md = orc.Model(rf.oracle_shape(orc, shape), N_PROMPT + N_GEN)
    assert md.prefill(wm, prompt) == 0
    prefill_logits = md.logits()
    st, ids, gap, _ = md.greedy_decode(wm, N_GEN)
    assert st == 0
    return dict(prefill_logits=prefill_logits, ids=ids, gap=gap, final=md.logits())


@pytest.mark.parametrize("kv", ["f32", "bf16"])
def test_s1_greedy_ids_and_logits(model, golden, kv):
    shape, table, prompt = model
    e = myos.Engine(shape, N_PROMPT + N_GEN, kv_dtype=kv)
    e.load_table(table)
    atol, rtol = TOL[kv]
    pl = e.prefill(prompt)
    np.testing.assert_allclose(pl, golden["prefill_logits"], atol=atol, rtol=rtol)
    ids = e.greedy_decode(N_GEN)
    ref = golden["ids"]
    # First step where the reference's top-2 gap is below tolerance; the
    # sequences must agree strictly before it.
    first_close = next((i for i in range(N_GEN) if golden["gap"][i] < atol), N_GEN)
    diverge = next((i for i in range(N_GEN) if ids[i] != ref[i]), N_GEN)
    assert diverge >= first_close, (diverge, first_close, ids[:diverge + 1], ref[:diverge + 1])
    if diverge == N_GEN:
        np.testing.assert_allclose(e.logits(), golden["final"], atol=atol, rtol=rtol)

    # Teacher-forced: every step comparable.
    e.reset()
    e.prefill(prompt)
    am = e.forced_decode(ref)
    # am[i] is the argmax of the logits that chose ref[i]
    bad = [i for i in range(N_GEN) if am[i] != ref[i] and golden["gap"][i] >= atol]
    assert not bad, bad
    np.testing.assert_allclose(e.logits(), golden["final"], atol=atol, rtol=rtol)


def test_gemm_prefill_matches_token_steps(model, monkeypatch):
    """The tensor-core prefill (two 128-token chunks and a ragged third) against
    the same prompt run as single-token steps: final logits within the logit
    tolerance and the cached K/V of early, chunk-boundary and last positions
    close; greedy continuations agree."""
    shape, table, _ = model
    prompt = synth.prompt_ids(SEED + 7, 300, shape["vocab"])
    out = {}
    for mode in ("gemm", "steps"):
        monkeypatch.setenv("MYOS_PREFILL", "gemm" if mode == "gemm" else "steps")
        e = myos.Engine(shape, 320)
        e.load_table(table)
        logits = e.prefill(prompt)
        kv = [e.kv_head(l, h, p) for l, h, p in ((0, 0, 5), (13, 1, 127), (27, 0, 128), (27, 1, 299))]
        ids = e.greedy_decode(8)
        out[mode] = (logits, kv, ids)
        e.close()
    np.testing.assert_allclose(out["gemm"][0], out["steps"][0], atol=ATOL, rtol=RTOL)
    for (kg, vg), (ks, vs) in zip(out["gemm"][1], out["steps"][1]):
        np.testing.assert_allclose(kg, ks, atol=2e-3, rtol=2e-3)
        np.testing.assert_allclose(vg, vs, atol=2e-3, rtol=2e-3)
    assert out["gemm"][2].tolist() == out["steps"][2].tolist()
