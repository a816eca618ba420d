"""Engine parity on the reference's block fixtures (qwen25_block.rs tests):
known answers, cursor semantics, errors that do not advance, chunk prefill
versus serial forward, and logits against the CPU oracle."""
import json
import os

import numpy as np
import pytest

import myos
from myos import _lib
import ref_fixtures as rf

pytestmark = pytest.mark.gpu
PINS = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_pins.json")))


def bits(a):
    return [int(b) for b in np.asarray(a, np.float32).reshape(-1).view(np.uint32)]


def engine(shape, table, max_seq, **kw):
    e = myos.Engine(shape, max_seq, **kw)
    e.load_table(table)
    return e


@pytest.mark.parametrize("kv", ["f32", "bf16"])
@pytest.mark.parametrize("graphs", [True, False])
def test_block_fixture_known_answers(kv, graphs):
    P = PINS["block"]
    shape, t = rf.block_fixture()
    e = engine(shape, t, 4, kv_dtype=kv, use_graphs=graphs)
    logits = e.forward_token(0, 0)
    assert logits.tolist() == P["fixture_logits"]
    assert myos.greedy_token(logits) == P["fixture_greedy"]
    assert e.kv_len() == 1
    k, v = e.kv_head(0, 0, 0)
    assert k.tolist() == [0.0, 0.0] and v.tolist() == P["fixture_cache_v0"]
    assert e.kv_head(0, 0, 1)[1].tolist() == [0.0, 0.0]  # one advance, next slot empty
    e2 = engine(shape, t, 8, kv_dtype=kv, use_graphs=graphs)
    assert e2.prefill([0]).tolist() == P["fixture_logits"]
    assert e2.greedy_decode(4).tolist() == P["fixture_decode4"]
    assert e2.kv_len() == 5
    assert e2.kv_head(0, 0, 4)[1].tolist() == [1.0, 0.0]


def test_swiglu_and_two_layer_fixtures(orc):
    for build in (rf.swiglu_fixture, rf.two_layer_fixture):
        shape, t = build()
        e = engine(shape, t, 4)
        wm = rf.load_into_oracle(orc, t)
        md = orc.Model(rf.oracle_shape(orc, shape), 4)
        for pos, tok in enumerate([0, 1, 3]):
            got = e.forward_token(tok, pos)
            assert md.forward_token(wm, tok, pos) == 0
            np.testing.assert_allclose(got, md.logits(), rtol=1e-6, atol=1e-6)
        for layer in range(shape["num_layers"]):
            for pos in range(3):
                k, v = e.kv_head(layer, 0, pos)
                st, k2, v2 = md.kv_head(layer, 0, pos)
                np.testing.assert_allclose(k, k2, rtol=1e-6, atol=1e-7)
                np.testing.assert_allclose(v, v2, rtol=1e-6, atol=1e-7)


def test_errors_do_not_advance():
    shape, t = rf.block_fixture()
    e = myos.Engine(shape, 2)
    with pytest.raises(myos.MyosError) as ex:
        e.forward_token(0, 0)
    assert ex.value.code == _lib.ERR_WEIGHT_MISSING and e.kv_len() == 0
    e.load_table(t)
    with pytest.raises(myos.MyosError) as ex:
        e.forward_token(0, 1)
    assert ex.value.code == _lib.ERR_POSITION and e.kv_len() == 0
    with pytest.raises(myos.MyosError) as ex:
        e.forward_token(9, 0)
    assert ex.value.code == _lib.ERR_TOKEN and e.kv_len() == 0
    assert e.logits().tolist() == [0.0] * 4
    e.forward_token(0, 0)
    e.forward_token(1, 1)
    before = e.logits()
    with pytest.raises(myos.MyosError) as ex:
        e.forward_token(1, 2)
    assert ex.value.code == _lib.ERR_CACHE_FULL and e.kv_len() == 2
    assert e.logits().tolist() == before.tolist()
    # prefill rejects before any store (qwen25_block.rs:1480-1513)
    e2 = engine(shape, t, 4)
    with pytest.raises(myos.MyosError) as ex:
        e2.prefill([0, 9])
    assert ex.value.code == _lib.ERR_TOKEN and e2.kv_len() == 0
    with pytest.raises(myos.MyosError) as ex:
        e2.prefill([])
    assert ex.value.code == _lib.ERR_SHAPE
    with pytest.raises(myos.MyosError) as ex:
        e2.prefill([0] * 5)
    assert ex.value.code == _lib.ERR_CACHE_FULL and e2.kv_len() == 0
    # weight checks: dtype and shape of a known key
    with pytest.raises(myos.MyosError) as ex:
        e2.load_tensor("model.norm.weight", [2], np.zeros(8, np.uint8), dtype=_lib.F32)
    assert ex.value.code == _lib.ERR_WEIGHT_DTYPE
    with pytest.raises(myos.MyosError) as ex:
        e2.load_tensor("model.norm.weight", [3], np.zeros(6, np.uint8))
    assert ex.value.code == _lib.ERR_WEIGHT_SHAPE
    # reset is KvCache::clear: cursor to 0
    e.reset()
    assert e.kv_len() == 0
    assert e.forward_token(0, 0).tolist() == PINS["block"]["fixture_logits"]


@pytest.mark.parametrize("kv", ["f32", "bf16"])
def test_chunk_prefill_matches_serial_and_oracle(orc, kv):
    # qwen25_block.rs:1403-1478 on the GPU, plus the oracle comparison
    shape = rf.rich_shape(2)
    t = rf.rich_map(shape)
    prompt = [1, 3, 0, 4, 2]
    es = engine(shape, t, 16, kv_dtype=kv)
    ec = engine(shape, t, 16, kv_dtype=kv)
    es.forward_token(2, 0)
    ec.forward_token(2, 0)
    for i, tok in enumerate(prompt):
        serial = es.forward_token(tok, 1 + i)
    chunk = ec.prefill(prompt)
    assert bits(chunk) == bits(serial)
    for layer in range(2):
        for head in range(2):
            for pos in range(6):
                assert bits(ec.kv_head(layer, head, pos)[0]) == bits(es.kv_head(layer, head, pos)[0])
    assert es.greedy_decode(3).tolist() == ec.greedy_decode(3).tolist()
    # oracle
    wm = rf.load_into_oracle(orc, t)
    md = orc.Model(rf.oracle_shape(orc, shape), 16)
    assert md.forward_token(wm, 2, 0) == 0 and md.prefill(wm, prompt) == 0
    tol = 1e-5 if kv == "f32" else 2e-2
    np.testing.assert_allclose(chunk, md.logits(), rtol=tol, atol=tol)
    st, out, gap, _ = md.greedy_decode(wm, 3)
    ed = engine(shape, t, 16, kv_dtype=kv)
    ed.forward_token(2, 0)
    ed.prefill(prompt)
    got = ed.greedy_decode(3)
    for i in range(3):
        if got[i] != out[i]:
            assert gap[i] < 1e-2, (i, got, out)
            break


def test_batch_tail_prefill_33(orc):
    wide = rf.rich_shape(1)
    t = rf.rich_map(wide)
    toks = [i % 5 for i in range(33)]
    e = engine(wide, t, 40)
    logits = e.prefill(toks)
    wm = rf.load_into_oracle(orc, t)
    md = orc.Model(rf.oracle_shape(orc, wide), 40)
    assert md.prefill(wm, toks) == 0
    np.testing.assert_allclose(logits, md.logits(), rtol=1e-5, atol=1e-5)
    assert e.kv_len() == 33


def test_safetensors_load_path(tmp_path, orc):
    from myos import synth
    shape, t = rf.block_fixture()
    p = str(tmp_path / "fixture.safetensors")
    synth.write_safetensors(p, t)
    e = myos.Engine(shape, 8)
    e.load_safetensors(p)
    assert e.weights_ready()
    assert e.prefill([0]).tolist() == PINS["block"]["fixture_logits"]
    assert e.greedy_decode(4).tolist() == [1, 1, 1, 1]
    bad = str(tmp_path / "bad.safetensors")
    open(bad, "wb").write(b"\xff" * 8)
    with pytest.raises(myos.MyosError) as ex:
        myos.Engine(shape, 8).load_safetensors(bad)
    assert ex.value.code == _lib.ERR_PARSE


def test_determinism_two_runs_same_bits():
    shape = rf.rich_shape(2)
    t = rf.rich_map(shape)
    outs = []
    for _ in range(2):
        e = engine(shape, t, 16)
        e.prefill([1, 3, 0])
        ids = e.greedy_decode(6)
        outs.append((ids.tolist(), bits(e.logits())))
    assert outs[0] == outs[1]
