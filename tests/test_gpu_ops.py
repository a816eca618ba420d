"""Per-kernel parity: the CUDA operators (through the C ABI) against the CPU
oracle on the same inputs.

Exact where the math is order-independent (RoPE from the host libm table,
argmax rules, single-term sums, the reference's small hand pins); within a
stated float-reassociation bound where the reference sums serially and the
GPU sums in a fixed tree.
"""
import json
import os

import numpy as np
import pytest

import myos
from myos import ops

pytestmark = pytest.mark.gpu

PINS = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_pins.json")))
U = 2.0 ** -24  # f32 unit roundoff


def hx(s):
    return int(s, 16)


def bits(a):
    return [int(b) for b in np.asarray(a, np.float32).reshape(-1).view(np.uint32)]


def gemv_bound(w_bytes, x, m, k):
    """|serial - tree| <= (k + 2) u sum_j |w_j x_j| per row (standard bound)."""
    wf = (w_bytes.view("<u2").astype(np.uint32) << 16).view(np.float32).reshape(m, k)
    mag = (np.abs(wf.astype(np.float64)) @ np.abs(np.asarray(x, np.float64)))
    return (k + 2) * U * mag + 1e-30


def rand_bf16(rng, n, std=0.02):
    f = (rng.standard_normal(n) * std).astype(np.float32)
    u = f.view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype("<u2").view(np.uint8)


@pytest.mark.parametrize("m,k", [(1, 1), (7, 9), (33, 40), (2, 3), (256, 1536), (1536, 1536),
                                 (2048, 1536), (8960, 1536), (1536, 8960), (5, 13824)])
def test_gemv_matches_oracle_within_reassociation_bound(orc, m, k):
    rng = np.random.default_rng(m * 7919 + k)
    w = rand_bf16(rng, m * k)
    x = rng.standard_normal(k).astype(np.float32)
    st, y = ops.gemv_bf16(w, x, m, k)
    assert st == 0
    st, want = orc.gemv_bf16(w, x, m, k)
    err = np.abs(y.astype(np.float64) - want)
    assert (err <= gemv_bound(w, x, m, k)).all(), err.max()


def test_gemv_hand_pins_and_errors(orc):
    P = PINS["bf16"]["gemv_2x3"]
    st, y = ops.gemv_bf16(orc.pack_bf16(P["w"]), P["x"], 2, 3)
    assert st == 0 and y.tolist() == P["expect"]
    c = PINS["gemv"]["cancellation"]
    st, y = ops.gemv_bf16(orc.pack_bf16(c["row"]), np.ones(8), 1, 8)
    assert bits(y) == [hx(c["expect_bits"])]  # one lane walks the 8 columns in order
    w = np.array([0x80, 0x3F, 0x00, 0x40], np.uint8)
    assert ops.gemv_bf16(w, [1.0, 1.0], 2, 2)[0] == myos._lib.ERR_ROW_OOB
    assert ops.gemv_bf16(np.array([0x80, 0x3F, 0x00, 0x40, 0], np.uint8), [1.0], 2, 1)[0] == \
        myos._lib.ERR_SHAPE
    st, y = ops.gemv_bf16(np.zeros(0, np.uint8), np.zeros(0), 2, 0)
    assert st == 0 and y.tolist() == [0.0, 0.0]


def test_gemv_every_bf16_pattern_exact(orc):
    # gemv_bf16_kernel.rs:1032-1048: one live weight per row -> single term, exact
    for k, live in ((16, 0), (17, 16)):
        m = 65536
        w = np.zeros((m, k), np.uint16)
        w[:, live] = np.arange(m, dtype=np.uint16)
        x = np.zeros(k, np.float32)
        x[live] = 1.0
        wb = w.astype("<u2").view(np.uint8).reshape(-1)
        st, y = ops.gemv_bf16(wb, x, m, k)
        st2, want = orc.gemv_bf16(wb, x, m, k, 8)
        nan = np.isnan(want)
        assert np.array_equal(np.isnan(y), nan)
        assert bits(y[~nan]) == bits(want[~nan])


def test_rmsnorm(orc):
    P = PINS["bf16"]
    for case in P["rmsnorm_hand"]:
        st, y = ops.rmsnorm_bf16_weight(orc.pack_bf16(case["w"]), case["x"], case["eps"])
        assert st == 0 and y.tolist() == case["expect"]
    c = P["rmsnorm_eps_qwen"]
    st, y = ops.rmsnorm_bf16_weight(orc.pack_bf16(c["w"]), c["x"], np.float32(c["eps"]))
    assert bits(y) == [hx(b) for b in c["expect_bits"]]
    rng = np.random.default_rng(3)
    for n in (2, 1536, 5120):
        x = rng.standard_normal(n).astype(np.float32)
        g = rand_bf16(rng, n, 0.01)
        st, y = ops.rmsnorm_bf16_weight(g, x, np.float32(1e-6))
        st, want = orc.rmsnorm_bf16_weight(g, x, np.float32(1e-6))
        np.testing.assert_allclose(y, want, rtol=4 * n * U, atol=0)
    assert ops.rmsnorm_bf16_weight(np.zeros(0, np.uint8), np.zeros(0), 1e-6)[0] == myos._lib.ERR_SHAPE


def test_rope_bit_exact(orc):
    P = PINS["rope"]
    for case in P["d2_pos1"]:
        st, y = ops.rope_f32(case["x"], 1, 2, 1e6)
        assert bits(y) == [hx(b) for b in case["expect_bits"]]
    st, y = ops.rope_f32(P["d4_pos3"]["x"], 3, 4, 1e6)
    assert bits(y) == [hx(b) for b in P["d4_pos3"]["expect_bits"]]
    rng = np.random.default_rng(5)
    for pos in (0, 1, 8, 127, 4095, 4351):
        x = rng.standard_normal(12 * 128).astype(np.float32)
        st, y = ops.rope_f32(x, pos, 128, 1e6)
        st2, want = orc.rope_f32(x, pos, 128, 1e6)
        assert st == 0 and bits(y) == bits(want), pos
    assert ops.rope_f32(np.zeros(5), 1, 4, 1e6)[0] == myos._lib.ERR_SHAPE


def test_swiglu_mul(orc):
    P = PINS["swiglu"]["mul"]
    st, h = ops.swiglu_mul_f32(P["gate"], P["up"])
    want = [hx(b) for b in P["expect_bits"]]
    got = bits(h)
    # CUDA expf is within 2 ulp of glibc's; the division form is kept.
    for g_, w_ in zip(got, want):
        assert abs(np.int64(g_) - np.int64(w_)) <= 2
    rng = np.random.default_rng(11)
    g = (rng.standard_normal(8960) * 3).astype(np.float32)
    u = rng.standard_normal(8960).astype(np.float32)
    st, h = ops.swiglu_mul_f32(g, u)
    st, want = orc.swiglu_mul_f32(g, u)
    np.testing.assert_allclose(h, want, rtol=8 * U, atol=1e-30)


def test_gqa_pins_and_oracle(orc):
    P = PINS["gqa"]
    g = P["groups"]
    hq, hkv, d, seq = g["shape"]
    st, y = ops.gqa_attn_f32(g["q"], g["k"], g["v"], hq, hkv, d, seq, causal_pos=0)
    assert y.tolist() == P["causal0"]["expect_y"]
    st, y = ops.gqa_attn_f32(g["q"], g["k"], g["v"], hq, hkv, d, seq)
    np.testing.assert_allclose(y, np.array([hx(b) for b in g["y_bits"]], np.uint32).view(np.float32),
                               rtol=4e-7)
    s = P["single_key_overflow"]
    assert ops.gqa_attn_f32(s["q"], s["k"], s["v"], 1, 1, 1, 1)[1].tolist() == [s["expect"]]
    e = P["equal_big_logits"]
    assert ops.gqa_attn_f32(e["q"], e["k"], e["v"], 1, 1, 1, 2)[1].tolist() == [e["expect_y"]]
    rng = np.random.default_rng(9)
    for hq, hkv, d, seq, cpos in ((12, 2, 128, 256, None), (12, 2, 128, 300, 150),
                                  (40, 8, 128, 97, None), (4, 2, 2, 5, 3), (8, 8, 64, 1000, None)):
        q = rng.standard_normal(hq * d).astype(np.float32)
        k = rng.standard_normal(hkv * seq * d).astype(np.float32)
        v = rng.standard_normal(hkv * seq * d).astype(np.float32)
        st, y = ops.gqa_attn_f32(q, k, v, hq, hkv, d, seq, causal_pos=cpos)
        st2, want, _ = orc.gqa_attn_f32(q, k, v, hq, hkv, d, seq, causal_pos=cpos)
        assert st == 0
        np.testing.assert_allclose(y, want, rtol=2e-5, atol=2e-6)
    assert ops.gqa_attn_f32([1, 2, 3], [1, 0, 0, 1], [4, 5, 6, 7], 3, 2, 1, 2)[0] == myos._lib.ERR_SHAPE


def test_greedy_token_rules():
    assert myos.greedy_token([1.0, 2.0, 0.0, -1.0]) == 1
    assert myos.greedy_token([3.0, 3.0, 1.0]) == 0
    assert myos.greedy_token([np.nan, 1.0, 1.0]) == 1
    assert myos.greedy_token([np.nan, -np.inf, -np.inf]) == 0
    assert myos.greedy_token([-np.inf, 5.0, np.inf]) == 2
    rng = np.random.default_rng(1)
    v = rng.standard_normal(151936).astype(np.float32)
    v[[100, 90000, 150000]] = 9.0  # ties: the first one wins
    assert myos.greedy_token(v) == 100
