"""Pin the CPU oracle to the reference's own known-answer tests.

Every assertion here restates one in the reference's #[cfg(test)] modules;
the constants come from tests/golden/reference_pins.json (file:line cited
there). A pass means the oracle reproduces the reference's CPU path bit for
bit on those cases, which is what lets it stand in for the (unbuildable
here) Rust reference as the parity oracle.
"""
import json
import math
import os

import numpy as np
import pytest

import ref_fixtures as rf

PINS = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_pins.json")))


def hx(s):
    return int(s, 16)


def bits(a):
    return [int(b) for b in np.asarray(a, np.float32).reshape(-1).view(np.uint32)]


def f(bits_hex):
    return np.array([hx(bits_hex)], np.uint32).view(np.float32)[0]


# ------------------------------------------------------------------ bf16.rs
def test_bf16_le_decode(orc):
    P = PINS["bf16"]
    assert np.float32(1e-6).view(np.uint32) == hx(P["rms_eps_bits"])
    for le, want in P["le_decode"]:
        arr = (np.array(le, np.uint8))
        v = orc.lib().orc_bf16_le_to_f32(arr.ctypes.data_as(orc._u8p))
        assert bits([v]) == [hx(want)]


def test_add_bias_and_errors(orc):
    P = PINS["bf16"]["add_bias"]
    y = np.array(P["y"], np.float32)
    assert orc.add_bf16_bias(y, orc.pack_bf16(P["bias"])) == 0
    assert y.tolist() == P["expect"]
    kept = np.array([7.0, 8.0, 9.0], np.float32)
    assert orc.add_bf16_bias(kept, orc.pack_bf16([0.5, 1.0])) == orc.SHAPE
    assert kept.tolist() == [7.0, 8.0, 9.0]
    assert orc.add_bf16_bias(np.zeros(0, np.float32), np.zeros(0, np.uint8)) == 0


def test_gemv_hand_values_zero_k_and_errors(orc):
    P = PINS["bf16"]["gemv_2x3"]
    st, y = orc.gemv_bf16(orc.pack_bf16(P["w"]), P["x"], 2, 3)
    assert st == 0 and y.tolist() == P["expect"]
    # k == 0 fills zeros; slack bytes are Shape (bf16.rs:400-411).
    y = np.array([1.0, 2.0], np.float32)
    st, y = orc.gemv_bf16(np.zeros(0, np.uint8), np.zeros(0, np.float32), 2, 0, y=y)
    assert st == 0 and y.tolist() == [0.0, 0.0]
    kept = np.array([1.0], np.float32)
    st, _ = orc.gemv_bf16(np.array([0], np.uint8), np.zeros(0, np.float32), 1, 0, y=kept)
    assert st == orc.SHAPE and kept.tolist() == [1.0]
    # short rows (bf16.rs:425-458)
    w = np.array([0x80, 0x3F, 0x00, 0x40], np.uint8)
    y = np.array([7.0, 8.0], np.float32)
    st, _ = orc.gemv_bf16(w, [1.0, 1.0], 2, 2, y=y)
    assert st == orc.ROW_OOB and y.tolist() == [7.0, 8.0]
    wide = np.array([0x80, 0x3F, 0x00, 0x40, 0x00], np.uint8)
    st, _ = orc.gemv_bf16(wide, [1.0, 1.0], 2, 1, y=np.zeros(2, np.float32))
    assert st == orc.SHAPE


def test_embed_gather(orc):
    table = orc.pack_bf16([1.0, 2.0, 3.0, -0.5, 0.5, 4.0])
    out = np.zeros(2, np.float32)
    for tok, want in [(1, [3.0, -0.5]), (2, [0.5, 4.0]), (0, [1.0, 2.0])]:
        assert orc.embed_gather_bf16(table, [3, 2], tok, out) == 0
        assert out.tolist() == want
    out1 = np.array([9.0], np.float32)
    t2 = orc.pack_bf16([1.0, 2.0])
    assert orc.embed_gather_bf16(t2, [2, 1], 2, out1) == orc.TOKEN
    assert orc.embed_gather_bf16(t2, [2, 1], 0xFFFFFFFF, out1) == orc.TOKEN
    short = orc.pack_bf16([1.0])
    assert orc.embed_gather_bf16(short, [2, 1], 1, out1) == orc.ROW_OOB
    assert orc.embed_gather_bf16(short, [2, 1], 0, out1) == orc.SHAPE
    assert out1.tolist() == [9.0]


def test_rmsnorm_pins(orc):
    P = PINS["bf16"]
    for case in P["rmsnorm_hand"]:
        st, y = orc.rmsnorm_f32(case["w"], case["x"], case["eps"])
        assert st == 0 and y.tolist() == case["expect"]
        st, y = orc.rmsnorm_bf16_weight(orc.pack_bf16(case["w"]), case["x"], case["eps"])
        assert st == 0 and y.tolist() == case["expect"]
    c = P["rmsnorm_left_to_right"]
    st, y = orc.rmsnorm_bf16_weight(orc.pack_bf16(c["w"]), c["x"], c["eps"])
    assert bits(y) == [hx(b) for b in c["expect_bits"]]
    c = P["rmsnorm_eps_qwen"]
    st, y = orc.rmsnorm_bf16_weight(orc.pack_bf16(c["w"]), c["x"], np.float32(c["eps"]))
    assert bits(y) == [hx(b) for b in c["expect_bits"]]
    # zeros stay zero with eps; eps 0 gives NaN (bf16.rs:541-555)
    st, y = orc.rmsnorm_bf16_weight(orc.pack_bf16([3.0, -1.0]), [0.0, 0.0], np.float32(1e-6))
    assert y.tolist() == [0.0, 0.0]
    st, y = orc.rmsnorm_f32([3.0, -1.0], [0.0, 0.0], 0.0)
    assert np.isnan(y).all()
    for le, want in P["rmsnorm_gamma_le"]:
        st, y = orc.rmsnorm_bf16_weight(np.array(le, np.uint8), [1.0], 0.0)
        assert bits(y) == [hx(want)]
    # empty / mismatched lengths
    st, _ = orc.rmsnorm_bf16_weight(np.zeros(0, np.uint8), np.zeros(0, np.float32), 1e-6,
                                    y=np.zeros(0, np.float32))
    assert st == orc.SHAPE


# ------------------------------------------------------------------ gemv kernel
def test_gemv_left_to_right_cancellation(orc):
    P = PINS["gemv"]["cancellation"]
    row = orc.pack_bf16(P["row"])
    for threads in (1, 8):
        st, y = orc.gemv_bf16(row, np.ones(8, np.float32), 1, 8, threads)
        assert bits(y) == [hx(P["expect_bits"])]
        wide = np.tile(row, 32)
        st, y = orc.gemv_bf16(wide, np.ones(8, np.float32), 32, 8, threads)
        assert set(bits(y)) == {hx(P["expect_bits"])}


def test_row_spans(orc):
    P = PINS["gemv"]
    for m, t, want in P["row_spans"]:
        assert orc.gemv_row_spans(m, t) == [tuple(s) for s in want], (m, t)
    for m, t, step in P["row_spans_even"]:
        assert orc.gemv_row_spans(m, t) == [(i * step, (i + 1) * step) for i in range(t)]
    h = P["row_spans_head"]
    spans = orc.gemv_row_spans(h["m"], h["threads"])
    sizes = [b - a for a, b in spans]
    assert sizes == [h["wide_rows"]] * h["wide_first"] + [h["narrow_rows"]] * (8 - h["wide_first"])


def _xorshift_patterned(m, k, seed):
    """gemv_bf16_kernel.rs:844-876 (patterned): finite bf16 payloads + full-range f32 x."""
    state = seed & 0xFFFFFFFF

    def nxt():
        nonlocal state
        x = state
        x ^= (x << 13) & 0xFFFFFFFF
        x ^= x >> 17
        x ^= (x << 5) & 0xFFFFFFFF
        if x == 0:
            x = 0xA5A51234
        state = x
        return x

    w = np.zeros(m * k, np.uint16)
    for i in range(m * k):
        b = nxt() & 0xFFFF
        if (b >> 7) & 0xFF == 0xFF:
            b = (b & 0x807F) | (0x70 << 7)
        w[i] = b
    x = np.zeros(k, np.uint32)
    for j in range(k):
        b = nxt()
        if (b >> 23) & 0xFF == 0xFF:
            b = (b & 0x807FFFFF) | (120 << 23)
        x[j] = b
    return w.astype("<u2").view(np.uint8), x.view(np.float32)


def _naive(w, x, m, k):
    wf = (w.view("<u2").astype(np.uint32) << 16).view(np.float32).reshape(m, k)
    y = np.zeros(m, np.float32)
    with np.errstate(all="ignore"):
        for j in range(k):
            y = y + wf[:, j] * np.float32(x[j])
    return y


@pytest.mark.parametrize("m,k", [(1, 1), (7, 9), (8, 8), (17, 15), (31, 24), (33, 40), (48, 31),
                                 (9, 1536), (40, 100)])
def test_gemv_paths_match_naive_chain(orc, m, k):
    # scalar_and_avx2_match_naive_on_tails_and_qwen_dims, :969-1011
    w, x = _xorshift_patterned(m, k, 0xC0FFEE00 ^ (m * 131 + k))
    want = _naive(w, x, m, k)
    for threads in (1, 3, 8):
        st, y = orc.gemv_bf16(w, x, m, k, threads)
        assert st == 0
        assert bits(y) == bits(want), threads


def test_every_bf16_pattern_through_simd_and_tail(orc):
    # :1032-1048: one live weight per row, 65536 rows
    for k, live in ((16, 0), (17, 16)):
        m = 65536
        w = np.zeros((m, k), np.uint16)
        w[:, live] = np.arange(m, dtype=np.uint16)
        x = np.zeros(k, np.float32)
        x[live] = 1.0
        wb = w.astype("<u2").view(np.uint8).reshape(-1)
        st, y = orc.gemv_bf16(wb, x, m, k, 8)
        want = _naive(wb, x, m, k)
        nan = np.isnan(want)
        assert np.array_equal(np.isnan(y), nan)
        assert bits(y[~nan]) == bits(want[~nan])


def test_gemm_matches_per_token_gemv(orc):
    # gemm_bf16.rs:547-572: chunk GEMM == per-token GEMV bits, batch tails
    for batch, m, k in ((33, 17, 40), (5, 32, 64), (8, 9, 130)):
        w, _ = _xorshift_patterned(m, k, 0x1234 + batch)
        rng = np.random.default_rng(batch)
        x = rng.standard_normal((batch, k)).astype(np.float32)
        st, y = orc.gemm_bf16(w, x, batch, m, k, 8)
        assert st == 0
        for b in range(batch):
            st, yb = orc.gemv_bf16(w, x[b], m, k, 1)
            assert bits(y[b * m:(b + 1) * m]) == bits(yb)


# ------------------------------------------------------------------ gqa.rs
def test_gqa_scale_and_groups(orc):
    P = PINS["gqa"]
    for d, want in P["scale_bits"]:
        st, s = orc.attn_scale_f32(d)
        assert st == 0 and bits([s]) == [hx(want)]
    assert orc.attn_scale_f32(0)[0] == orc.SHAPE
    g = P["groups"]
    hq, hkv, d, seq = g["shape"]
    st, y, probs = orc.gqa_attn_f32(g["q"], g["k"], g["v"], hq, hkv, d, seq)
    assert bits(y) == [hx(b) for b in g["y_bits"]]
    assert bits(probs) == [hx(b) for b in g["probs_bits"]]
    st, y, probs = orc.gqa_attn_f32(g["q"], g["k"], g["v"], hq, hkv, d, seq, causal_pos=0)
    assert y.tolist() == P["causal0"]["expect_y"] and probs.tolist() == P["causal0"]["expect_probs"]
    st, yfull, _ = orc.gqa_attn_f32(g["q"], g["k"], g["v"], hq, hkv, d, seq)
    for qp in (1, 2 ** 63):
        st, yc, _ = orc.gqa_attn_f32(g["q"], g["k"], g["v"], hq, hkv, d, seq, causal_pos=qp)
        assert bits(yc) == bits(yfull)
    s = P["single_key_overflow"]
    st, y, probs = orc.gqa_attn_f32(s["q"], s["k"], s["v"], 1, 1, 1, 1)
    assert y.tolist() == [s["expect"]] and probs.tolist() == [1.0]


def test_gqa_softmax_pins(orc):
    P = PINS["gqa"]
    q = [2.0, 0.0, 0.0, 0.0]
    k = np.zeros(8, np.float32)
    k[0] = 1.0
    v = np.zeros(8, np.float32)
    v[0], v[4] = 4.0, 8.0
    st, y, probs = orc.gqa_attn_f32(q, k, v, 1, 1, 4, 2)
    assert bits(probs) == [hx(b) for b in P["softmax_d4"]["probs_bits"]]
    assert bits(y[:1]) == [hx(P["softmax_d4"]["y0_bits"])] and y[1:].tolist() == [0.0] * 3
    e = P["equal_big_logits"]
    st, y, probs = orc.gqa_attn_f32(e["q"], e["k"], e["v"], 1, 1, 1, 2)
    assert probs.tolist() == e["expect_probs"] and y.tolist() == [e["expect_y"]]
    q = np.zeros(128, np.float32)
    q[0] = 1.0
    k = np.zeros(256, np.float32)
    k[0] = 1.0
    v = np.zeros(256, np.float32)
    v[0], v[128] = 2.0, 6.0
    st, y, probs = orc.gqa_attn_f32(q, k, v, 1, 1, 128, 2)
    assert bits(probs) == [hx(b) for b in P["softmax_d128"]["probs_bits"]]
    assert bits(y[:1]) == [hx(P["softmax_d128"]["y0_bits"])] and not y[1:].any()


def test_gqa_dot_left_to_right_and_qwen_groups(orc):
    P = PINS["gqa"]
    q = [1.0] * 4
    k = [16777216.0, 1, 1, 1, 1, 1, 1, 16777216.0]
    v = [2.0, 0, 0, 0, 8.0, 0, 0, 0]
    st, y, _ = orc.gqa_attn_f32(q, k, v, 1, 1, 4, 2)
    assert bits(y[:1]) == [hx(P["dot_left_to_right"]["y0_bits"])]
    H = 128
    q = np.zeros(12 * H, np.float32)
    k = np.zeros(2 * 2 * H, np.float32)
    v = np.zeros(2 * 2 * H, np.float32)
    v[0], v[H], v[2 * H], v[3 * H] = 2.0, 6.0, 10.0, 30.0
    st, y, probs = orc.gqa_attn_f32(q, k, v, 12, 2, H, 2)
    assert probs.tolist() == [0.5, 0.5]
    lanes = P["qwen_width_six"]["full_lane0"]
    for h in range(12):
        assert y[h * H] == lanes[0 if h < 6 else 1] and not y[h * H + 1:(h + 1) * H].any()
    st, y, probs = orc.gqa_attn_f32(q, k, v, 12, 2, H, 2, causal_pos=0)
    lanes = P["qwen_width_six"]["causal0_lane0"]
    for h in range(12):
        assert y[h * H] == lanes[0 if h < 6 else 1]


def test_gqa_shape_errors_do_not_write(orc):
    y = np.array([7.0, 8.0, 9.0, 10.0], np.float32)
    probs = np.array([3.0, 4.0], np.float32)
    st, _, _ = orc.gqa_attn_f32([1, 2, 3], [1, 0, 0, 1], [4, 5, 6, 7], 3, 2, 1, 2,
                                y=y[:3].copy(), probs=probs)
    assert st == orc.SHAPE and probs.tolist() == [3.0, 4.0]
    st, _, _ = orc.gqa_attn_f32([1, 2, 3, 4], [1, 0, 0, 1], [4, 5, 6, 7], 4, 2, 1, 2, y=y,
                                probs=np.full(8, 3.0, np.float32))
    assert st == orc.SHAPE and y.tolist() == [7.0, 8.0, 9.0, 10.0]
    # MHA and MQA are the same rule (gqa.rs:830-858)
    st, y2, _ = orc.gqa_attn_f32([9.0, 8.0], [1.0, 2.0], [3.0, 4.0], 2, 2, 1, 1)
    assert y2.tolist() == [3.0, 4.0]
    st, y2, _ = orc.gqa_attn_f32([9.0, 8.0], [1.0], [5.0], 2, 1, 1, 1, causal_pos=0)
    assert y2.tolist() == [5.0, 5.0]


# ------------------------------------------------------------------ rope.rs
def test_rope_pins(orc):
    P = PINS["rope"]
    assert np.float32(1e6).view(np.uint32) == hx(P["theta_bits"])
    heads = [1.0, -2.0, 3.5, -4.25]
    st, y = orc.rope_f32(heads, 0, 4, 1e6)
    assert y.tolist() == heads
    for case in P["d2_pos1"]:
        st, y = orc.rope_f32(case["x"], 1, 2, 1e6)
        assert bits(y) == [hx(b) for b in case["expect_bits"]]
    st, table = orc.rope_inv_freqs(4, 1e6)
    assert bits(table) == [hx(b) for b in P["d4_inv_freqs_bits"]]
    st, y = orc.rope_f32(P["d4_pos1_e1"]["x"], 1, 4, 1e6)
    assert bits(y) == [hx(b) for b in P["d4_pos1_e1"]["expect_bits"]]
    st, y = orc.rope_f32(P["d4_pos3"]["x"], 3, 4, 1e6)
    assert bits(y) == [hx(b) for b in P["d4_pos3"]["expect_bits"]]
    both = np.array(P["d4_pos3"]["x"] * 2, np.float32)
    st, yy = orc.rope_f32(both, 3, 4, 1e6)
    assert bits(yy[:4]) == bits(y) and bits(yy[4:]) == bits(y)
    x = np.zeros(128, np.float32)
    x[0] = 1.0
    st, y = orc.rope_f32(x, 1, 128, 1e6)
    assert bits(y[[0]]) == [hx(P["d128_pos1_e0"]["lane0_bits"])]
    assert bits(y[[64]]) == [hx(P["d128_pos1_e0"]["lane64_bits"])]
    st, table = orc.rope_inv_freqs(128, 1e6)
    for i, b in P["d128_table"].items():
        assert bits(table[[int(i)]]) == [hx(b)]
    last = np.zeros(128, np.float32)
    last[63], last[127] = 1.0, -2.0
    assert orc.rope_f32_inplace(last, 8, 128, 1e6) == 0
    assert bits(last[[63]]) == [hx(P["d128_pos8_last_pair"]["lane63_bits"])]
    assert bits(last[[127]]) == [hx(P["d128_pos8_last_pair"]["lane127_bits"])]


def test_rope_rejects_bad_shapes(orc):
    x = np.array([1, 2, 3, 4, 5], np.float32)
    st, y = orc.rope_f32(x, 1, 4, 1e6)
    assert st == orc.SHAPE
    three = np.array([9.0, 8.0, 7.0], np.float32)
    assert orc.rope_f32_inplace(three, 1, 3, 1e6) == orc.SHAPE and three.tolist() == [9, 8, 7]
    assert orc.rope_f32_inplace(np.zeros(0, np.float32), 0, 2, 1e6) == orc.SHAPE
    assert orc.rope_inv_freqs(3, 1e6)[0] == orc.SHAPE


# ------------------------------------------------------------------ swiglu.rs
def test_silu_and_mul_pins(orc):
    P = PINS["swiglu"]
    for z, want in P["silu_bits"]:
        assert bits([orc.silu_f32(z)]) == [hx(want)], z
    for z, not_want in P["silu_not_reciprocal"]:
        assert bits([orc.silu_f32(z)]) != [hx(not_want)]
    st, h = orc.swiglu_mul_f32(P["mul"]["gate"], P["mul"]["up"])
    assert bits(h) == [hx(b) for b in P["mul"]["expect_bits"]]
    st, _ = orc.swiglu_mul_f32([], [])
    assert st == orc.SHAPE


def test_swiglu_mlp_pins(orc):
    P = PINS["swiglu"]["mlp_2x2"]
    st, y, g, u, h = orc.swiglu_bf16(P["x"], orc.pack_bf16(P["gate_w"]), orc.pack_bf16(P["up_w"]),
                                     orc.pack_bf16(P["down_w"]), 2, 2)
    assert st == 0 and g.tolist() == P["gate"] and u.tolist() == P["up"]
    assert bits(h) == [hx(b) for b in P["h_bits"]] and bits(y) == [hx(b) for b in P["y_bits"]]
    st, y, g, u, h = orc.swiglu_bf16([1.0], np.array([0x80, 0x3F], np.uint8),
                                     np.array([0x00, 0x40], np.uint8),
                                     np.array([0x00, 0x40], np.uint8), 1, 1)
    assert bits(y) == [hx(PINS["swiglu"]["mlp_le"]["y_bits"])]


# ------------------------------------------------------------------ greedy_token
def test_greedy_token_rules(orc):
    assert orc.greedy_token([1.0, 2.0, 0.0, -1.0]) == 1
    assert orc.greedy_token([3.0, 3.0, 1.0]) == 0  # ties keep the lower index
    assert orc.greedy_token([np.nan, 1.0, 1.0]) == 1  # NaN never wins
    assert orc.greedy_token([np.nan, -np.inf, -np.inf]) == 0  # nothing beats -inf
    assert orc.greedy_token([-np.inf, 5.0, np.inf]) == 2


# ------------------------------------------------------------------ model_core
def _model(orc, shape, tensors, max_seq):
    wm = rf.load_into_oracle(orc, tensors)
    md = orc.Model(rf.oracle_shape(orc, shape), max_seq)
    assert md.status == 0
    return wm, md


def test_block_fixture_forward_prefill_decode(orc):
    P = PINS["block"]
    shape, t = rf.block_fixture()
    wm, md = _model(orc, shape, t, 4)
    assert md.forward_token(wm, 0, 0) == 0
    assert md.logits().tolist() == P["fixture_logits"]
    assert orc.greedy_token(md.logits()) == P["fixture_greedy"]
    assert md.kv_len() == 1
    st, k, v = md.kv_head(0, 0, 0)
    assert k.tolist() == [0.0, 0.0] and v.tolist() == P["fixture_cache_v0"]
    st, k, v = md.kv_head(0, 0, 1)
    assert v.tolist() == [0.0, 0.0]
    wm2, md2 = _model(orc, shape, t, 8)
    assert md2.prefill(wm2, []) == orc.SHAPE
    assert md2.prefill(wm2, [0]) == 0
    assert md2.logits().tolist() == P["fixture_logits"]
    st, out, gap, _ = md2.greedy_decode(wm2, 4)
    assert st == 0 and out.tolist() == P["fixture_decode4"] and md2.kv_len() == 5


def test_two_layers_and_errors_do_not_advance(orc):
    shape, t = rf.two_layer_fixture()
    wm, md = _model(orc, shape, t, 4)
    assert md.forward_token(wm, 0, 0) == 0
    assert md.logits().tolist() == [1.0, 2.0, 0.0, -1.0]
    assert md.kv_head(1, 0, 0)[2].tolist() == [0.0, 8.0]
    # errors (qwen25_block.rs:1224-1300)
    shape1, t1 = rf.block_fixture()
    wm1, md1 = _model(orc, shape1, t1, 2)
    assert md1.forward_token(wm1, 0, 1) == orc.POSITION
    assert md1.forward_token(wm1, 9, 0) == orc.TOKEN
    assert md1.kv_len() == 0
    empty = orc.WeightMap()
    assert md1.forward_token(empty, 0, 0) == orc.W_MISSING
    full_wm, full = _model(orc, shape1, t1, 1)
    assert full.forward_token(full_wm, 0, 0) == 0
    before = full.logits()
    assert full.forward_token(full_wm, 1, 1) == orc.CACHE_FULL
    assert full.kv_len() == 1 and full.logits().tolist() == before.tolist()
    # prefill rejects before any store (:1480-1513)
    wm3, md3 = _model(orc, shape1, t1, 4)
    assert md3.prefill(wm3, [0, 9]) == orc.TOKEN and md3.kv_len() == 0
    wm4, md4 = _model(orc, shape1, t1, 2)
    assert md4.prefill(wm4, [0, 0, 0]) == orc.CACHE_FULL


def _kv_bits(md, shape):
    out = []
    for layer in range(shape["num_layers"]):
        for head in range(shape["num_kv_heads"]):
            for pos in range(md.kv_len()):
                st, k, v = md.kv_head(layer, head, pos)
                out += bits(k) + bits(v)
    return out


def test_chunk_prefill_matches_serial_forward_bits(orc):
    # qwen25_block.rs:1403-1478
    shape = rf.rich_shape(2)
    t = rf.rich_map(shape)
    prompt = [1, 3, 0, 4, 2]
    wm_s, ms = _model(orc, shape, t, 16)
    wm_c, mc = _model(orc, shape, t, 16)
    assert ms.forward_token(wm_s, 2, 0) == 0 and mc.forward_token(wm_c, 2, 0) == 0
    for i, tok in enumerate(prompt):
        assert ms.forward_token(wm_s, tok, 1 + i) == 0
    assert mc.prefill(wm_c, prompt) == 0
    assert bits(mc.logits()) == bits(ms.logits())
    assert _kv_bits(mc, shape) == _kv_bits(ms, shape)
    st, os_, _, _ = ms.greedy_decode(wm_s, 3)
    st, oc, _, _ = mc.greedy_decode(wm_c, 3)
    assert os_.tolist() == oc.tolist() and bits(mc.logits()) == bits(ms.logits())
    wide = rf.rich_shape(1)
    t1 = rf.rich_map(wide)
    toks = [i % 5 for i in range(33)]
    wm_s, ms = _model(orc, wide, t1, 40)
    wm_c, mc = _model(orc, wide, t1, 40)
    for i, tok in enumerate(toks):
        assert ms.forward_token(wm_s, tok, i) == 0
    assert mc.prefill(wm_c, toks) == 0
    assert bits(mc.logits()) == bits(ms.logits()) and mc.kv_len() == 33
    assert _kv_bits(mc, wide) == _kv_bits(ms, wide)


def test_thread_count_does_not_change_tokens(orc):
    # weights_cli.rs:428-495: --threads does not change tokens
    shape = rf.rich_shape(2)
    t = rf.rich_map(shape)
    outs = []
    for threads in (1, 3, 8):
        orc.set_threads(threads)
        wm, md = _model(orc, shape, t, 16)
        assert md.prefill(wm, [1, 3, 0]) == 0
        st, out, _, _ = md.greedy_decode(wm, 5)
        outs.append((out.tolist(), bits(md.logits())))
    orc.set_threads(8)
    assert outs[0] == outs[1] == outs[2]
