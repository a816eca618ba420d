"""Model fixtures restated from the reference's tests.

Each builder returns ``(shape_dict, tensors)`` where ``tensors`` maps a
SafeTensors key to ``(shape, little-endian bf16 bytes)``. The same table feeds
the CPU oracle and the CUDA engine, so the two run on identical bytes.

Sources (reference project paths):
  block_fixture / fixture_shape / fill_layer  crates/model_core/src/qwen25_block.rs:788-938
  rich_map / pat                              crates/model_core/src/qwen25_block.rs:1302-1382
"""
from __future__ import annotations

import numpy as np

LAYER_SUFFIXES = [
    "input_layernorm.weight",
    "self_attn.q_proj.weight",
    "self_attn.q_proj.bias",
    "self_attn.k_proj.weight",
    "self_attn.k_proj.bias",
    "self_attn.v_proj.weight",
    "self_attn.v_proj.bias",
    "self_attn.o_proj.weight",
    "post_attention_layernorm.weight",
    "mlp.gate_proj.weight",
    "mlp.up_proj.weight",
    "mlp.down_proj.weight",
]
EMBED = "model.embed_tokens.weight"
FINAL_NORM = "model.norm.weight"
LM_HEAD = "lm_head.weight"


def key(layer, suffix):
    return f"model.layers.{layer}.{suffix}"


def pack_bf16(values) -> np.ndarray:
    a = np.asarray(values, dtype=np.float32).reshape(-1)
    bits = a.view(np.uint32)
    assert np.all(bits & 0xFFFF == 0), "fixture value is not exact in bf16"
    return (bits >> 16).astype("<u2").view(np.uint8).copy()


def fixture_shape(num_layers=1):
    """qwen25_block.rs:788-801: hidden 2, 2 q heads, 1 kv head, head_dim 2, vocab 4, eps 0."""
    return dict(hidden=2, num_q_heads=2, num_kv_heads=1, head_dim=2, rope_theta=1e6,
                intermediate=2, vocab=4, num_layers=num_layers, rms_eps=0.0, tied_head=True)


def _put(t, name, shape, values):
    t[name] = (tuple(shape), pack_bf16(values))


def insert_embed_and_final(t):
    _put(t, EMBED, [4, 2], [1.0, 1.0, 2.0, 0.0, 0.0, 4.0, -1.0, 0.0])
    _put(t, FINAL_NORM, [2], [1.0, 0.0])


def fill_layer(t, layer, q_b, v_b, o_w, gate, up, down):
    _put(t, key(layer, "input_layernorm.weight"), [2], [1.0, 1.0])
    _put(t, key(layer, "self_attn.q_proj.weight"), [4, 2], [0.0] * 8)
    _put(t, key(layer, "self_attn.q_proj.bias"), [4], q_b)
    _put(t, key(layer, "self_attn.k_proj.weight"), [2, 2], [0.0] * 4)
    _put(t, key(layer, "self_attn.k_proj.bias"), [2], [0.0] * 2)
    _put(t, key(layer, "self_attn.v_proj.weight"), [2, 2], [0.0] * 4)
    _put(t, key(layer, "self_attn.v_proj.bias"), [2], v_b)
    _put(t, key(layer, "self_attn.o_proj.weight"), [2, 4], o_w)
    _put(t, key(layer, "post_attention_layernorm.weight"), [2], [1.0, 1.0])
    _put(t, key(layer, "mlp.gate_proj.weight"), [2, 2], gate)
    _put(t, key(layer, "mlp.up_proj.weight"), [2, 2], up)
    _put(t, key(layer, "mlp.down_proj.weight"), [2, 2], down)


def block_fixture():
    t = {}
    insert_embed_and_final(t)
    fill_layer(t, 0, [0.5, 0.0, 0.0, 0.25], [1.0, 0.0],
               [1.0, 0.0, 0.0, 0.0, 1.0, 0.0, 0.0, 0.0], [0.0] * 4, [0.0] * 4, [0.0] * 4)
    return fixture_shape(), t


def swiglu_fixture():
    """qwen25_block.rs:1073-1130 (swiglu_residual_changes_the_logits)."""
    t = {}
    insert_embed_and_final(t)
    fill_layer(t, 0, [0.5, 0.0, 0.0, 0.25], [1.0, 0.0],
               [1.0, 0.0, 0.0, 0.0, 1.0, 0.0, 0.0, 0.0],
               [1.0, 0.0, 0.0, 0.0], [1.0, 0.0, 0.0, 0.0], [1.0, 0.0, 0.0, 1.0])
    return fixture_shape(), t


def two_layer_fixture():
    """qwen25_block.rs:1132-1198 (two_layers_advance_once_per_token)."""
    t = {}
    insert_embed_and_final(t)
    z8, z4 = [0.0] * 8, [0.0] * 4
    fill_layer(t, 0, [0.0] * 4, [2.0, 0.0], z8, z4, z4, z4)
    fill_layer(t, 1, [0.0] * 4, [0.0, 8.0], z8, z4, z4, z4)
    return fixture_shape(2), t


_PAT = [0.5, -0.25, 1.0, 0.0, -1.0, 0.125, 2.0, -0.5]


def _put_pat(t, name, shape, salt):
    n = int(np.prod(shape))
    _put(t, name, shape, [_PAT[(i + salt) % 8] for i in range(n)])


def rich_shape(num_layers=2):
    """qwen25_block.rs:1405-1418 (chunk_prefill_matches_serial_forward_token_bits)."""
    return dict(hidden=8, num_q_heads=4, num_kv_heads=2, head_dim=2, rope_theta=1e6,
                intermediate=6, vocab=5, num_layers=num_layers, rms_eps=1e-6, tied_head=True)


def rich_map(shape):
    """qwen25_block.rs:1313-1382: patterned multi-layer weights."""
    h = shape["hidden"]
    qd = shape["num_q_heads"] * shape["head_dim"]
    kvd = shape["num_kv_heads"] * shape["head_dim"]
    inter = shape["intermediate"]
    t = {}
    _put_pat(t, EMBED, [shape["vocab"], h], 1)
    _put_pat(t, FINAL_NORM, [h], 2)
    for layer in range(shape["num_layers"]):
        salt = 10 + layer * 20
        _put_pat(t, key(layer, "input_layernorm.weight"), [h], salt)
        _put_pat(t, key(layer, "self_attn.q_proj.weight"), [qd, h], salt + 1)
        _put_pat(t, key(layer, "self_attn.q_proj.bias"), [qd], salt + 2)
        _put_pat(t, key(layer, "self_attn.k_proj.weight"), [kvd, h], salt + 3)
        _put_pat(t, key(layer, "self_attn.k_proj.bias"), [kvd], salt + 4)
        _put_pat(t, key(layer, "self_attn.v_proj.weight"), [kvd, h], salt + 5)
        _put_pat(t, key(layer, "self_attn.v_proj.bias"), [kvd], salt + 6)
        _put_pat(t, key(layer, "self_attn.o_proj.weight"), [h, qd], salt + 7)
        _put_pat(t, key(layer, "post_attention_layernorm.weight"), [h], salt + 8)
        _put_pat(t, key(layer, "mlp.gate_proj.weight"), [inter, h], salt + 9)
        _put_pat(t, key(layer, "mlp.up_proj.weight"), [inter, h], salt + 10)
        _put_pat(t, key(layer, "mlp.down_proj.weight"), [h, inter], salt + 11)
    return t


def load_into_oracle(orc, tensors):
    """Insert a fixture table into an oracle WeightMap (borrowed bytes)."""
    wm = orc.WeightMap()
    for name, (shape, data) in tensors.items():
        st = wm.insert_bf16(name, list(shape), data)
        assert st == 0, (name, st)
    return wm


def oracle_shape(orc, shape):
    return orc.Shape(**shape)
