"""Seeded synthetic inputs: deterministic, thread-count independent, and
distributed as the BASELINE configs describe (CPU only)."""
import numpy as np
import pytest

from myos import synth


@pytest.fixture(scope="module", autouse=True)
def built():
    import build as pkg_build

    pkg_build.build()


def bf16_to_f32(u16):
    return (u16.astype(np.uint32) << 16).view(np.float32)


def test_deterministic_and_thread_invariant():
    a = synth.normal_bf16(7, 3, 300001, 0.0, 0.02, threads=1)
    b = synth.normal_bf16(7, 3, 300001, 0.0, 0.02, threads=8)
    assert np.array_equal(a, b)
    c = synth.normal_bf16(7, 4, 300001, 0.0, 0.02, threads=8)
    assert not np.array_equal(a, c)
    # prefix property: element i does not depend on n
    d = synth.normal_bf16(7, 3, 1001, 0.0, 0.02, threads=3)
    assert np.array_equal(a[:1001], d)


def test_distributions():
    w = bf16_to_f32(synth.normal_bf16(1, 0, 1 << 20, 0.0, 0.02))
    assert abs(w.mean()) < 2e-4 and abs(w.std() - 0.02) < 2e-4
    g = bf16_to_f32(synth.normal_bf16(1, 1, 1 << 20, 1.0, 0.01))
    assert abs(g.mean() - 1.0) < 2e-4 and abs(g.std() - 0.01) < 3e-4
    x = synth.normal_f32(1, 2, 1 << 20)
    assert abs(x.mean()) < 5e-3 and abs(x.std() - 1.0) < 5e-3


def test_bf16_is_round_to_nearest_even():
    # regenerate the f32 values and round them here
    f = synth.normal_f32(5, 9, 4096, 0.0, 0.02)
    u = f.view(np.uint32)
    rne = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    assert np.array_equal(synth.normal_bf16(5, 9, 4096, 0.0, 0.02), rne)


def test_prompt_ids_in_range_and_seeded():
    p = synth.prompt_ids(1234, 4096, 151936)
    assert p.dtype == np.uint32 and p.max() < 151936 and len(set(p.tolist())) > 4000
    assert np.array_equal(p, synth.prompt_ids(1234, 4096, 151936))
    assert not np.array_equal(p, synth.prompt_ids(1235, 4096, 151936))


def test_tensor_specs_match_layout():
    specs = synth.tensor_specs(synth.shape_qwen25_1_5b())
    assert len(specs) == 28 * 12 + 2  # TENSOR_COUNT, qwen25_layout.rs:49-50
    assert synth.weight_bytes(synth.shape_qwen25_1_5b()) == 3_087_428_608
    specs14 = synth.tensor_specs(synth.shape_qwen25_14b())
    assert specs14[-1][0] == "lm_head.weight" and len(specs14) == 48 * 12 + 3
