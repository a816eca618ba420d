"""myos_dev_gqa_attn_f32_noalloc: the split-KV attention with its scratch in a
fixed static device array (no allocation), against the allocating host-slice
entry point myos_gqa_attn_f32 (tensor_core::gqa_attn_f32,
crates/tensor_core/src/gqa.rs:174-218) on the same seeded inputs, two calls in
a row on one stream.

The device buffers here are the test's own (torch); the entry point under
test allocates nothing, which the driver's free-memory count confirms across
the calls. Collected last so it also runs after every other GPU test in the
same process; it passes alone in a fresh process too.
"""
import ctypes as C

import numpy as np
import pytest

from myos import _lib

pytestmark = pytest.mark.gpu

# Both entry points run the same kernel with the same split geometry, so the
# outputs are expected to be bit-identical; the stated bound is float noise.
RTOL, ATOL = 1e-6, 1e-6

# (hq, hkv, d, seq, mask_kind, query_pos)
CASES = [
    (12, 2, 128, 200, 0, 0),      # Qwen2.5-1.5B heads, 7 splits
    (12, 2, 128, 256, 1, 130),    # causal: keys 0..130
    (40, 8, 128, 1000, 1, 999),   # Qwen2.5-14B heads, 32 splits
    (8, 8, 64, 5, 0, 0),          # one query head per KV head, a single ragged split
    (12, 2, 128, 2048, 0, 0),     # the most splits (64)
]


def _inputs(hq, hkv, d, seq, seed):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal(hq * d).astype(np.float32)
    k = rng.standard_normal(hkv * seq * d).astype(np.float32)
    v = rng.standard_normal(hkv * seq * d).astype(np.float32)
    return q, k, v


def _host(L, q, k, v, hq, hkv, d, seq, mask, qpos):
    y = np.empty(hq * d, np.float32)
    f = C.POINTER(C.c_float)
    st = L.myos_gqa_attn_f32(y.ctypes.data_as(f), y.size, q.ctypes.data_as(f), q.size,
                             k.ctypes.data_as(f), k.size, v.ctypes.data_as(f), v.size,
                             hq, hkv, d, seq, mask, qpos)
    assert st == _lib.OK, _lib.status_name(st)
    return y


@pytest.mark.parametrize("case", CASES, ids=lambda c: "hq%d_hkv%d_d%d_seq%d_m%d" % c[:5])
def test_noalloc_matches_allocating_entry(case):
    import torch

    hq, hkv, d, seq, mask, qpos = case
    L = _lib.load()
    q, k, v = _inputs(hq, hkv, d, seq, seed=hq * 7919 + seq)
    ref = _host(L, q, k, v, hq, hkv, d, seq, mask, qpos)

    dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, k, v))
    dy = torch.empty(hq * d, dtype=torch.float32, device="cuda")

    def call():
        dy.fill_(float("nan"))
        st = L.myos_dev_gqa_attn_f32_noalloc(dy.data_ptr(), dq.data_ptr(), dk.data_ptr(),
                                             dv.data_ptr(), hq, hkv, d, seq, mask, qpos, None)
        assert st == _lib.OK, _lib.status_name(st)
        torch.cuda.synchronize()
        return dy.cpu().numpy()

    call()  # the first call on a device resolves the scratch address
    free0 = torch.cuda.mem_get_info()[0]
    first = call()
    second = call()
    free1 = torch.cuda.mem_get_info()[0]
    assert free1 == free0, "device memory changed across the calls"
    for out in (first, second):
        assert np.isfinite(out).all()
        np.testing.assert_allclose(out, ref, rtol=RTOL, atol=ATOL)
    assert np.array_equal(first.view(np.uint32), second.view(np.uint32))


def test_noalloc_rejects_beyond_scratch():
    import torch

    L = _lib.load()
    hq, hkv, d, seq = 64, 8, 256, 4096
    # Buffers of the full declared size, so that the call reads only memory it
    # owns even if the scratch size or the split rule ever changed and the
    # request were accepted.
    dq = torch.zeros(hq * d, device="cuda")
    dk = torch.zeros(hkv * seq * d, device="cuda")
    dv = torch.zeros(hkv * seq * d, device="cuda")
    dy = torch.full((hq * d,), float("nan"), device="cuda")
    # 8 KV heads x 64 splits x 8 query heads x 256 lanes of f32 partials = 4 MiB
    st = L.myos_dev_gqa_attn_f32_noalloc(dy.data_ptr(), dq.data_ptr(), dk.data_ptr(),
                                         dv.data_ptr(), hq, hkv, d, seq, 0, 0, None)
    assert st == _lib.ERR_SCRATCH_LIMIT, _lib.status_name(st)
    torch.cuda.synchronize()
    assert torch.isnan(dy).all(), "a rejected call wrote its output"
    st = L.myos_dev_gqa_attn_f32_noalloc(None, dy.data_ptr(), dy.data_ptr(), dy.data_ptr(),
                                         12, 2, 128, 16, 0, 0, None)
    assert st == _lib.ERR_ARG
