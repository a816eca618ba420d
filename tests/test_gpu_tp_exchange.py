"""The tensor-parallel exchange's reduce kernel on one GPU
(myos_tp_reduce_selftest): with every rank's words present it sums them in
rank order exactly as f32 adds do; with an inbox that nothing writes, its
bounded wait gives up after the requested time and the host reads
MYOS_ERR_TIMEOUT (the GPU is never hung: the kernel returns)."""
import time

import numpy as np
import pytest

from myos import _lib, tp

pytestmark = pytest.mark.gpu


def expected(n, H):
    i = np.arange(H, dtype=np.float32)
    s = np.float32(0.25) * np.float32(1) + i * np.float32(1.0 / 1024)
    for p in range(1, n):
        s = s + (np.float32(0.25) * np.float32(p + 1) + i * np.float32(1.0 / 1024))
    return s.astype(np.float32)


@pytest.mark.parametrize("n,H", [(1, 256), (2, 1536), (2, 5120), (8, 5120), (3, 1000)])
def test_reduce_sums_every_rank_in_order(n, H):
    st, out = tp.reduce_selftest(n, H, fill=True)
    assert st == 0, _lib.status_name(st)
    np.testing.assert_array_equal(out, expected(n, H))


def test_reduce_wait_gives_up_and_reports():
    t0 = time.time()
    st, _ = tp.reduce_selftest(2, 1536, fill=False, timeout_ms=200)
    assert st == _lib.ERR_TIMEOUT, _lib.status_name(st)
    assert time.time() - t0 < 10.0
    # the device stays usable after a timed-out wait
    st, out = tp.reduce_selftest(2, 1536, fill=True)
    assert st == 0 and np.array_equal(out, expected(2, 1536))
