"""Launch-timeline summary (myos.ktrace) on a synthetic trace: host only."""
import numpy as np

from myos import ktrace


def test_summary_of_a_regular_timeline(tmp_path):
    layers, ns = 2, 11
    t = np.zeros((ktrace.STEPS, ns, ktrace.WIDTH), np.uint64)
    # every kernel: 1 us prologue, 3 us run, then 2 us until the next one's wait
    for st in range(ktrace.STEPS):
        base = 100_000 * st
        for sl in range(ns):
            start = base + 5_000 * sl
            t[st, sl, 0] = start
            t[st, sl, 1] = start + 1_000
            t[st, sl, 2] = start + 4_000
    p = tmp_path / "kt.bin"
    t.tofile(p)
    out = ktrace.summarize(str(p), layers)
    assert abs(out["token_us"] - 100.0) < 1e-9
    for k in ktrace.KINDS:
        assert out[k] == {"gap_us": 2.0 if k != "qkv" else 1.0, "run_us": 3.0, "prewait_us": 1.0}
    assert out["head"] == {"gap_us": 2.0, "run_us": 3.0, "prewait_us": 1.0}
