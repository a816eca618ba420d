"""The GEMM path's split attention under its scheduling switches, each read
once per process (so each setting runs in a child process of its own):

- MYOS_PF_ATTN_DYN=0: blocks walk the (row, KV head, split) items at a
  fixed stride instead of taking them from the shared queue, which the
  default uses for 256-row prompt chunks (a 512-id prompt). Which block
  computes an item does not change its arithmetic: bit-identical logits.
- MYOS_PF_MERGE_FUSED=0: the splits merged by a separate launch instead of
  by the last arriving split, which the default does for a 128-id chunk.
  Both run the same per-head merge: bit-identical logits.
- MYOS_PF_ATTN_WARPS=0: the dims-split kernel instead of the key-split one.
  The scores and p*v are summed in another order: logits within the GEMM
  path's tolerance (1e-2 absolute, 1e-3 relative) and the same argmax
  wherever the top-2 gap exceeds it."""
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "an-operating-system-for-ai-models-and-tensor-inference_b200")

CHILD = r"""
import sys
import numpy as np
sys.path.insert(0, sys.argv[1])
import myos
from myos import synth
shape = synth.shape_qwen25_1_5b()
e = myos.Engine(shape, 640)
try:
    e.load_table(synth.weights(shape, 1234))
    out = {}
    for n in (512, 128):
        e.reset()
        out["p%d" % n] = e.prefill(synth.prompt_ids(1234 + n, n, shape["vocab"]))
finally:
    e.close()
np.savez(sys.argv[2], **out)
"""


def _run(tmp_path, name, env_extra):
    env = dict(os.environ)
    for k in ("MYOS_PF_ATTN_DYN", "MYOS_PF_MERGE_FUSED", "MYOS_PF_ATTN_WARPS"):
        env.pop(k, None)
    env.update(env_extra)
    path = str(tmp_path / f"{name}.npz")
    r = subprocess.run([sys.executable, "-c", CHILD, PKG, path], env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    with np.load(path) as z:
        return {k: z[k] for k in z.files}


def test_split_attention_switches(tmp_path):
    ATOL, RTOL = 1e-2, 1e-3
    base = _run(tmp_path, "default", {})
    fixed = _run(tmp_path, "fixed_stride", {"MYOS_PF_ATTN_DYN": "0"})
    sep = _run(tmp_path, "separate_merge", {"MYOS_PF_MERGE_FUSED": "0"})
    dims = _run(tmp_path, "dims_split", {"MYOS_PF_ATTN_WARPS": "0"})
    for k in ("p512", "p128"):
        assert np.all(np.isfinite(base[k])), k
        assert np.array_equal(base[k].view(np.uint32), fixed[k].view(np.uint32)), k
        assert np.array_equal(base[k].view(np.uint32), sep[k].view(np.uint32)), k
        np.testing.assert_allclose(base[k], dims[k], atol=ATOL, rtol=RTOL, err_msg=k)
        top2 = np.sort(dims[k])[-2:]
        assert np.argmax(base[k]) == np.argmax(dims[k]) or top2[1] - top2[0] < ATOL, k
