"""The product path has no CPU fallback: without the built CUDA library the
bindings refuse to load, and on a host without a GPU every compute entry
point returns MYOS_ERR_CUDA instead of computing (host-only checks such as
shape validation still answer first). Runs on CPU only."""
import os

import numpy as np
import pytest

import myos
from myos import _lib, ops


def _has_gpu():
    return os.path.exists("/dev/nvidiactl") or os.path.exists("/dev/nvidia0")


def test_missing_library_raises(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "CUDA_LIB", str(tmp_path / "libmyos_cuda.so"))
    monkeypatch.setattr(_lib, "_lib", None)
    with pytest.raises(RuntimeError, match="missing"):
        _lib.load()


@pytest.mark.skipif(_has_gpu(), reason="checks the no-GPU behaviour")
def test_compute_calls_fail_with_cuda_status_on_a_cpu_host():
    import build as pkg_build
    pkg_build.build()
    from myos import synth
    w = np.zeros(4 * 256, np.uint16).view(np.uint8)
    st, _ = ops.gemv_bf16(w, np.ones(256, np.float32), 4, 256)
    assert st == _lib.ERR_CUDA
    with pytest.raises(myos.MyosError) as e:
        myos.Engine(synth.shape_qwen25_1_5b(), 16)
    assert e.value.code == _lib.ERR_CUDA
    from myos import tp
    st, _ = tp.reduce_selftest(2, 256, fill=True)
    assert st == _lib.ERR_CUDA
