import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "an-operating-system-for-ai-models-and-tensor-inference_b200")
for p in (REPO, PKG, os.path.join(REPO, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: takes more than a few seconds on CPU")


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle as orc_mod

    orc_mod.build()
    return orc_mod


def pytest_collection_modifyitems(config, items):
    """GPU tests need a CUDA device; on a CPU-only host they are skipped."""
    has_gpu = os.path.exists("/dev/nvidiactl") or os.path.exists("/dev/nvidia0")
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device on this host")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
