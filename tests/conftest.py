import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN_DIR = os.path.join(ROOT, "tests", "golden")
if GOLDEN_DIR not in sys.path:
    sys.path.insert(0, GOLDEN_DIR)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built libturbopolar.so")


@pytest.fixture(scope="session")
def golden():
    return np.load(os.path.join(GOLDEN_DIR, "golden.npz"))


@pytest.fixture(scope="session")
def golden_meta():
    import json
    with open(os.path.join(GOLDEN_DIR, "golden_meta.json")) as f:
        return json.load(f)


def has_cuda():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(autouse=True)
def _guard_bytes(request):
    """GPU tests run with canary guard bytes around the runtime's device buffers (page pools,
    radius scales, dense tails, state words; turbopolar_b200.guard) and check them afterwards:
    a kernel write past any of those buffers fails the test that made it."""
    if request.node.get_closest_marker("gpu") is None or not has_cuda():
        yield
        return
    from turbopolar_b200 import guard
    guard.enable(4096)
    try:
        yield
        guard.check()
    finally:
        guard.disable()
