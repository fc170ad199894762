import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "mono-qwen27_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200 / sm_100a)")


@pytest.fixture(scope="session")
def golden():
    return np.load(os.path.join(ROOT, "tests", "golden", "golden.npz"))


@pytest.fixture(scope="session")
def orc():
    from oracle import build as ob
    ob.build_oracle()
    from oracle import oracle
    return oracle


@pytest.fixture(scope="session")
def m27b():
    import m27b as M
    M.lib()
    return M


@pytest.fixture(scope="session")
def torch():
    import torch as T
    assert T.cuda.is_available(), "GPU tests need a CUDA device"
    return T
