import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

GOLDEN = os.path.join(REPO, "tests", "golden", "golden_v1.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle.oracle import Reference
    try:
        return Reference()
    except FileNotFoundError as e:
        pytest.skip(str(e))


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return np.load(GOLDEN)


@pytest.fixture(scope="session")
def kq():
    """The library, initialised on cuda:0 (GPU tests only)."""
    import torch
    assert torch.cuda.is_available(), "GPU test without a GPU"
    torch.cuda.init()
    from trailblaze_b200 import load
    lib = load()
    assert lib.tb_cuda_init() == 1
    return lib
