import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built libq8cuda.so")
    config.addinivalue_line("markers", "slow: long-running (full-size model dims)")


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN


@pytest.fixture(scope="session")
def cuda():
    """GPU tests run only where a GPU exists and fail loudly otherwise."""
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    from lama32_mojo_b200 import _lib
    _lib.lib()  # raises if libq8cuda.so is missing: no fallback path exists
    torch.cuda.set_device(0)
    return torch.device("cuda:0")
