"""pytest configuration: import paths for the package directory and the oracle, and the `gpu` marker."""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "glm53-exl3-prefill_b200")
ORACLE = os.path.join(REPO, "oracle")
GOLDEN = os.path.join(REPO, "tests", "golden")
for p in (PKG, ORACLE):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a); run with -m gpu on the GPU host")


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but CUDA is not available")
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def ext(cuda_device):
    """The C-ABI binding; fails (never skips) when the library is missing."""
    import b200_ext
    b200_ext.load()
    return b200_ext
