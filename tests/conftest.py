import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "oracle"))
GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device; run with -m gpu")


@pytest.fixture(scope="session")
def oracle():
    import oracle as _oracle  # oracle/oracle.py (test infrastructure)

    _oracle.lib()
    return _oracle


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device (run GPU tests with -m gpu on a B200)")
    from origami_b200 import _lib

    _lib.lib()  # the CUDA library must load: no fallback exists
    return torch.device("cuda", 0)
