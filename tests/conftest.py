import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the kernels through the C ABI")


@pytest.fixture(scope="session")
def cuda():
    """The CUDA device for gpu-marked tests.  Absence is a failure, not a skip
    (like the reference's CUDA_REQUIRED=1 gate, compute-cuda/tests/convolution.rs:10-25)."""
    import torch

    if not torch.cuda.is_available():
        pytest.fail("gpu test without a CUDA device")
    from forma_b200 import _lib

    _lib.load()  # the in-tree sm_100a library must load; there is no fallback
    return torch.device("cuda:0")
