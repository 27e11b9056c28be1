"""Test configuration: the `gpu` marker and shared helpers.

`-m "not gpu"` runs on any host (oracle, host logic, the C ABI's exports);
`-m gpu` runs the parity tests on a B200 through libvoxcpm_b200.so.
"""

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device (run with -m 'not gpu' on CPU hosts)")
    torch.cuda.init()
    return torch.device("cuda:0")
