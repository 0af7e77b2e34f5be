"""Test configuration: the ``gpu`` marker and import paths.

``-m "not gpu"`` tests run on any host: the oracle against the golden vectors made
from the reference, host-side logic, and the C-ABI library's symbol table.
``-m gpu`` tests launch the sm_100a kernels through the C-ABI and compare them with
the oracle.
"""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PACKAGE_DIR = ROOT / "-sglang-decode-_b200"
for path in (str(ROOT), str(PACKAGE_DIR)):
    if path not in sys.path:
        sys.path.insert(0, path)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: launches sm_100a kernels on a CUDA device")


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    return torch.device("cuda", 0)
