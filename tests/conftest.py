"""pytest configuration: the ``gpu`` marker and shared fixtures.

``-m "not gpu"`` runs on any host (oracle vs golden vectors, host logic, the C ABI's
exports and host-side validation).  ``-m gpu`` needs a B200 and calls the kernels
through the C ABI.
"""
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
for path in (ROOT, ROOT / "tests"):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device; calls the native kernels")


def load_golden(name):
    return torch.load(GOLDEN / name, weights_only=False)


@pytest.fixture(scope="session")
def golden():
    return load_golden
