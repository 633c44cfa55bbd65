"""Shared test setup: import paths, the ``gpu`` marker and common fixtures.

Tests marked ``gpu`` run on a B200 and call the CUDA library through its C ABI;
everything else runs on the CPU (oracle vs golden fixtures, host-side logic,
ABI exports, multi-process gloo tests).
"""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "mlsys26-flashinfer-moe_b200")
for p in (PKG, os.path.join(REPO, "oracle"), os.path.join(REPO, "tests", "golden"),
          os.path.join(REPO, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
