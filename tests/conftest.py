"""Shared test setup.

The package lives in ``stream-mm2026_b200/`` (``mdq_b200``); the CPU oracle and
the reference-extension recipe live in ``oracle/`` and are test
infrastructure.  Tests marked ``gpu`` need a B200; the rest run on CPU.
"""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_ROOT = os.path.join(REPO, "stream-mm2026_b200")
for p in (PKG_ROOT, REPO, os.path.join(REPO, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("gpu test collected without a CUDA device")
    return torch.device("cuda:0")
