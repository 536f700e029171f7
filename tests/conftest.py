"""Shared pytest configuration.

``-m gpu`` tests need a CUDA device and the built library
(``python -m flatrun_b200.build``); everything else runs on CPU.
"""

from __future__ import annotations

import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libfrcuda.so")


@pytest.fixture(scope="session")
def cuda_backend():
    from flatrun_b200 import CudaBackend

    be = CudaBackend(0)
    if not be.available:
        raise RuntimeError(f"CUDA backend unavailable on a GPU test run: {be._load_error}")
    yield be
    be.close()
