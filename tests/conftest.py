"""Test setup: import paths, the ``gpu`` marker and shared helpers.

``-m "not gpu"`` runs on any host (oracle vs golden vectors, host logic, C-ABI exports).
``-m gpu`` runs the parity tests proper on a B200: CUDA kernels through the C ABI against the
CPU oracle in ``oracle/``.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
for path in (ROOT / "llm-serving_b200", ROOT):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (runs the sm_100a kernels)")


@pytest.fixture(autouse=True)
def _seed():
    torch.manual_seed(0)
    yield


@pytest.fixture(scope="session")
def cuda_device():
    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device; run it with -m gpu on a B200")
    return torch.device("cuda", 0)
