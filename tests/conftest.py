"""Test setup: the package lives in ``ssd-tpu-_b200/`` (a hyphenated directory), the
oracle in ``oracle/``.  ``-m gpu`` tests need a CUDA device and the built library."""

from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "ssd-tpu-_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built libssdverify.so")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


@pytest.fixture(autouse=True)
def _use_toy_model(monkeypatch):
    # tests/conftest.py:10-13 of the reference: toy backend unless real weights are asked for
    if os.getenv("SSD_USE_REAL_MODEL") not in ("1", "true", "yes"):
        monkeypatch.setenv("SSD_USE_TOY_MODEL", "1")
