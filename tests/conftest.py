"""Shared pytest setup: import paths, the ``gpu`` marker and golden-vector helpers."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "spikegpt-myelin_b200", ROOT / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device; run with -m gpu")


@pytest.fixture(scope="session")
def cuda():
    """The CUDA device for -m gpu tests. Fails (does not skip) without one, so a
    GPU run can never pass by skipping."""
    import torch

    assert torch.cuda.is_available(), "this test needs a CUDA device"
    return torch.device("cuda", 0)
