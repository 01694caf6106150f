"""Shared test setup: the `gpu` marker, repo paths, fixture loading helpers."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = Path(__file__).resolve().parent / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU and libgsa_b200.so")


@pytest.fixture(autouse=True)
def _gpu_guard(request):
    """A gpu-marked test fails loudly (never skips) when no CUDA device is present."""
    if request.node.get_closest_marker("gpu") is not None and not torch.cuda.is_available():
        pytest.fail("gpu test selected but torch.cuda.is_available() is False")
    yield


def load_golden(name: str) -> dict:
    return torch.load(GOLDEN / f"{name}.pt", weights_only=False)
