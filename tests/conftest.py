"""Shared pytest setup: the ``gpu`` marker, the repo root on ``sys.path``, and a fixed torch
seed before every test, so a test sees the same random inputs whichever tests ran before it."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 and the built sm_100a library")


@pytest.fixture(autouse=True)
def _fixed_torch_seed():
    torch.manual_seed(0)
    yield
