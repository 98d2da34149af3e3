"""Shared pytest setup: the ``gpu`` marker and the repo root on ``sys.path``."""

from __future__ import annotations

import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 and the built sm_100a library")
