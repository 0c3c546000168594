"""Shared test setup: the repository root on sys.path, the `gpu` marker, and
helpers that bind the oracle (test infrastructure) and golden fixtures."""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests" / "golden"))

GOLDEN_DIR = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


def has_cuda() -> bool:
    import torch

    return torch.cuda.is_available()


@pytest.fixture(scope="session")
def golden():
    data = np.load(GOLDEN_DIR / "golden.npz")
    meta = json.loads((GOLDEN_DIR / "golden.json").read_text())
    return {k: data[k].astype(np.int64) for k in data.files}, meta


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle

    if not oracle.LIB.exists():
        oracle.build()
    return oracle
