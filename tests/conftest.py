"""Shared test setup: import paths, the `gpu` marker, seeded RNG helpers."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT / "oracle"))
sys.path.insert(0, str(ROOT / "oxide-forge_b200"))
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built liboxf.so")


@pytest.fixture
def rng():
    return np.random.default_rng(1234)


def rel_err(got, want) -> float:
    """max |got - want| / max |want| (normwise relative error)."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    denom = max(np.abs(want).max(), 1e-30)
    return float(np.abs(got - want).max() / denom)
