"""Shared pytest configuration.

Markers:
- ``gpu``: needs a CUDA device with the built ``libmround_b200.so``; the
  CPU suite runs with ``-m "not gpu"``.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a B200 and the compiled CUDA library")


@pytest.fixture(scope="session")
def golden() -> dict[str, np.ndarray]:
    with np.load(GOLDEN / "golden.npz") as data:
        return {k: data[k] for k in data.files}


def relative_error(got: np.ndarray, expected: np.ndarray) -> float:
    """Max |difference| over max |expected| (reference tests/unit/test_mlx_parity.py:95-98)."""
    got = np.asarray(got, dtype=np.float64)
    expected = np.asarray(expected, dtype=np.float64)
    denom = max(1e-12, float(np.abs(expected).max(initial=0.0)))
    return float(np.abs(got - expected).max(initial=0.0) / denom)


os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
