"""Pytest configuration: the ``gpu`` marker and shared fixtures.

Tests marked ``gpu`` need a CUDA device and the in-tree CUDA library; the
CPU suite (``-m "not gpu"``) checks the oracle against golden vectors, the
host-side logic and that the C-ABI library exports its declared symbols.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU and the built sm_100a library")


@pytest.fixture(scope="session")
def golden():
    with np.load(ROOT / "tests" / "golden" / "golden.npz") as data:
        return {key: data[key] for key in data.files}
