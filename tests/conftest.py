"""Shared pytest setup: the ``gpu`` marker and import paths.

Tests marked ``gpu`` need a CUDA device and the built ``libtorque_b200.so``;
everything else runs on CPU."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN_PATH = ROOT / "tests" / "golden" / "golden.npz"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built CUDA library")


@pytest.fixture(scope="session")
def golden():
    with np.load(GOLDEN_PATH) as z:
        return {k: z[k] for k in z.files}
