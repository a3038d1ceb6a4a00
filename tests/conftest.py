"""Shared test set-up: import paths, the ``gpu`` marker, fixture loaders."""

from __future__ import annotations

import os
import sys
from pathlib import Path

# The host math library picks its thread count per call under load unless told not to, and a float32
# matmul's rounding then varies from run to run; the drop-in tests compare against fixtures made with
# a fixed thread count.
os.environ.setdefault("MKL_DYNAMIC", "FALSE")
os.environ.setdefault("OMP_DYNAMIC", "FALSE")

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
for path in (ROOT, ROOT / "dimmer-kv_b200", GOLDEN):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a) and the built library")


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz", allow_pickle=False) as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def golden():
    cache = {}

    def get(name):
        if name not in cache:
            cache[name] = load_golden(name)
        return cache[name]

    return get
