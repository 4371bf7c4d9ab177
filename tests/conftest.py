"""Shared test setup: import paths, the `gpu` marker, seeded input helpers."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
PKG_ROOT = REPO / "quantem-cuda_b200"
for p in (str(PKG_ROOT), str(REPO)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); parity tests proper")


@pytest.fixture(scope="session")
def tv_golden():
    with np.load(GOLDEN / "tv_golden.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def kp_golden():
    with np.load(GOLDEN / "kplanes_golden.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def kp_tv_golden():
    with np.load(GOLDEN / "kplanes_tv_golden.npz") as z:
        return {k: z[k] for k in z.files}


def golden_cases(data: dict) -> list[str]:
    return sorted({k.split("/")[0] for k in data})
