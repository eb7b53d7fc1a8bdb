"""Shared pytest setup: import paths and the ``gpu`` marker."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
PKG_ROOT = REPO / "ssd-rwkv-engine_b200"
for p in (str(REPO), str(PKG_ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden_dir() -> Path:
    return GOLDEN


def load_golden(name: str) -> dict:
    import numpy as np

    with np.load(GOLDEN / name, allow_pickle=False) as z:
        return {k: z[k] for k in z.files}


def cases(d: dict) -> list[str]:
    return sorted({k.split("/")[0] for k in d if "/" in k})
