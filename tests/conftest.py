"""Pytest configuration: the ``gpu`` marker and shared fixtures."""

from __future__ import annotations

import pathlib
import sys

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden" / "oracle_golden.npz"


def pytest_configure(config) -> None:
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built libtempo_b200.so")


@pytest.fixture(scope="session")
def golden() -> dict:
    with np.load(GOLDEN, allow_pickle=False) as data:
        return {name: data[name] for name in data.files}


def cuda_ready() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:  # noqa: BLE001
        return False
