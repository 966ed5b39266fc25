"""Shared pytest setup: the `gpu` marker, fixture loading, scenario building."""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(GOLDEN))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def _has_gpu() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False


def pytest_collection_modifyitems(config, items):
    if _has_gpu():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def load_golden(name: str):
    meta = json.loads((GOLDEN / f"{name}.json").read_text())
    arrays = dict(np.load(GOLDEN / f"{name}.npz"))
    return meta, arrays


@pytest.fixture(scope="session")
def golden():
    return load_golden
