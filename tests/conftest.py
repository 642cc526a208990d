"""Shared pytest setup: the ``gpu`` marker and fixture loaders."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the sm_100a kernels")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="CUDA is unavailable")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as f:
        return {key: f[key] for key in f.files}


def rel_err(actual, expected) -> float:
    """max |a - e| / max |e| (normwise relative error)."""
    a = torch.as_tensor(actual).double().cpu()
    e = torch.as_tensor(expected).double().cpu()
    return float((a - e).abs().max() / e.abs().max().clamp_min(1e-30))
