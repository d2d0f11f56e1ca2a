"""Shared test set-up: import paths, markers, seeding, fixture loading."""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
PKG_DIR = ROOT / "realtime-gs_b200"
for p in (str(ROOT), str(PKG_DIR)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running test")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="needs a CUDA GPU")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(autouse=True)
def _seed_everything():
    torch.manual_seed(0)
    yield


def load_golden(name: str) -> dict[str, np.ndarray]:
    with np.load(GOLDEN / f"{name}.npz") as data:
        return {k: data[k] for k in data.files}


def t(a) -> torch.Tensor:
    """numpy -> torch (keeps dtype)."""
    return torch.from_numpy(np.ascontiguousarray(a))


def has_gpu() -> bool:
    return torch.cuda.is_available() and os.environ.get("RTGS_B200_FORCE_NO_GPU") != "1"


def rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    """max |a - b| / max |b| (0 when both are zero)."""
    a = a.detach().double().cpu()
    b = b.detach().double().cpu()
    den = float(b.abs().max()) if b.numel() else 0.0
    num = float((a - b).abs().max()) if b.numel() else 0.0
    return 0.0 if num == 0.0 else num / max(den, 1e-30)
