"""Shared pytest setup: markers, import paths and golden-fixture loading."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "dsalt-library_b200"
GOLDEN = ROOT / "tests" / "golden"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_golden(name: str):
    import torch
    return torch.load(GOLDEN / name, weights_only=False)


@pytest.fixture(scope="session")
def golden_ops():
    return load_golden("ops.pt")


@pytest.fixture(scope="session")
def golden_selectors():
    return load_golden("selectors.pt")


def cuda_ok() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False
