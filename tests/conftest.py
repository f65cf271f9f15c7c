"""Shared pytest setup: markers, import paths, GPU detection."""
from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "pallas-kernel_b200"
for p in (str(ROOT), str(PKG), str(ROOT / "tests" / "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device; the parity tests proper")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def cuda_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture
def device():
    return "cuda"
