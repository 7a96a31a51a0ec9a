"""Test configuration: import paths and the ``gpu`` marker.

``-m "not gpu"`` runs on any machine (oracle vs golden fixtures, host logic,
C-ABI exports, gloo multi-process harness). ``-m gpu`` needs a B200 and runs
the CUDA paths through the C-ABI library against the oracle.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT / "sm90-fp8-wgrad_b200", ROOT / "oracle", ROOT / "tests" / "golden", ROOT):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (sm_100a) and the built C-ABI library")


@pytest.fixture(scope="session")
def golden_dir() -> Path:
    return GOLDEN


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.skip(f"needs compute capability 10.0, got {major}.{minor}")
    return torch.device("cuda:0")


@pytest.fixture(autouse=True)
def _isolated_layout_mode(monkeypatch):
    """Every test starts without KERNEL_LAB_WGRAD_LAYOUT_MODE and gets the
    caller's value back afterwards: the synthetic-input builder sets it for the
    whole process, as the reference harness does (synthetic.py:218)."""
    monkeypatch.delenv("KERNEL_LAB_WGRAD_LAYOUT_MODE", raising=False)
    yield
