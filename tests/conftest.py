"""Test configuration: import paths, the `gpu` marker, the native build."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "ouroboros-triton_b200"
for p in (str(PKG), str(ROOT), str(ROOT / "tests" / "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the sm_100a kernels")


def pytest_sessionstart(session):
    # Build (or confirm up to date) the native library once per session.
    sys.path.insert(0, str(PKG))
    import build as native_build  # ouroboros-triton_b200/build.py

    try:
        native_build.build()
    except RuntimeError as exc:  # no nvcc: tests that need the library fail loudly later
        print(f"native build skipped: {exc}", file=sys.stderr)


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device")
    return torch.device("cuda", 0)
