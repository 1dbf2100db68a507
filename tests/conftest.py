"""Shared test set-up.

Markers: `gpu` tests need a CUDA device and run the product library through
its C ABI; everything else runs on the CPU (oracle, host logic, library
loading, gloo multi-process paths).
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(REPO / "oracle"))
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "tests"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    import oracle as O  # noqa: E402  (oracle/oracle.py, test infrastructure)

    O.lib()
    return O


@pytest.fixture(scope="session")
def uv():
    """The product package, loaded from the in-tree build."""
    import uvb200_loader

    return uvb200_loader.load()
