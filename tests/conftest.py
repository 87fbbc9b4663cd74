"""Shared pytest setup: the `gpu` marker, the in-tree build, common helpers."""
from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "multigpu: needs two or more GPUs on one node")


@pytest.fixture(scope="session", autouse=True)
def _built():
    """Builds (or confirms up to date) every native library the tests load."""
    from megacu_b200 import build
    build.build_all()
    yield


def gpu_count() -> int:
    try:
        import torch
        return torch.cuda.device_count() if torch.cuda.is_available() else 0
    except Exception:
        return 0
