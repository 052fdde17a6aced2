"""Test configuration: package path, the `gpu` marker, shared fixtures."""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "pallas-unbound_b200"
for p in (str(ROOT), str(PKG), str(Path(__file__).resolve().parent)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (runs the CUDA kernels)")
    config.addinivalue_line("markers", "stress: large-shape test (the reference's stress marker)")


def load_build_module():
    spec = importlib.util.spec_from_file_location("pu_build", PKG / "build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="session")
def built_lib():
    """Path of libpu_attn.so, building it (nvcc) if it is missing or stale."""
    return load_build_module().build()
