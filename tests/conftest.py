"""Shared test setup.

Markers: ``gpu`` tests need a CUDA device and run the CUDA library; the rest
run on the CPU (oracle pinning, host logic, the C ABI's argument checks and
symbol table, gloo multi-process tests).
"""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device; runs the sm_100a kernels")


@pytest.fixture(scope="session", autouse=True)
def _checkers_built():
    """Builds the C oracle if it is missing (it normally ships prebuilt)."""
    lib = ROOT / "oracle" / "_build" / "liboracle.so"
    if not lib.exists():
        subprocess.run(["make", "-C", str(ROOT / "oracle")], check=True, capture_output=True)
    yield


@pytest.fixture(scope="session")
def cuda_lib():
    """The CUDA library (built if missing).  Only for gpu tests."""
    from verbo_b200 import build, load_library

    build.build()
    return load_library()
