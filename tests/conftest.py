"""Shared pytest configuration.

Tests marked ``gpu`` need a B200 and run with ``pytest -m gpu``; everything
else runs on a CPU-only machine (``pytest -m "not gpu"``).
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for path in (ROOT, os.path.join(ROOT, "tests")):
    if path not in sys.path:
        sys.path.insert(0, path)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def lib_built():
    """Build (or reuse) libask_b200.so; building needs only nvcc, no GPU."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("ask_b200_build", os.path.join(ROOT, "ask_b200", "build.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.build()
    return True


@pytest.fixture(scope="session")
def device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA; run GPU tests with -m gpu on a B200")
    torch.cuda.set_device(0)
    return 0
