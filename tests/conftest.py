"""Shared test setup: import paths, the `gpu` marker, device fixtures."""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "shannon-prime-llama_b200"
for p in (ROOT, PKG, ROOT / "oracle"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def load_build_module():
    """shannon-prime-llama_b200/build.py as a module."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("spb200_build", PKG / "build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")


@pytest.fixture(scope="session")
def built_lib():
    """The in-tree C-ABI library (built on demand)."""
    return load_build_module().build()


@pytest.fixture(scope="session")
def cuda(built_lib):
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test ran without a CUDA device")
    torch.cuda.init()
    return torch.device("cuda:0")
