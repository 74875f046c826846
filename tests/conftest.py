import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
PKG_DIR = os.path.join(ROOT, "rdna4-gemm-wmma_b200")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a) GPU")


def load_b2g():
    """Import the package's ctypes binding (the package directory name has hyphens)."""
    if "b2g" in sys.modules:
        return sys.modules["b2g"]
    spec = importlib.util.spec_from_file_location("b2g", os.path.join(PKG_DIR, "b2g.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules["b2g"] = mod
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="session")
def b2g():
    mod = load_b2g()
    mod.load()
    return mod


@pytest.fixture(scope="session")
def orc():
    from oracle import orc as o
    o.lib()
    return o


@pytest.fixture(scope="session")
def cuda(b2g):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()
    return torch
