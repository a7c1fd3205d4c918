"""Shared fixtures.  Tests marked `gpu` need a CUDA device; everything else runs on CPU."""
import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TESTS = os.path.dirname(os.path.abspath(__file__))
for p in (ROOT, TESTS):
    if p not in sys.path:
        sys.path.insert(0, p)

PKG = "paged-kv-cache-manager_b200"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def load_pkg():
    """Imports the product package, building libkvpage_b200.so first if it is missing."""
    lib = os.path.join(ROOT, PKG, "libkvpage_b200.so")
    if not os.path.exists(lib):
        build = importlib.import_module(PKG + ".build_lib")
        build.build()
    return importlib.import_module(PKG)


@pytest.fixture(scope="session")
def kvb():
    return load_pkg()


@pytest.fixture(scope="session")
def ora():
    import oracle
    oracle.c_oracle()
    return oracle


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
