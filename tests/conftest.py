"""Shared fixtures.  `-m gpu` tests need a B200 and the built libmoe_b200.so;
everything else runs on the CPU."""
import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def load_package():
    """Import llm.c_b200/ (not a valid identifier) as module `moe_b200`."""
    if "moe_b200" in sys.modules:
        return sys.modules["moe_b200"]
    spec = importlib.util.spec_from_file_location(
        "moe_b200", os.path.join(ROOT, "llm.c_b200", "__init__.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules["moe_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and libmoe_b200.so")


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle
    oracle.lib()
    return oracle


@pytest.fixture(scope="session")
def moe_lib():
    """The CUDA library, initialised on device 0.  Fails loudly (no fallback)."""
    m = load_package()
    m.lib()
    m.init(0)
    return m


@pytest.fixture
def moe(moe_lib):
    """Per test: the weight registry is keyed by host address, and numpy
    reuses freed addresses, so every test starts from an empty registry."""
    moe_lib.reset(0)
    return moe_lib
