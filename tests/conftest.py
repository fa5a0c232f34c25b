import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "ornith-flight_b200")
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs through the C ABI")


def load_ofb():
    """The package's Python binding (directory name is not importable as-is)."""
    if "ornith_flight_b200.ofb" in sys.modules:
        return sys.modules["ornith_flight_b200.ofb"]
    spec = importlib.util.spec_from_file_location("ornith_flight_b200.ofb", os.path.join(PKG_DIR, "ofb.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules["ornith_flight_b200.ofb"] = mod
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="session")
def ofb():
    return load_ofb()


def load_ep():
    """The expert-parallel host module (ornith-flight_b200/ep.py)."""
    load_ofb()
    if "ornith_flight_b200.ep" in sys.modules:
        return sys.modules["ornith_flight_b200.ep"]
    spec = importlib.util.spec_from_file_location("ornith_flight_b200.ep", os.path.join(PKG_DIR, "ep.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules["ornith_flight_b200.ep"] = mod
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="session")
def oracle():
    import binding
    binding.orc()
    return binding


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
