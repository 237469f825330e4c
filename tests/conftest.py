import importlib.util
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "comfyui-int8-fast-rocm_b200")
PKG_NAME = "comfyui_int8_fast_rocm_b200"
for p in (ROOT, os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (sm_100a B200)")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def load_package():
    """Import the node-pack directory (its name has dashes, as ComfyUI custom
    node folders do) as a regular package."""
    if PKG_NAME in sys.modules:
        return sys.modules[PKG_NAME]
    spec = importlib.util.spec_from_file_location(
        PKG_NAME, os.path.join(PKG_DIR, "__init__.py"), submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[PKG_NAME] = mod
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="session")
def pkg():
    return load_package()


@pytest.fixture(scope="session")
def golden():
    return np.load(os.path.join(ROOT, "tests", "golden", "golden.npz"))


@pytest.fixture(scope="session")
def golden_c1():
    return np.load(os.path.join(ROOT, "tests", "golden", "golden_c1.npz"))


def cuda_ok():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False
