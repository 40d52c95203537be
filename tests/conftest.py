import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "onnx-light_b200")
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))


def load_package():
    """Imports the package directory onnx-light_b200/ as module onnx_light_b200."""
    if "onnx_light_b200" in sys.modules:
        return sys.modules["onnx_light_b200"]
    spec = importlib.util.spec_from_file_location(
        "onnx_light_b200", os.path.join(PKG_DIR, "__init__.py"), submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["onnx_light_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: large-size property tests")


@pytest.fixture(scope="session")
def b2():
    return load_package()


@pytest.fixture(scope="session")
def O():
    import oracle
    return oracle


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    return torch.device("cuda:0")


def pytest_sessionfinish(session, exitstatus):
    path = os.environ.get("ONNXL_RELERR_LOG")
    if not path:
        return
    import json
    import util
    with open(path, "w") as f:
        json.dump(util.RELERR_LOG, f)
