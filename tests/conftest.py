"""Shared fixtures. GPU tests carry @pytest.mark.gpu; everything else runs on the CPU."""
import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "-damn-low-level-fence-inference-version-1_b200")
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def load_pkg():
    """The binding module of libfence_b200.so (its directory name is not a Python identifier)."""
    if "fence_b200" in sys.modules:
        return sys.modules["fence_b200"]
    spec = importlib.util.spec_from_file_location("fence_b200", os.path.join(PKG_DIR, "__init__.py"),
                                                  submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["fence_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


@pytest.fixture(scope="session")
def fb():
    return load_pkg()


@pytest.fixture(scope="session")
def orc():
    import oracle as o  # oracle/oracle.py
    return o


@pytest.fixture(scope="session")
def tmpdir_session(tmp_path_factory):
    return tmp_path_factory.mktemp("fence")


@pytest.fixture(autouse=True)
def _device_error_word(request):
    """After every GPU test: no kernel of the library gave up on a bounded wait (the device error
    word, read and cleared by fence_device_error, is 0). Tests that make a wait run out on purpose
    read and clear the word themselves."""
    yield
    if request.node.get_closest_marker("gpu") is None:
        return
    mod = sys.modules.get("fence_b200")
    if mod is None or mod._lib is None:
        return
    import torch
    if not torch.cuda.is_available():
        return
    for d in range(torch.cuda.device_count()):
        with torch.cuda.device(d):
            word = mod.lib().fence_device_error()
            assert word == 0, f"device {d}: device error word {word} after {request.node.nodeid}"
