import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the C-ABI kernels")
    config.addinivalue_line("markers", "slow: full-size model parity (minutes)")


@pytest.fixture(scope="session")
def e4b():
    import __graft_entry__
    __graft_entry__.build()
    return importlib.import_module("e4b-webgpu_b200")


@pytest.fixture(scope="session")
def dev(e4b):
    """Device with a workspace attached, so GEMVs take the streaming tensor-core path."""
    import ctypes
    d = e4b.Device(0)
    ws = int(d.L.e4b_workspace_bytes())
    buf = d.alloc(ws, "workspace")
    d.call("e4b_set_workspace", buf.ptr, ctypes.c_size_t(ws))
    yield d
    d.close()


@pytest.fixture(scope="session")
def models(e4b):
    """Synthetic GGUF images of the small configs, built once per session."""
    cache = {}

    def get(name):
        if name not in cache:
            cache[name] = e4b.synth.build_model(e4b.config.get(name))
        return cache[name]
    return get
