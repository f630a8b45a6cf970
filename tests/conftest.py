"""Test configuration.

Markers: ``gpu`` tests need a B200 and run through the C ABI of
libvortexrt_b200.so; everything else runs on CPU (oracle, fixtures, host
logic, library exports).
"""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("vortex-rt_b200", "oracle"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 device (sm_100a)")


@pytest.fixture(scope="session")
def model_dir(tmp_path_factory):
    d = os.environ.get("VRT_MODEL_CACHE")
    if d:
        os.makedirs(d, exist_ok=True)
        return d
    return str(tmp_path_factory.mktemp("models"))


@pytest.fixture(scope="session")
def ctx():
    import vrt
    c = vrt.Context(0)
    yield c
    c.close()
