import json
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (run on the GPU box)")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def _ensure_built():
    from oracle import oracle
    if not os.path.exists(os.path.join(ROOT, "oracle", "liboracle.so")):
        oracle.build()
    lib = os.path.join(ROOT, "barracuda_b200", "lib", "libbarracuda_fhe.so")
    if not os.path.exists(lib):
        from barracuda_b200 import build
        build.build()


_ensure_built()


@pytest.fixture(scope="session")
def kats():
    with open(os.path.join(ROOT, "tests", "golden", "reference_kats.json")) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def device():
    """The CUDA device for parity tests (product path only; fails loudly without it)."""
    from barracuda_b200 import Device
    d = Device(0)
    yield d
    d.close()
