import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "contract-stablehlo-mlx_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running check")


def load_pins(flavour: str) -> dict:
    pins = {}
    with open(os.path.join(ROOT, "tests", "golden", "ref-%s.sha256" % flavour)) as f:
        for ln in f:
            h, p = ln.split()
            pins[p] = h
    return pins


@pytest.fixture(scope="session")
def pins():
    return {"pinned": load_pins("pinned"), "stock": load_pins("stock")}
