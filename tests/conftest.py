import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "hive-limited_b200"
for p in (str(PKG), str(REPO / "oracle"), str(REPO)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA kernels)")
    config.addinivalue_line("markers", "slow: long-running case")


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    cache = {}

    def load(name):
        if name not in cache:
            cache[name] = dict(np.load(GOLDEN / name, allow_pickle=False))
        return cache[name]
    return load


@pytest.fixture(scope="session")
def hv():
    """The native library, loaded once; GPU tests fail loudly when it cannot run."""
    import hvdrv
    hvdrv.init()
    return hvdrv
