import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA path through the C ABI)")
    config.addinivalue_line("markers", "slow: takes tens of seconds on the CPU")


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    cache = {}

    def load(name):
        if name not in cache:
            cache[name] = np.load(os.path.join(GOLDEN, name + ".npz"))
        return cache[name]
    return load


@pytest.fixture(scope="session")
def synth_model_path(tmp_path_factory):
    """the seeded random-init POISD model of seed 1 (written once per session by the library's writer)"""
    import vela_b200 as V
    path = str(tmp_path_factory.mktemp("model") / "synth_seed1.poisd")
    V.synth_model_write(path, 1)
    return path
