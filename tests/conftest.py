import importlib
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)
GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built CUDA library")


def pkg():
    """The product package (its directory name carries hyphens, so it is
    imported through importlib)."""
    return importlib.import_module("gpt-oss-tvm_b200")


def synth():
    return importlib.import_module("gpt-oss-tvm_b200.synthetic")


def golden(name):
    path = os.path.join(GOLDEN, name)
    if not os.path.exists(path):
        pytest.skip(f"golden fixture {name} missing")
    return np.load(path)


@pytest.fixture(scope="session")
def oracle():
    import oracle as orc
    orc.build()
    return orc
