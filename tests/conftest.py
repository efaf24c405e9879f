import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "imr-mlp_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "tests"))

GOLDEN = os.path.join(ROOT, "tests", "golden")
MODELS = os.path.join(GOLDEN, "models")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")
    config.addinivalue_line("markers", "slow: long-running")


@pytest.fixture(scope="session")
def oracle():
    from oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle import Reference
    if not Reference.available():
        pytest.skip("oracle/_ref/libref.so not built (reference checkout absent)")
    return Reference()


def load_model(name):
    from mtpb200 import read_mtp
    return read_mtp(os.path.join(MODELS, name))


@pytest.fixture(scope="session")
def model_l16():
    return load_model("l16_k2.mtp")


@pytest.fixture(scope="session")
def model_l20():
    return load_model("l20_k2.mtp")


@pytest.fixture(scope="session")
def model_l20_k3():
    return load_model("l20_k3.mtp")
