import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200; runs through libfoxcuda on the device")


@pytest.fixture(scope="session")
def tiny_model():
    from rustfox_b200 import synth
    return synth.generate(synth.CONFIGS["tiny"])


@pytest.fixture(scope="session")
def oracle_tiny(tiny_model):
    from oracle import oracle as O
    return O.OracleModel(tiny_model)


@pytest.fixture(scope="session")
def gpu_tiny(tiny_model):
    import rustfox_b200 as rf
    m = rf.Model.from_synthetic(tiny_model)
    yield m
    m.close()


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
