import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    return np.load(os.path.join(ROOT, "tests", "golden", "reference_py.npz"))


@pytest.fixture(scope="session")
def gpt2_tensors():
    from llm_mojo_b200 import synth

    return synth.gpt2_random_init(0)


@pytest.fixture(scope="session")
def oracle_a16(gpt2_tensors):
    """The oracle's int4-g32-a16 model with an int8 head and QuantKV[8]."""
    from oracle import oracle as O

    return O.Model(gpt2_tensors)
