import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); runs the CUDA library")


@pytest.fixture(scope="session")
def synth_weights():
    from krikil_rs_b200 import synth
    return synth.make_weights(0)


@pytest.fixture(scope="session")
def synth_weights_perturbed():
    from krikil_rs_b200 import synth
    return synth.make_weights(0, perturb=True)
