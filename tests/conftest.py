import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

REFERENCE_MODELS = "/root/reference/models"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA library)")


@pytest.fixture(scope="session")
def synth_model_dir(tmp_path_factory):
    """A FlyHighFG model directory with seeded N(0, 0.05) weights (the shipped weights are not redistributed)."""
    from flyhigh_engine_b200 import synth_model
    d = tmp_path_factory.mktemp("model")
    return synth_model.write(str(d), seed=0)


@pytest.fixture(scope="session")
def reference_models():
    """The reference's shipped model directory, where this machine has it (never on the GPU hosts)."""
    if not os.path.exists(os.path.join(REFERENCE_MODELS, "flyhighfg.bin")):
        pytest.skip("the reference model directory is not on this machine")
    return REFERENCE_MODELS


@pytest.fixture(scope="session")
def oracle_lib():
    from oracle import oracle
    return oracle.lib()
