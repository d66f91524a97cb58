import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

def reference_checkout():
    """A checkout of the reference repository: the directory FLYHIGH_REFERENCE names, else one named `reference` beside
    this repository; None where there is none (it is never on the GPU hosts)."""
    for d in (os.environ.get("FLYHIGH_REFERENCE"), os.path.join(os.path.dirname(ROOT), "reference")):
        if d and os.path.isdir(os.path.join(d, "crates")):
            return d
    return None


# The reference's shipped model directory (graph.json, flyhighfg.json, flyhighfg.bin; CC BY-NC, never committed): the
# directory FLYHIGH_MODELS names, else tests/_models (a local, git-ignored copy that travels with the working tree),
# else the checkout's models/. Tests that need it skip where none is present.
def _reference_models_dir():
    ref = reference_checkout()
    cands = [os.environ.get("FLYHIGH_MODELS"), os.path.join(ROOT, "tests", "_models"),
             os.path.join(ref, "models") if ref else None]
    for d in cands:
        if d and os.path.exists(os.path.join(d, "flyhighfg.bin")):
            return d
    return None


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
    """The reference's shipped model directory, where this machine has a copy."""
    d = _reference_models_dir()
    if d is None:
        pytest.skip("no copy of the reference's model directory (FLYHIGH_MODELS, tests/_models)")
    return d


@pytest.fixture(scope="session")
def oracle_lib():
    from oracle import oracle
    return oracle.lib()


@pytest.fixture(scope="session")
def reference_repo():
    d = reference_checkout()
    if d is None:
        pytest.skip("no checkout of the reference repository (FLYHIGH_REFERENCE)")
    return d
