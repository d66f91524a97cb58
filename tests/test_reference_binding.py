"""The reference's own Python binding (bindings/python/flyhigh.py of a reference checkout, imported unchanged where one
is present; never on the GPU hosts) against this libflyhigh.so: every function it binds at load time resolves, the
option defaults it reads come back as the reference's, and without a device its Engine and its Pacer fail with this
library's messages instead of crashing. The Session / Stream steps of its test_flyhigh.py run on the GPU through this
package's binding (tests/test_gpu_stream.py::test_reference_binding_call_sequence); the Pacer is not part of this library."""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "flyhigh_engine_b200", "libflyhigh.so")

SCRIPT = r"""
import sys
sys.path.insert(0, sys.argv[1])
import flyhigh
lib = flyhigh._load()
print("loaded", flyhigh.library_path())
o = lib.fh_session_options_default(1920, 1080)
print("session", o.width, o.height, o.k, o.repair, o.keep_static, o.static_frames, o.static_tolerance)
p = lib.fh_pacer_options_default()
print("pacer", p.max_factor, p.display_headroom, p.delay_floor_ms, p.queue_capacity, p.settle_ms, p.gpu_timestamps)
try:
    flyhigh.Engine()
except flyhigh.FlyHighError as e:
    print("engine:", e)
try:
    flyhigh.Pacer("auto", min_present_interval_ms=0)
except flyhigh.FlyHighError as e:
    print("pacer:", e)
"""


def test_reference_binding_loads_unchanged(reference_repo):
    if not os.path.exists(LIB):
        pytest.skip("libflyhigh.so is not built")
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present: this checks the load without one")
    binding = os.path.join(reference_repo, "bindings", "python")
    env = dict(os.environ, FLYHIGH_LIB=LIB)
    r = subprocess.run([sys.executable, "-c", SCRIPT, binding], env=env, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, (r.stdout, r.stderr)
    lines = r.stdout.splitlines()
    assert lines[0] == f"loaded {LIB}"
    assert lines[1] == "session 1920 1080 1 1 1 8 4"
    assert lines[2] == "pacer 6 0.97 60.0 24 1200.0 1"
    assert lines[3].startswith("engine: ") and "no CUDA device" in lines[3]
    assert lines[4].startswith("pacer: ") and "not part of this library" in lines[4]
