"""The conv autotuner (ops/conv/autotune.rs:74-150 conv_pick, ops/conv/tune_cache.rs): when a session is built, each
conv shape (cin, cout, h, w, stride) not chosen before on the device is timed over its candidate kernels (mma.sync at
1, 2 and 4 rows per CTA pair, tcgen05 and its persistent variant where they fit) and the fastest kept; FhEngineOptions.tune_cache persists the
choices per GPU and driver, FhSessionOptions.tune imposes a table, autotune = 0 keeps the fixed rule. Every other GPU
test runs on autotuned sessions (the default) against the oracle."""
import os
import subprocess
import sys

import numpy as np
import pytest

from tests.parity import LAYER_REL_L2, rel_l2

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


# a size no other test builds, so that its shapes are new to this process's table
W, H = 704, 416

_CHILD = r"""
import sys, json
sys.path.insert(0, sys.argv[1])
import numpy as np
import flyhigh_engine_b200 as fh
from flyhigh_engine_b200 import synth_frames
e = fh.Engine(tune_cache=sys.argv[3])
s = fh.Session(e, fh.Model(sys.argv[2]), %d, %d)
fa, fb, _ = synth_frames.pair_c0(%d, %d, seed=5)
a, b, o = s.add_input(), s.add_input(), s.add_output()
s.write(a, fa); s.write(b, fb); s.pair(a, b); s.mid(0.5, o)
np.save(sys.argv[4], np.frombuffer(s.read(o), np.uint8))
print(json.dumps({"session": s.report(), "engine": e.report()}))
""" % (W, H, W, H)


def _child(model_dir, cache, out):
    r = subprocess.run([sys.executable, "-c", _CHILD, ROOT, model_dir, str(cache), str(out)], capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    import json
    return json.loads(r.stdout.strip().splitlines()[-1])


def test_tune_cache_persists_and_reloads(synth_model_dir, cuda, tmp_path):
    """A fresh process times every new shape and writes the device's file; a second fresh process reads the same
    choices from it (no timing) and renders the same bytes."""
    cache = tmp_path / "tune"
    cache.mkdir()
    first = _child(synth_model_dir, cache, tmp_path / "a.npy")
    convs = first["session"]["convs"]
    # each distinct shape is timed once; the session's further layers of that shape take the fresh entry
    assert first["session"]["autotuned"] > 0, convs
    assert all(c["choice"] in ("tuned", "table") for c in convs.values()), convs
    assert sum(c["choice"] == "tuned" for c in convs.values()) == first["session"]["autotuned"]
    assert first["engine"]["autotune_entries"] >= first["session"]["autotuned"]
    files = os.listdir(cache)
    assert len(files) == 1 and files[0].startswith("tune-10de-") and files[0].endswith("-f16-tc-b200.txt"), files
    lines = open(cache / files[0]).read().splitlines()
    assert len(lines) == first["engine"]["autotune_entries"] and lines == sorted(lines)
    for ln in lines:
        key, val = ln.split("=")
        assert len(key.split(",")) == 5 and int(val) in (0x11, 0x21, 0x41, 0x02, 0x12), ln
    second = _child(synth_model_dir, cache, tmp_path / "b.npy")
    assert second["session"]["autotuned"] == 0
    assert all(c["choice"] == "table" for c in second["session"]["convs"].values())
    assert {k: c["kernel"] for k, c in convs.items()} == {k: c["kernel"] for k, c in second["session"]["convs"].items()}
    assert np.array_equal(np.load(tmp_path / "a.npy"), np.load(tmp_path / "b.npy"))


@pytest.mark.parametrize("cand,kernel", [(0x11, "mma.sync/wm1"), (0x41, "mma.sync/wm4"), (0x02, "tcgen05")])
def test_session_tune_text_imposes_the_kernel(synth_model_dir, cuda, cand, kernel):
    """FhSessionOptions.tune names a kernel for every conv shape of the session: each layer runs it (tcgen05 only where
    it fits: stride 1, coarse.c1's 279-channel slice through its streamed-weights variant; the rest keep the fixed
    rule), and the layers stay within 1e-2 of the oracle."""
    import flyhigh_engine_b200 as fh
    from flyhigh_engine_b200 import synth_frames
    from oracle.oracle import OracleModel, OracleSession
    w, h = 640, 360
    model = fh.Model(synth_model_dir)
    p = model.plan_params(w, h)
    geo = {"e1": (p["qh"], p["qw"], 2), "e2": (p["h8"], p["w8"], 1), "e3": (p["h8"], p["w8"], 2),
           "e4": (p["h16"], p["w16"], 1)}
    shapes = {("enc.e1", 3, 36), ("enc.e2", 36, 36), ("enc.e3", 36, 72), ("enc.e4", 72, 72)}
    lines = [f"{ci},{co},{geo[n[4:]][0]},{geo[n[4:]][1]},{geo[n[4:]][2]}={cand}" for n, ci, co in shapes]
    for ci, co in ((279, 96), (96, 96), (96, 12)):
        lines.append(f"{ci},{co},{p['h16']},{p['w16']},1={cand}")
    for ci, co in ((155, 48), (48, 48), (48, 7), (48, 36), (48, 5)):
        lines.append(f"{ci},{co},{p['h8']},{p['w8']},1={cand}")
    for ci, co in ((14, 24), (24, 24), (24, 3)):
        lines.append(f"{ci},{co},{p['qh']},{p['qw']},1={cand}")
    s = fh.Session(fh.Engine(), model, w, h, tune="\n".join(lines))
    convs = s.report()["convs"]
    for name, c in convs.items():
        strided = name in ("enc.e1", "enc.e3")
        if kernel == "tcgen05" and strided:
            assert c["choice"] == "fixed", (name, c)  # tcgen05 does not take stride 2
        else:
            assert c == {"kernel": kernel, "choice": "session"}, (name, c)
    fa, fb, _ = synth_frames.pair_c0(w, h, seed=9)
    a, b, out = s.add_input(), s.add_input(), s.add_output()
    s.write(a, fa)
    s.write(b, fb)
    s.pair(a, b)
    s.mid(0.5, out)
    o = OracleSession(OracleModel(synth_model_dir), w, h)
    o.pair(fa, fb)
    o.mid(0.5)
    for n, stage in (("f16a", 0), ("o", 0), ("fr3", 0), ("up7", 1), ("R_t", 1)):
        assert rel_l2(s.tensor(n), o.tensor(n, stage)) <= LAYER_REL_L2, n


def test_autotune_off_keeps_the_fixed_rule(synth_model_dir, cuda):
    import flyhigh_engine_b200 as fh
    s = fh.Session(fh.Engine(autotune=False), fh.Model(synth_model_dir), 320, 192)
    assert s.report()["autotuned"] == 0
    assert all(c == {"kernel": "mma.sync", "choice": "fixed"} for c in s.report()["convs"].values())
    sb = fh.Session(fh.Engine(autotune=False), fh.Model(synth_model_dir), 320, 192, batch=4)
    kinds = {c["kernel"] for c in sb.report()["convs"].values()}
    assert kinds == {"mma.sync", "tcgen05"}  # batched: tcgen05 where it fits, mma.sync for the rest
