"""The planner against the reference's golden plan dumps (CPU only).

tests/golden/plan_params.json holds the parameter words of the reference's own golden plans
(crates/flyhigh-engine/tests/golden/<config>.tc-f16.txt, extracted by tests/golden/make_plan_params.py). Every size,
window radius, threshold and render word that this build's planner derives (fh_session_plan_params, no GPU needed)
and that the CPU oracle derives must equal them, and the conv layers the FlyHighFG graph runs must be exactly the
reference plan's conv dispatches.
"""
import json
import os
from collections import Counter

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = json.load(open(os.path.join(HERE, "golden", "plan_params.json")))


def _opts(rec):
    o = dict(k=rec["k"], repair=rec["repair"], static_protection=False)
    iw, ih = rec["internal"]
    if (iw, ih) == (rec["width"], rec["height"]):
        o["internal"] = "frame"
    return o


@pytest.fixture(scope="module")
def model(synth_model_dir):
    import flyhigh_engine_b200 as fh
    return fh.Model(synth_model_dir)


def expected_convs(p, k):
    """(cin, h, w, hout, wout, stride, cout) of every conv of one pair + one mid of the FlyHighFG graph."""
    q, e8, e16 = (p["qh"], p["qw"]), (p["h8"], p["w8"]), (p["h16"], p["w16"])
    enc = [(3, *q, *e8, 2, 36), (36, *e8, *e8, 1, 36), (36, *e8, *e16, 2, 72), (72, *e16, *e16, 1, 72)] * 2
    coarse = [(279, *e16, *e16, 1, 96)] + [(96, *e16, *e16, 1, 96)] * 3 + [(96, *e16, *e16, 1, 12)]
    fine = [(155, *e8, *e8, 1, 48), (48, *e8, *e8, 1, 48), (48, *e8, *e8, 1, 48), (48, *e8, *e8, 1, 7)] * k
    mid = [(48, *e8, *e8, 1, 48)] * 2 + [(48, *e8, *e8, 1, 5), (48, *e8, *e8, 1, 36)]
    refine = [(14, *q, *q, 1, 24), (24, *q, *q, 1, 24), (24, *q, *q, 1, 24), (24, *q, *q, 1, 3)]
    return enc + coarse + fine + mid + refine


@pytest.mark.parametrize("rec", GOLDEN, ids=[r["config"] for r in GOLDEN])
def test_planner_matches_golden_plan(model, rec, monkeypatch):
    monkeypatch.setenv("FH_STILL", "0")  # the golden plans are built with NetOpts::new: no still test
    p = model.plan_params(rec["width"], rec["height"], **_opts(rec))
    r = rec["render"]
    assert (p["hp"], p["wp"]) == (r["H"], r["W"]) or not p["internal"]
    assert (p["qh"], p["qw"]) == (r["hq"], r["wq"])
    assert p["fsx"] == pytest.approx(r["fsx"], abs=0) and p["fsy"] == pytest.approx(r["fsy"], abs=0)
    assert p["cubic"] == r["cubic"] and p["render_flags"] == r["flags"]
    sads = {s["radius"]: (s["h"], s["w"]) for s in rec["sads"]}
    assert sads[3] == (p["h16"], p["w16"]) and sads[2] == (p["h8"], p["w8"])
    if rec["repair"] > 0:
        g = rec["gm"]
        assert (g["h"], g["w"]) == (p["NH"], p["NW"]) and (g["hc"], g["wc"]) == (p["hc"], p["wc"])
        assert (g["h8"], g["w8"]) == (p["h8"], p["w8"])
        assert g["radii"] == [p["r_blk"], p["r_dwin"]]
        assert np.float32(g["dmin"]) == np.float32(p["dmin"]) and np.float32(g["delta"]) == np.float32(p["delta"])
    # the network input: the internal downscale when the network runs below the frame size
    aa = [i for i in rec["interps"] if i["aa"] == 1]
    if p["internal"]:
        assert (aa[0]["ih"], aa[0]["iw"], aa[0]["oh"], aa[0]["ow"]) == (p["hp"], p["wp"], p["NH"], p["NW"])
    assert (aa[-1]["oh"], aa[-1]["ow"]) == (p["qh"], p["qw"])
    got = Counter(expected_convs(p, rec["k"]))
    ref = Counter((c["cin"], c["h"], c["w"], c["hout"], c["wout"], c["stride"], c["cout"]) for c in rec["convs"])
    assert got == ref
    # the fine warps read the flow at 1/8 (its E8 view) and the refine warps at 1/4
    assert {w["fs"] for w in rec["warps"] if w["stage"] == "pair"} == {0.125}
    assert {w["fs"] for w in rec["warps"] if w["stage"] == "mid"} == {0.25}


@pytest.mark.parametrize("rec", GOLDEN, ids=[r["config"] for r in GOLDEN])
def test_oracle_matches_golden_plan(synth_model_dir, rec):
    from oracle.oracle import OracleModel, OracleSession
    iw, ih = rec["internal"]
    internal = (iw, ih) if (iw, ih) != (rec["width"], rec["height"]) else (rec["width"], rec["height"])
    o = OracleSession(OracleModel(synth_model_dir), rec["width"], rec["height"], internal=internal, k=rec["k"],
                      repair=max(rec["repair"], 1), keep_static=False, still=False)
    d = o.dims()
    r = rec["render"]
    if d["internal"]:
        assert (d["hp"], d["wp"]) == (r["H"], r["W"])
        assert np.float32(d["fsx"]) == np.float32(r["fsx"]) and np.float32(d["fsy"]) == np.float32(r["fsy"])
    if rec["repair"] > 0:
        g = rec["gm"]
        assert [d["r_blk"], d["r_dwin"]] == g["radii"] and (d["hc"], d["wc"]) == (g["hc"], g["wc"])
        assert np.float32(d["delta"]) == np.float32(g["delta"])
        if rec["repair"] == 1:
            assert np.float32(d["dmin"]) == np.float32(g["dmin"])


def test_plan_validation(model):
    """SessionOptions::validate (session.rs:170-197): out-of-range options are refused with the field's name."""
    import flyhigh_engine_b200 as fh
    for kw, msg in [(dict(k=4), "k"), (dict(repair=3), "repair"), (dict(linear_t=True), "linear_t"),
                    (dict(static_protection={"frames": 300}), "static_protection"),
                    (dict(static_protection={"frames": 8, "tolerance": 256}), "static_protection")]:
        with pytest.raises(fh.FlyHighError, match=msg):
            model.plan_params(640, 360, **kw)
    with pytest.raises(fh.FlyHighError, match="64x64"):
        model.plan_params(32, 360)
    with pytest.raises(fh.FlyHighError, match="32x32"):
        model.plan_params(640, 360, internal=(16, 16))
    # the automatic internal size: the frame up to 960 px, above that the 480-line rung (options.rs:348-356)
    assert (model.plan_params(1920, 1080)["NW"], model.plan_params(1920, 1080)["NH"]) == (864, 480)
    assert model.plan_params(960, 540)["internal"] == 0
    assert model.plan_params(3840, 2160)["NH"] == 480
