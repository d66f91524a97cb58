"""The frame-parity classifier itself (CPU only): on the oracle's own render of perturbed network outputs it explains
every pixel beyond 2 levels, and it rejects planted mistakes (planted on the CPU, in the frames and maps it is given)."""
import numpy as np
import pytest

from tests.frame_parity import check_frame


@pytest.fixture(scope="module")
def oracle_pair(synth_model_dir):
    import flyhigh_engine_b200 as fh
    from flyhigh_engine_b200 import synth_frames
    from oracle.oracle import OracleModel, OracleSession
    W, H = 640, 360
    fr = synth_frames.sequence_c2(3, W, H, seed=3)
    o = OracleSession(OracleModel(synth_model_dir), W, H)
    o.pair(fr[0], fr[1])
    o.mid(0.5)
    o.pair(fr[1], fr[2])
    ref = o.mid(0.5)
    pp = fh.Model(synth_model_dir).plan_params(W, H)
    gm = o.gmhs_select(o.tensor("flow_pre"))
    return dict(W=W, H=H, fa=fr[1], fb=fr[2], ref=ref, pp=pp, up7=o.tensor("up7", 1), rt=o.tensor("R_t", 1),
                age=o.tensor("age"), gm=(gm, gm), flow_pre=o.tensor("flow_pre"))


def _render(d, up7):
    from oracle import oracle
    pp = d["pp"]
    return oracle.render_planes(d["fa"], d["fb"], d["W"], d["H"], up7, d["rt"], d["age"][0], pp["fsx"], pp["fsy"],
                                pp["min_age"], pp["static_thr"], cubic=bool(pp["cubic"]), flags=pp["render_flags"])


def _perturbed(d, ulps=2, seed=0):
    """The oracle's flow / visibility maps moved by up to `ulps` f16 ulps each (what another summation order does)."""
    rng = np.random.default_rng(seed)
    h = d["up7"].astype(np.float16)
    return (h.astype(np.float32) + rng.integers(-ulps, ulps + 1, h.shape) * np.spacing(np.abs(h)).astype(np.float32))


def _check(d, got, up7):
    return check_frame(got, d["ref"], d["fa"], d["fb"], d["W"], d["H"], d["pp"], (up7, d["rt"]), (d["up7"], d["rt"]),
                       d["age"], d["gm"])


def test_identical_maps_give_identical_frames(oracle_pair):
    d = oracle_pair
    rep = _check(d, _render(d, d["up7"]), d["up7"])
    assert rep["ok"] and rep["over"] == 0 and rep["render_gap"] == 0 and rep["max"] == 0, rep


def test_ulp_noise_is_explained(oracle_pair):
    d = oracle_pair
    up7 = _perturbed(d, 2)
    rep = _check(d, _render(d, up7), up7)
    assert rep["ok"], rep
    assert rep["over"] > 0 and rep["cats"]["unexplained"] == 0
    assert rep["max_pos_tol"] <= 1.0


def test_planted_pixel_error_is_rejected(oracle_pair):
    d = oracle_pair
    up7 = _perturbed(d, 1)
    got = _render(d, up7).reshape(d["H"], d["W"], 4).copy()
    got[100, 200, 1] = np.uint8((int(got[100, 200, 1]) + 40) % 256)
    rep = _check(d, got.reshape(-1), up7)
    assert not rep["ok"]
    assert rep["render_gap"] >= 40 - 1
    assert any(u["x"] == 200 and u["y"] == 100 for u in rep["unexplained"]), rep["unexplained"]


def test_planted_flow_error_is_rejected(oracle_pair):
    """Half a pixel of flow in a patch, with no repair decision behind it: far beyond a few ulps, unexplained."""
    d = oracle_pair
    up7 = d["up7"].copy()
    up7[0:4, 40:52, 60:80] += 0.5
    rep = _check(d, _render(d, up7), up7)
    assert not rep["ok"]
    assert rep["cats"]["unexplained"] > 0
    assert all(u["dtol"] > 1.0 for u in rep["unexplained"])


def _flipped_records(d, flow_shift):
    """The oracle's repair record twice: the second with one cell's decision flipped by a cost margin of 3e-3 (beyond
    GMHS_TOL) and its pre-repair flow moved by flow_shift px around that cell."""
    go = {k: np.array(v, copy=True) for k, v in d["gm"][0].items()}
    gg = {k: np.array(v, copy=True) for k, v in d["gm"][0].items()}
    i, j = 10, 20
    go["m_cost"][i, j], gg["m_cost"][i, j] = 0.003, -0.003
    gg["sel"][i, j] = 1.0 - go["sel"][i, j]
    go["flow"] = np.asarray(d["flow_pre"], np.float32)
    gg["flow"] = go["flow"].copy()
    gg["flow"][:, i - 2:i + 3, j - 2:j + 3] += flow_shift
    return go, gg


def test_repair_flip_within_flow_rounding_is_explained(oracle_pair):
    """A repair decision flipped away from its threshold is accepted when the two pre-repair flows agree within
    POS_ULPS f16 ulps around the cell (here 0.01 px), and rejected when they do not (0.3 px)."""
    d = oracle_pair
    frame = _render(d, d["up7"])
    up7 = d["up7"]
    ok = check_frame(frame, d["ref"], d["fa"], d["fb"], d["W"], d["H"], d["pp"], (up7, d["rt"]), (up7, d["rt"]),
                     d["age"], _flipped_records(d, 0.01))
    assert ok["ok"] and ok["gmhs_flipped"] == 1 and not ok["gmhs_not_adjacent"], ok
    assert ok["gmhs_margins"][0]["pre_flow_tol"] <= 1.0
    bad = check_frame(frame, d["ref"], d["fa"], d["fb"], d["W"], d["H"], d["pp"], (up7, d["rt"]), (up7, d["rt"]),
                      d["age"], _flipped_records(d, 0.3))
    assert not bad["ok"] and len(bad["gmhs_not_adjacent"]) == 1, bad
