"""The drop-in C ABI without a GPU: every declared symbol is exported, the model loader refuses malformed models
with a message instead of crashing (crates/flyhigh-engine/tests/models.rs), the synthetic model is the FlyHighFG
graph, and the calls that need a device fail cleanly where there is none."""
import ctypes
import json
import os
import re

import numpy as np
import pytest

import flyhigh_engine_b200 as fh

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in ("flyhigh.h", "flyhigh_b200.h", "flyhigh_kernels.h"):
        text = open(os.path.join(ROOT, "include", h)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"\b(fhk?_[a-z0-9_]+)\s*\(", text))
    return names


def test_every_declared_symbol_is_exported():
    lib = ctypes.CDLL(fh.library_path())
    names = declared_functions()
    assert len(names) > 35
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, missing
    # and the Python front binds every one of them
    assert names == {n for n, _, _ in fh.EXPORTS}


def _load(graph, manifest, weights):
    return fh.Model.from_bytes(json.dumps(graph).encode(), json.dumps(manifest).encode(), weights)


def _manifest(tensors):
    return {"meta": {"model": "t", "format_version": 1}, "tensors": tensors}


def test_well_formed_model_loads():
    graph = {"ops": [{"op": "conv", "in": ["a"], "out": ["b"], "w": ["w0", "b0"]}]}
    man = _manifest({"w0": {"shape": [2, 3], "offset": 0}, "b0": {"shape": [], "offset": 6}})
    m = _load(graph, man, b"\0" * 14)
    assert m.info()["tensors"] == 2 and m.info()["graph_ops"] == 1


@pytest.mark.parametrize("what,tensors,n", [
    ("non-integer dimension", {"w0": {"shape": [2, "3"], "offset": 0}}, 64),
    ("float dimension", {"w0": {"shape": [2, 1.5], "offset": 0}}, 64),
    ("zero dimension", {"w0": {"shape": [0], "offset": 32}}, 64),
    ("negative offset", {"w0": {"shape": [2], "offset": -4}}, 64),
    ("past the end", {"w0": {"shape": [2], "offset": 31}}, 64),
    ("overflowing shape", {"w0": {"shape": [18446744073709551615, 2], "offset": 0}}, 64),
    ("overflowing offset", {"w0": {"shape": [2], "offset": 18446744073709551615}}, 64),
])
def test_malformed_manifests_are_refused(what, tensors, n):
    graph = {"ops": [{"op": "conv", "in": ["a"], "out": ["b"], "w": ["w0"]}]}
    with pytest.raises(fh.FlyHighError, match="tensor w0"):
        _load(graph, _manifest(tensors), b"\0" * n)


@pytest.mark.parametrize("graph,msg", [
    ({"ops": []}, "no ops"),
    ({"nodes": []}, "no ops"),
    ({"ops": [{"in": ["a"]}]}, "has no name"),
    ({"ops": [{"op": "conv", "in": "a"}]}, "not a list"),
    ({"ops": [{"op": "conv", "in": [1]}]}, "non-string"),
    ({"ops": [{"op": "conv", "in": ["a"], "w": ["missing"]}]}, "lacks"),
    ({"ops": [{"op": "repeat"}]}, "without a body"),
    ({"ops": [{"op": "film_mlp", "in": ["t"]}]}, "film_mlp needs"),
])
def test_malformed_graphs_are_refused(graph, msg):
    with pytest.raises(fh.FlyHighError, match=msg):
        _load(graph, _manifest({"w0": {"shape": [2], "offset": 0}}), b"\0" * 8)


def test_bad_json_and_versions_are_refused():
    with pytest.raises(fh.FlyHighError, match="manifest"):
        fh.Model.from_bytes(b'{"ops": [{"op": "conv"}]}', b"\x00\xff not json", b"\0" * 8)
    with pytest.raises(fh.FlyHighError, match="no tensors"):
        _load({"ops": [{"op": "conv"}]}, {"tensors": []}, b"\0" * 8)
    man = _manifest({})
    man["meta"]["format_version"] = 2
    with pytest.raises(fh.FlyHighError, match="format_version"):
        _load({"ops": [{"op": "conv"}]}, man, b"")
    with pytest.raises(fh.FlyHighError, match="cannot open"):
        fh.Model("/nonexistent/model/dir")


def test_synthetic_model_is_the_flyhighfg_graph(synth_model_dir, reference_models):
    """The graph and tensor shapes written by flyhigh_engine_b200.synth_model equal the reference's own files."""
    from flyhigh_engine_b200 import synth_model
    ref_ops = json.load(open(os.path.join(reference_models, "graph.json")))["ops"]
    canon = lambda ops: [json.dumps(o, sort_keys=True) for o in ops]
    assert canon(synth_model.graph_ops()) == canon(ref_ops)
    ref_t = json.load(open(os.path.join(reference_models, "flyhighfg.json")))["tensors"]
    mine = synth_model.manifest(synth_model.tensor_shapes())["tensors"]
    assert list(mine) == list(ref_t)
    assert all(mine[k]["shape"] == ref_t[k]["shape"] and mine[k]["offset"] == ref_t[k]["offset"] for k in ref_t)
    assert fh.Model(synth_model_dir).fingerprint() == fh.Model(reference_models).fingerprint()
    info = fh.Model(reference_models).info()
    assert info == {"name": "FlyHighFG", "train_step": 110000, "graph_ops": 83, "tensors": 62,
                    "render_sampling": "bicubic", "format_version": 1}


def test_another_graph_is_refused_by_the_planner(synth_model_dir):
    g = json.load(open(os.path.join(synth_model_dir, "graph.json")))
    g["ops"][14]["k"] = 3  # a different avgpool
    m = fh.Model.from_bytes(json.dumps(g).encode(), open(os.path.join(synth_model_dir, "flyhighfg.json"), "rb").read(),
                            open(os.path.join(synth_model_dir, "flyhighfg.bin"), "rb").read())
    with pytest.raises(fh.FlyHighError, match="not the FlyHighFG v1 graph"):
        m.plan_params(640, 360)


def test_options_defaults_match_the_reference():
    """fh_session_options_default = SessionOptions::new (session.rs:118-135) as core.rs:165-168 converts it."""
    o = fh.lib().fh_session_options_default(1920, 1080)
    assert (o.width, o.height, o.internal_w, o.internal_h, o.k, o.repair, o.render) == (1920, 1080, 0, 0, 1, 1, 0)
    assert (o.keep_static, o.static_frames, o.static_tolerance) == (1, 8, 4)
    assert (o.fast_render, o.linear_t, o.keep_maps, o.protection_mask) == (0, 0, 0, 0)
    g = fh.lib().fh_options_default(1920, 1080)  # capi/src/lib.rs:100-120 over Options::new (api.rs:113-148)
    assert (g.width, g.height, g.k, g.internal_w, g.internal_h, g.mode, g.repair, g.cadence) == (1920, 1080, 1, 856, 480,
                                                                                               0, 1, 0)
    assert (g.render_sampling, g.keep_static, g.static_frames, g.static_tolerance, g.fast_render, g.linear_t) == \
        (0, 1, 8, 4, 0, 0)
    assert (fh.lib().fh_options_default(640, 360).internal_w, fh.lib().fh_options_default(640, 360).internal_h) == (0, 0)
    p = fh.lib().fh_pacer_options_default()  # pacer/mod.rs:198-231
    assert (p.mode, p.max_factor, p.limit_to_display, p.queue_capacity, p.penalty_max, p.motion_adaptive) == (0, 6, 1, 24,
                                                                                                            3, 1)
    assert (p.display_headroom, p.compute_budget, p.delay_floor_ms, p.delay_max_ms, p.settle_ms) == (0.97, 0.9, 60.0,
                                                                                                   180.0, 1200.0)
    assert fh.lib().fh_vk_row_pitch(1920) == 7680 and fh.lib().fh_vk_row_pitch(100) == 512
    assert fh.lib().fh_pacer_create(None) is None and b"not part of this library" in fh.lib().fh_last_error()
    e = fh.lib().fh_engine_options_default()
    assert (e.backend, e.tensor_cores, e.autotune, e.precision, e.compact_memory) == (0, 1, 1, 0, 1)


def test_no_device_is_a_clean_error():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    with pytest.raises(fh.FlyHighError, match="no CUDA device"):
        fh.Engine()
    assert fh.lib().fh_session_pair(None, 0, 1) == -1
    assert b"null" in fh.lib().fh_last_error()
