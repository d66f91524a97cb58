"""The Stream layer on the GPU (fh_stream_*, crates/flyhigh-engine/src/stream/ and crates/flyhigh-capi/src/stream.rs):
its pair classifier against the oracle's restatement of classify.wgsl and classify.rs, its frames against a plain
session's, video mode's one frame of lookahead, and the call sequence of the reference's own binding test
(bindings/python/test_flyhigh.py's Stream part)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _scene_frames(w, h, scenes, n, seed=40):
    from flyhigh_engine_b200 import synth_frames
    return [synth_frames.sequence_c2(n, w, h, seed=seed + k, hud=False) for k in range(scenes)]


def _c4_frames(w, h, n=64, cut_every=16, hold_every=10, offset=0):
    from flyhigh_engine_b200 import synth_frames
    order = synth_frames.stream_c4(n, cut_every, hold_every, scenes=3, offset=offset)
    pool = _scene_frames(w, h, 3, cut_every)
    return [pool[sc][j] for sc, j in order]


def test_classify_matches_oracle(synth_model_dir, cuda):
    """Every pair of a config-4-like sequence (cuts, 2-frame holds, a flash): the kind, mean, max and black the GPU
    reports equal the oracle's (classify.wgsl's sums restated on the CPU, classify.rs's decisions with their history)."""
    import flyhigh_engine_b200 as fh
    from oracle import oracle
    w, h = 320, 180
    frames = _c4_frames(w, h)
    flash = frames[20].copy()
    flash[..., :3] = np.clip(frames[20][..., :3].astype(np.int32) + 48, 0, 255).astype(np.uint8)
    frames[21] = flash
    eng = fh.Engine()
    st = fh.Stream(eng, fh.Model(synth_model_dir), w, h, held_frames=True)
    cl = oracle.Classifier(held_frames=True)
    kinds = []
    prev = None
    for i, f in enumerate(frames):
        slot = st.next_input([] if prev is None else [prev])
        st.write(slot, f)
        if prev is not None:
            c = st.classify(prev, slot)
            ref = cl.decide(oracle.classify_stats(frames[i - 1], f, w, h))
            assert (c.kind, c.mean, c.max, c.black) == (ref["kind"], ref["mean"], ref["max"], ref["black"]), (i, c, ref)
            assert c.motion == pytest.approx(ref["motion"], rel=1e-12)
            kinds.append(c.kind)
        st.push(slot, i * 1000.0 / 24.0)
        prev = slot
    assert {"motion", "cut", "hold"} <= set(kinds), kinds
    assert kinds[20] == "cut"  # the flash: a coherent brightness step
    assert st.report()["counters"]["classified"] == len(frames) - 1


def test_stream_frames_equal_session_frames(synth_model_dir, cuda):
    """Realtime: each push runs the pair (previous, newest) and generate(t) renders its phase t; the frames are the same
    bytes a session gives for the same pairs and phases, static protection included."""
    import flyhigh_engine_b200 as fh
    from flyhigh_engine_b200 import synth_frames
    w, h = 384, 192
    frames = synth_frames.sequence_c2(6, w, h, seed=9)
    model = fh.Model(synth_model_dir)
    st = fh.Stream(fh.Engine(), model, w, h, scene_cut=0)
    s = fh.Session(fh.Engine(), model, w, h)
    a, b, out = s.add_input(), s.add_input(), s.add_output()
    s.write(a, frames[0])
    prev = None
    for i, f in enumerate(frames):
        slot = st.next_input([] if prev is None else [prev])
        st.write(slot, f)
        p = st.push(slot, float(i))
        if i == 0:
            assert not p.ready
        else:
            assert p.ready and p.base_slot == prev and (p.start_pts, p.end_pts) == (i - 1.0, float(i))
            s.write(b if i % 2 else a, f)
            s.pair(a if i % 2 else b, b if i % 2 else a)
            for t in (0.25, 0.75):
                assert st.generate(t, 1)
                s.mid(t, out)
                assert st.read(1) == s.read(out), (i, t)
        prev = slot
    assert not st.generate(0.0, 0), "t = 0: the source frame is enough"
    rep = st.report()["counters"]
    assert (rep["pushes"], rep["pairs"], rep["mids"], rep["source_enough"]) == (6, 5, 10, 1)


def test_video_mode_has_one_frame_of_lookahead(synth_model_dir, cuda):
    """Video mode: the first interval is ready after the third push and starts two frames back; its frames equal the
    realtime stream's for the same interval."""
    import flyhigh_engine_b200 as fh
    from flyhigh_engine_b200 import synth_frames
    w, h = 320, 192
    frames = synth_frames.sequence_c2(5, w, h, seed=12)
    model = fh.Model(synth_model_dir)
    rt = fh.Stream(fh.Engine(), model, w, h)
    vd = fh.Stream(fh.Engine(), model, w, h, mode="video")
    got_rt, got_vd = {}, {}
    for i, f in enumerate(frames):
        for st, got in ((rt, got_rt), (vd, got_vd)):
            slot = i % 4
            st.write(slot, f)
            p = st.push(slot, 10.0 * i)
            if st is vd:
                assert p.ready == (i >= 2), i
                if p.ready:
                    assert (p.base_slot, p.start_pts, p.end_pts) == ((i - 2) % 4, 10.0 * (i - 2), 10.0 * (i - 1))
            if p.ready:
                assert st.generate(0.5, 0)
                got[p.start_pts] = st.read(0)
    assert set(got_vd) == {0.0, 10.0, 20.0}
    for k, v in got_vd.items():
        assert v == got_rt[k], k


def test_reference_binding_call_sequence(synth_model_dir, cuda):
    """bindings/python/test_flyhigh.py's Stream part, call for call: the warm-up push, a classified motion pair, the
    interval's slots and timestamps, phase 0 left to the source frame, no camera warp."""
    import flyhigh_engine_b200 as fh
    from flyhigh_engine_b200.synth_frames import sinusoid_pair
    W, H = 256, 192
    with fh.Engine() as engine, fh.Model(synth_model_dir) as model:
        with fh.Stream(engine, model, W, H) as st:
            s0 = st.next_input()
            st.write(s0, sinusoid_pair(W, H, 0.0))
            assert not st.push(s0, 0.0).ready
            s1 = st.next_input([s0])
            st.write(s1, sinusoid_pair(W, H, 2.0))
            c = st.classify(s0, s1)
            assert c is not None and c.kind == "motion"
            p = st.push(s1, 41.7)
            assert p.ready and p.base_slot == s0 and p.end_pts == 41.7, p
            assert not st.generate(0.0, 0), "the source frame is enough at t 0"
            assert st.generate(0.5, 0)
            assert not st.warp(0, 0, 42.0, output=True), "no camera warp before any mouse input"
            st.mouse(42.0, 5.0, 0.0)
            st.set_mouse_captured(True)
            assert not st.warp(0, 0, 43.0, output=True)
            assert st.report()["camera_warp"]["on"] is False


def test_stream_errors(synth_model_dir, cuda):
    import flyhigh_engine_b200 as fh
    eng, model = fh.Engine(), fh.Model(synth_model_dir)
    with pytest.raises(fh.FlyHighError, match="cadence"):
        fh.Stream(eng, model, 256, 192, mode="video", cadence=True)
    st = fh.Stream(eng, model, 256, 192, inputs=2, outputs=1)
    with pytest.raises(fh.FlyHighError, match="push two frames first"):
        st.generate(0.5, 0)
    with pytest.raises(fh.FlyHighError, match="bad input slot"):
        st.push(2, 0.0)
    with pytest.raises(fh.FlyHighError, match="bad output slot"):
        st.generate(0.5, 1)
    with pytest.raises(fh.FlyHighError, match="bytes"):
        st.write(0, b"\0" * 10)
    assert st.next_input([0, 1]) is None
    assert st.add_input() == 2 and st.next_input([0, 1]) == 2
    st.reset()
    assert st.report()["counters"]["resets"] == 1


def test_reference_classifier_cases(synth_model_dir, cuda):
    """crates/flyhigh-engine/tests/stream.rs:161-203 on the GPU: motion, hold and cut told apart; a local flash and its
    clear frame are both cuts though below the ordinary cut threshold."""
    import flyhigh_engine_b200 as fh
    from flyhigh_engine_b200.synth_frames import sinusoid_pair
    W, H = 256, 192
    eng, model = fh.Engine(), fh.Model(synth_model_dir)
    st = fh.Stream(eng, model, W, H, held_frames=True)
    flat = np.full((H, W, 4), 30, np.uint8)
    for slot, f in enumerate((sinusoid_pair(W, H, 0.0), sinusoid_pair(W, H, 2.0), sinusoid_pair(W, H, 0.0), flat)):
        st.write(slot, f)
    motion, hold, cut = st.classify(0, 1), st.classify(0, 2), st.classify(0, 3)
    assert motion.kind == "motion" and 0.0033 < motion.mean < 0.08 and not motion.black
    assert (hold.kind, hold.black) == ("hold", True)
    assert cut.kind == "cut"
    assert st.report()["counters"]["classified"] == 3
    st2 = fh.Stream(eng, model, W, H)
    original = np.zeros((H, W, 4), np.uint8)
    original[..., :3], original[..., 3] = 48, 255
    flash = original.copy()
    flash[:, 3 * W // 4:, :3] = 112
    st2.write(0, original)
    st2.write(1, flash)
    onset, clear = st2.classify(0, 1), st2.classify(1, 0)
    assert onset.mean < 0.08
    assert (onset.kind, clear.kind) == ("cut", "cut")


def _pan_pair(w, h, dx, dy, seed=21):
    """Two noise-free frames of a texture with a fence (dark 3-px bars every 16 px over its middle third), the second
    the first translated by (dx, dy) px: a camera pan that a single translation aligns exactly."""
    from flyhigh_engine_b200 import synth_frames
    m = 32
    tex = synth_frames.texture(w, h, np.random.default_rng(seed), margin=m)
    yy, xx = np.mgrid[0:h + 2 * m, 0:w + 2 * m]
    band = (yy > (h + 2 * m) // 3) & (yy < 2 * (h + 2 * m) // 3)
    bars = ((xx % 16) < 3) | ((yy % 16) < 3)
    tex[band & bars] = 30.0
    img = np.clip(tex, 0, 255).astype(np.uint8)

    def crop(ox, oy):
        f = np.empty((h, w, 4), np.uint8)
        f[..., :3] = img[m + oy:m + oy + h, m + ox:m + ox + w]
        f[..., 3] = 255
        return f
    return crop(0, 0), crop(dx, dy)


@pytest.mark.parametrize("t", [0.25, 0.5])
def test_pan_stage_matches_oracle(synth_model_dir, cuda, t):
    """Repair level 2 in a Stream adds the pan stage (pan.rs): the search after the pair and the apply on the generated
    frame. On an exact camera pan the pan is trusted, and the Stream's frame equals the session's frame of the same
    options with the oracle's pan search and apply on it, byte for byte."""
    import flyhigh_engine_b200 as fh
    from oracle import oracle
    w, h = 640, 360
    fa, fb = _pan_pair(w, h, 7, -3)
    fit = oracle.pan_search(fa, fb, w, h)
    assert fit[2] == 1.0 and abs(fit[0] + 7.0) < 0.5 and abs(fit[1] - 3.0) < 0.5, fit  # b(x) = a(x + (7, -3))
    model = fh.Model(synth_model_dir)
    st = fh.Stream(fh.Engine(), model, w, h, repair=2, scene_cut=0)
    st.write(0, fa)
    st.push(0, 0.0)
    st.write(1, fb)
    assert st.push(1, 1.0).ready
    assert st.generate(t, 0)
    got = np.frombuffer(st.read(0), np.uint8)
    s = fh.Session(fh.Engine(), model, w, h, repair=2)
    a, b, out = s.add_input(), s.add_input(), s.add_output()
    s.write(a, fa)
    s.write(b, fb)
    s.pair(a, b)
    s.mid(t, out)
    plain = np.frombuffer(s.read(out), np.uint8)
    p = model.plan_params(w, h, repair=2)
    ref = oracle.pan_apply(fa, fb, w, h, fit, t, plain, age=s.tensor("age")[0], min_age=p["min_age"])
    changed = int((ref != plain).reshape(-1, 4).any(1).sum())
    assert changed > (w * h) // 4, changed  # the pan rewrites most of the frame
    assert np.array_equal(got, ref), int((got != ref).reshape(-1, 4).any(1).sum())


def test_pan_stage_stays_off_without_a_pan(synth_model_dir, cuda):
    """Independent motion (config-2 rectangles over a random-walk pan with sensor noise) is not one translation: the
    pan is not trusted and a repair-2 Stream's frames equal the session's."""
    import flyhigh_engine_b200 as fh
    from flyhigh_engine_b200 import synth_frames
    from oracle import oracle
    w, h = 384, 192
    frames = synth_frames.sequence_c2(3, w, h, seed=31)
    assert oracle.pan_search(frames[1], frames[2], w, h)[2] <= 0.0
    model = fh.Model(synth_model_dir)
    st = fh.Stream(fh.Engine(), model, w, h, repair=2, scene_cut=0)
    s = fh.Session(fh.Engine(), model, w, h, repair=2)
    a, b, out = s.add_input(), s.add_input(), s.add_output()
    for i, f in enumerate(frames):
        st.write(i, f)
        st.push(i, float(i))
        s.write(a if i % 2 == 0 else b, f)
        if i:
            s.pair(b if i % 2 == 0 else a, a if i % 2 == 0 else b)
    st.generate(0.5, 0)
    s.mid(0.5, out)
    assert st.read(0) == s.read(out)
