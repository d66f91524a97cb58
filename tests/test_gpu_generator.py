"""The Generator (fh_generator_*, crates/flyhigh-engine/src/api.rs:173-349 and crates/flyhigh-capi/src/lib.rs:66-258) on
the GPU: the frames to display in the reference's order (realtime: the in-betweens of (previous, newest) then the
newest; video: from the third push on, the interval two frames back: its source frame, then its in-betweens), each
generated frame the same bytes a plain session gives for that pair and phase, and its errors."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _session_frames(fh, model, w, h, frames, pairs, ts):
    """{(i, t): bytes} of a plain session for the pairs (i - 1, i) and phases ts, run in order."""
    s = fh.Session(fh.Engine(), model, w, h)
    a, b, out = s.add_input(), s.add_input(), s.add_output()
    got = {}
    for i in pairs:
        s.write(a, frames[i - 1])
        s.write(b, frames[i])
        s.pair(a, b)
        for t in ts:
            s.mid(t, out)
            got[(i, t)] = s.read(out)
    return got


def test_realtime_generator(synth_model_dir, cuda):
    import flyhigh_engine_b200 as fh
    from flyhigh_engine_b200 import synth_frames
    w, h, factor = 384, 192, 3
    frames = synth_frames.sequence_c2(6, w, h, seed=21)
    model = fh.Model(synth_model_dir)
    ts = [1.0 / 3.0, 2.0 / 3.0]
    want = _session_frames(fh, model, w, h, frames, range(1, 6), [np.float32(t).item() for t in ts])
    with fh.Generator(fh.Engine(), model, w, h) as g:
        assert g.warmup() == 1
        for i, f in enumerate(frames):
            out = g.frames(f, factor)
            if i == 0:
                assert [(p, r) for _, p, r in out] == [(0.0, True)]
            else:
                assert [r for _, _, r in out] == [False, False, True]
                for (rgba, p, _), t in zip(out[:2], ts):
                    assert p == pytest.approx(t)
                    assert rgba == want[(i, np.float32(t).item())], (i, t)
            assert out[-1][0] == f.tobytes()
        assert g.pop() is None


def test_video_generator(synth_model_dir, cuda):
    import flyhigh_engine_b200 as fh
    from flyhigh_engine_b200 import synth_frames
    w, h = 320, 192
    frames = synth_frames.sequence_c2(6, w, h, seed=22)
    model = fh.Model(synth_model_dir)
    want = _session_frames(fh, model, w, h, frames, range(1, 5), [0.5])
    with fh.Generator(fh.Engine(), model, w, h, mode="video") as g:
        assert g.warmup() == 3
        for i, f in enumerate(frames):
            out = g.frames(f, 2)
            if i < 2:
                assert out == []
                continue
            # the interval [f(i-2), f(i-1)): its source frame, then its middle
            assert [(p, r) for _, p, r in out] == [(0.0, True), (0.5, False)]
            assert out[0][0] == frames[i - 2].tobytes()
            assert out[1][0] == want[(i - 1, 0.5)], i


def test_generator_errors(synth_model_dir, cuda):
    import flyhigh_engine_b200 as fh
    from flyhigh_engine_b200 import synth_frames
    model = fh.Model(synth_model_dir)
    eng = fh.Engine()
    with pytest.raises(fh.FlyHighError, match="frame size too small"):
        fh.Generator(eng, model, 32, 32)
    with pytest.raises(fh.FlyHighError, match="cadence"):
        fh.Generator(eng, model, 256, 192, mode="video", cadence=True)
    with fh.Generator(eng, model, 256, 192) as g:
        with pytest.raises(fh.FlyHighError, match="frame size mismatch"):
            g.push(b"\0" * 100, 2)
        assert g.push(synth_frames.sequence_c2(1, 256, 192, seed=3, hud=False)[0], 2) == 1
        import ctypes
        small = (ctypes.c_uint8 * 16)()
        assert fh.lib().fh_generator_pop(g._h, ctypes.cast(small, ctypes.c_void_p), 16, None, None) == -1
        assert b"output buffer too small" in fh.lib().fh_last_error()
        assert g.pop() is not None and g.pop() is None
