"""The reference's known-answer tests on the CUDA path with the reference's shipped weights (models/flyhighfg.bin),
on a session run one interval at a time and on a batched session (4 intervals per launch, tcgen05 convs), then the
same frames against the oracle at the end-to-end frame criterion (tests/frame_parity.check_frame).

The weights are the reference's (CC BY-NC): a local copy (tests/_models, git-ignored, or FLYHIGH_MODELS) is read at
test time and never committed; without one these tests skip. They exercise the decision stages (the repair select,
the static rules, the still test) on real flows, which seeded N(0, 0.05) weights barely do.

- crates/flyhigh-engine/tests/core.rs:67-123: a soft pattern shifted 8 px; the in-between at t = 0.5 is closer to the
  true middle than to either source, MAE < 6; at t = 0.25 it is closer to the quarter shift than to the three-quarter.
- the same at 1280 x 720, where the network runs at the 480-line rung;
- tests/core.rs:137-184: the host's protection mask keeps the sources' pixels inside it;
- tests/core.rs:222-262 and tests/gpu_smoke.rs:286-325: the fast render reproduces the exact one (MAE < 0.5), and with
  linear_t stays within MAE < 4 of the true frame at t = 0.25 / 0.5 / 0.75.
"""
import numpy as np
import pytest

from tests.frame_parity import check_frame
from tests.parity import LAYER_REL_L2, rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _mae(a, b):
    a = np.asarray(a).reshape(-1, 4)[:, :3].astype(np.float64)
    b = np.asarray(b).reshape(-1, 4)[:, :3].astype(np.float64)
    return float(np.abs(a - b).mean())


def _shift_pattern(w, h, dx):
    """crates/flyhigh-engine/tests/core.rs:233-246: a soft pattern shifted dx px to the right."""
    x = np.arange(w, dtype=np.float32)[None, :]
    y = np.arange(h, dtype=np.float32)[:, None]
    u = (x - np.float32(dx)) * np.float32(0.05)
    f = np.zeros((h, w, 4), np.uint8)
    f[..., 0] = np.broadcast_to(128 + 100 * np.sin(u), (h, w)).astype(np.uint8)
    f[..., 1] = (128 + 90 * np.cos(u * np.float32(0.7) + y * np.float32(0.03))).astype(np.uint8)
    f[..., 2] = np.broadcast_to(128 + 80 * np.sin(y * np.float32(0.04)), (h, w)).astype(np.uint8)
    f[..., 3] = 255
    return f


def _run(models, w, h, shifts, t=0.5, batch=None, **opts):
    """Consecutive intervals of the sinusoid pattern at the given shifts: (GPU frames, oracle frames, session, oracle
    session, per-interval (network maps, oracle maps, age, gmhs records)) for the last interval."""
    import flyhigh_engine_b200 as fh
    from flyhigh_engine_b200.synth_frames import sinusoid_pair
    from oracle.oracle import OracleModel, OracleSession
    frames = [sinusoid_pair(w, h, dx) for dx in shifts]
    model = fh.Model(models)
    s = fh.Session(fh.Engine(), model, w, h, batch=batch, **opts)
    ins = [s.add_input(), s.add_input()]
    outs = [s.add_output() for _ in frames]
    s.write(ins[0], frames[0])
    for i in range(1, len(frames)):
        s.write(ins[i % 2], frames[i])
        s.pair(ins[(i - 1) % 2], ins[i % 2])
        s.mid(t, outs[i])
    got = [np.frombuffer(s.read(outs[i]), np.uint8).copy() for i in range(1, len(frames))]
    o = OracleSession(OracleModel(models), w, h, **{k: v for k, v in opts.items() if k in ("protection_mask",)})
    ref = []
    for i in range(1, len(frames)):
        o.pair(frames[i - 1], frames[i])
        ref.append(o.mid(t))
    return frames, got, ref, s, o


@pytest.mark.parametrize("batch", [None, 4])
def test_inbetween_known_answer(reference_models, cuda, batch):
    """8-px shifts: one interval on its own; with a batch, two chained intervals (0 -> 8 -> 16) in one launch."""
    import flyhigh_engine_b200 as fh
    from flyhigh_engine_b200.synth_frames import sinusoid_pair
    W, H = 256, 192
    shifts = [0.0, 8.0] if batch is None else [0.0, 8.0, 16.0]
    frames, got, ref, s, o = _run(reference_models, W, H, shifts, batch=batch)
    for i, g in enumerate(got):
        mid = sinusoid_pair(W, H, shifts[i] + 4.0)
        to_mid, to_a, to_b = _mae(g, mid), _mae(g, frames[i]), _mae(g, frames[i + 1])
        assert to_mid < to_a and to_mid < to_b and to_mid < 6.0, (i, to_mid, to_a, to_b)
    # the last interval against the oracle: layers and the frame criterion
    k = len(got) - 1
    iv = -1 if batch is None else k
    pp = fh.Model(reference_models).plan_params(W, H)
    for n, stage in (("o", 0), ("flow", 0), ("fr3", 0), ("up7", 1)):
        assert rel_l2(s.tensor(n, iv), o.tensor(n, stage)) <= LAYER_REL_L2, n
    # the residual nearly vanishes on this smooth pattern (|R_t| ~ 1e-3, the sum of much larger terms of the last
    # refine conv), so its relative L2 measures f16 ulps of a cancellation; what the frame sees of it is the absolute
    # difference, which the render adds to [0, 1] values: below a twentieth of a level
    assert np.abs(s.tensor("R_t", iv) - o.tensor("R_t", 1)).max() * 255 < 0.05
    age = s.tensor("age", iv)
    assert np.array_equal(age, o.tensor("age"))
    rep = check_frame(got[k], ref[k], frames[k], frames[k + 1], W, H, pp, (s.tensor("up7", iv), s.tensor("R_t", iv)),
                      (o.tensor("up7", 1), o.tensor("R_t", 1)), age)
    assert rep["ok"], rep
    if batch is None:  # a further phase of the same pair moves with t (generate(0, 1, 0.25, 0) in tests/core.rs)
        out = s.add_output()
        s.mid(0.25, out)
        q = np.frombuffer(s.read(out), np.uint8)
        assert _mae(q, sinusoid_pair(W, H, 2.0)) < _mae(q, sinusoid_pair(W, H, 6.0))


@pytest.mark.parametrize("batch", [None, 4])
def test_internal_size_known_answer(reference_models, cuda, batch):
    """1280 x 720: the network at the 480-line rung, the render upsamples its flow to the frame."""
    import flyhigh_engine_b200 as fh
    from flyhigh_engine_b200.synth_frames import sinusoid_pair
    W, H = 1280, 720
    shifts = [0.0, 8.0] if batch is None else [0.0, 8.0, 16.0]
    frames, got, ref, s, o = _run(reference_models, W, H, shifts, batch=batch)
    for i, g in enumerate(got):
        mid = sinusoid_pair(W, H, shifts[i] + 4.0)
        to_mid, to_a = _mae(g, mid), _mae(g, frames[i])
        assert to_mid < to_a and to_mid < 6.0, (i, to_mid, to_a)
    k = len(got) - 1
    iv = -1 if batch is None else k
    pp = fh.Model(reference_models).plan_params(W, H)
    age = s.tensor("age", iv)
    assert np.array_equal(age, o.tensor("age"))
    rep = check_frame(got[k], ref[k], frames[k], frames[k + 1], W, H, pp, (s.tensor("up7", iv), s.tensor("R_t", iv)),
                      (o.tensor("up7", 1), o.tensor("R_t", 1)), age)
    assert rep["ok"], rep


def test_protection_mask_known_answer(reference_models, cuda):
    import flyhigh_engine_b200 as fh
    from flyhigh_engine_b200.synth_frames import sinusoid_pair
    W, H = 256, 192
    f0, f1 = sinusoid_pair(W, H, 0.0), sinusoid_pair(W, H, 8.0)
    mask = np.zeros((H, W), np.uint8)
    mask[60:120, 100:160] = 1
    s = fh.Session(fh.Engine(), fh.Model(reference_models), W, H, protection_mask=True)
    a, b, out = s.add_input(), s.add_input(), s.add_output()
    s.write_mask(mask)
    s.write(a, f0)
    s.write(b, f1)
    s.pair(a, b)
    s.mid(0.5, out)
    got = np.frombuffer(s.read(out), np.uint8).reshape(H, W, 4).astype(np.float64)
    src = (f0.astype(np.float64) + f1.astype(np.float64)) / 2
    assert np.abs(got[62:118, 102:158, :3] - src[62:118, 102:158, :3]).mean() < 1.0
    mid = sinusoid_pair(W, H, 4.0).astype(np.float64)
    outside = np.ones((H, W), bool)
    outside[56:124, 96:164] = False
    assert np.abs(got[outside][:, :3] - mid[outside][:, :3]).mean() < 6.0


def test_fast_render_known_answer(reference_models, cuda):
    """1280 x 720: fast_render reproduces the exact render (MAE < 0.5); fast_render + linear_t stays within MAE < 4 of
    the true frame at three phases of linear motion, close to the exact render's own error."""
    import flyhigh_engine_b200 as fh
    W, H = 1280, 720
    model = fh.Model(reference_models)
    f0, f1 = _shift_pattern(W, H, 0.0), _shift_pattern(W, H, 16.0)
    runs = {}
    for name, kw in (("exact", {}), ("fast", dict(fast_render=True)), ("linear", dict(fast_render=True, linear_t=True))):
        s = fh.Session(fh.Engine(), model, W, H, **kw)
        a, b, out = s.add_input(), s.add_input(), s.add_output()
        s.write(a, f0)
        s.write(b, f1)
        s.pair(a, b)
        frames = []
        for t in (0.25, 0.5, 0.75):
            s.mid(t, out)
            frames.append(np.frombuffer(s.read(out), np.uint8).copy())
        runs[name] = frames
    for i, dx in enumerate((4.0, 8.0, 12.0)):
        truth = _shift_pattern(W, H, dx)
        assert _mae(runs["fast"][i], runs["exact"][i]) < 0.5
        assert _mae(runs["linear"][i], truth) < 4.0
        assert _mae(runs["linear"][i], truth) < _mae(runs["exact"][i], truth) + 1.0
