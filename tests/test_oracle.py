"""The CPU oracle itself (CPU only): pinned against the reference's known-answer tests with the shipped weights, and
per op against torch where the shaders follow torch semantics (interp.wgsl:2-3 antialias = F.interpolate
antialias=True, warp.wgsl:2-3 = grid_sample align_corners=True border, conv = conv2d pad 1)."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import oracle


def _mae(a, b):
    return float(np.abs(a.astype(np.float64) - b.astype(np.float64)).mean())


def test_oracle_inbetween_known_answer(reference_models):
    """crates/flyhigh-engine/tests/core.rs:67-123 (and examples/c/main.c): a soft pattern shifted 8 px; the
    in-between at t = 0.5 is closer to the true middle (shift 4) than to either source, with MAE < 6. Session
    defaults (static protection and the still test on)."""
    from flyhigh_engine_b200.synth_frames import sinusoid_pair
    W, H = 256, 192
    f0, f1, mid = sinusoid_pair(W, H, 0.0), sinusoid_pair(W, H, 8.0), sinusoid_pair(W, H, 4.0)
    o = oracle.OracleSession(oracle.OracleModel(reference_models), W, H)
    o.pair(f0, f1)
    got = o.mid(0.5).reshape(H, W, 4)
    to_mid, to_f0, to_f1 = _mae(got, mid), _mae(got, f0), _mae(got, f1)
    assert to_mid < to_f0 and to_mid < to_f1 and to_mid < 6.0, (to_mid, to_f0, to_f1)
    # the generated frame at another phase moves with t (generate(0, 1, 0.25, 0) in tests/core.rs)
    q = o.mid(0.25).reshape(H, W, 4)
    assert _mae(q, sinusoid_pair(W, H, 2.0)) < _mae(q, sinusoid_pair(W, H, 6.0))


def test_oracle_internal_size_known_answer(reference_models):
    """The same pattern at 1280 x 720, where the network runs at the 480-line rung and the full-resolution render
    upsamples its flow."""
    from flyhigh_engine_b200.synth_frames import sinusoid_pair
    W, H = 1280, 720
    f0, f1, mid = sinusoid_pair(W, H, 0.0), sinusoid_pair(W, H, 8.0), sinusoid_pair(W, H, 4.0)
    o = oracle.OracleSession(oracle.OracleModel(reference_models), W, H)
    assert o.dims()["internal"]
    o.pair(f0, f1)
    got = o.mid(0.5).reshape(H, W, 4)
    to_mid, to_f0 = _mae(got, mid), _mae(got, f0)
    assert to_mid < to_f0 and to_mid < 6.0, (to_mid, to_f0)


def test_oracle_protection_mask(reference_models):
    """tests/core.rs:137-184: the host's mask takes the sources' pixels inside; outside it the in-between is kept."""
    from flyhigh_engine_b200.synth_frames import sinusoid_pair
    W, H = 256, 192
    f0, f1 = sinusoid_pair(W, H, 0.0), sinusoid_pair(W, H, 8.0)
    mask = np.zeros((H, W), np.uint8)
    mask[60:120, 100:160] = 1
    o = oracle.OracleSession(oracle.OracleModel(reference_models), W, H, protection_mask=True)
    o.write_mask(mask)
    o.pair(f0, f1)
    got = o.mid(0.5).reshape(H, W, 4).astype(np.float64)
    src = (f0.astype(np.float64) + f1.astype(np.float64)) / 2
    inside = np.abs(got[62:118, 102:158, :3] - src[62:118, 102:158, :3]).mean()
    assert inside < 1.0, inside


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


def test_oracle_fast_render_known_answer(reference_models):
    """tests/core.rs:222-262 and tests/gpu_smoke.rs:286-325 at 1280 x 720: the fast render reproduces the exact one
    (MAE < 0.5), and fast_render + linear_t stays within MAE < 4 of the true frame at t = 0.25, 0.5, 0.75 on linear
    motion, close to the exact render's own error."""
    W, H = 1280, 720
    m = oracle.OracleModel(reference_models)
    f0, f1 = _shift_pattern(W, H, 0.0), _shift_pattern(W, H, 16.0)
    runs = {}
    for name, kw in (("exact", {}), ("fast", dict(fast_render=True)), ("linear", dict(fast_render=True, linear_t=True))):
        o = oracle.OracleSession(m, W, H, **kw)
        o.pair(f0, f1)
        runs[name] = [o.mid(t).reshape(H, W, 4) for t in (0.25, 0.5, 0.75)]
    for i, dx in enumerate((4.0, 8.0, 12.0)):
        truth = _shift_pattern(W, H, dx)
        mae = lambda a, b: _mae(a[..., :3], b[..., :3])
        assert mae(runs["fast"][i], runs["exact"][i]) < 0.5
        assert mae(runs["linear"][i], truth) < 4.0
        assert mae(runs["linear"][i], truth) < mae(runs["exact"][i], truth) + 1.0


def _f16(a):
    return a.astype(np.float16)


def test_conv_matches_torch():
    rng = np.random.default_rng(0)
    for cin, cout, stride in [(3, 36, 2), (36, 36, 1), (96, 12, 1), (14, 24, 1)]:
        x = _f16(rng.standard_normal((cin, 23, 31)))
        w = _f16(rng.standard_normal((cout, cin, 3, 3)) / np.sqrt(9 * cin)).astype(np.float32)
        b = _f16(rng.standard_normal(cout) * 0.1).astype(np.float32)
        slope = np.full(cout, 0.1, np.float32)
        got = oracle.conv(x, w, b, slope, stride).astype(np.float32)
        ref = F.conv2d(torch.from_numpy(x.astype(np.float32))[None], torch.from_numpy(w), torch.from_numpy(b),
                       stride=stride, padding=1)
        ref = F.prelu(ref, torch.from_numpy(slope))[0].numpy().astype(np.float16).astype(np.float32)
        assert got.shape == ref.shape
        assert np.abs(got - ref).max() <= 2e-3 * max(1.0, np.abs(ref).max())


@pytest.mark.parametrize("src,dst", [((96, 160), (24, 40)), ((1088, 1920), (480, 864)), ((480, 864), (120, 216))])
def test_antialias_downscale_matches_torch(src, dst):
    rng = np.random.default_rng(1)
    x = _f16(rng.uniform(0, 1, (3,) + src))
    got = oracle.interp(x, dst[0], dst[1], aa=True).astype(np.float32)
    ref = F.interpolate(torch.from_numpy(x.astype(np.float32))[None], size=dst, mode="bilinear", align_corners=False,
                        antialias=True)[0].numpy()
    assert np.abs(got - ref).max() < 2e-3


def test_bilinear_upsample_matches_torch():
    rng = np.random.default_rng(2)
    x = _f16(rng.standard_normal((4, 30, 54)))
    got = oracle.interp(x, 60, 108, aa=False, scale=16.0).astype(np.float32)
    ref = 16.0 * F.interpolate(torch.from_numpy(x.astype(np.float32))[None], size=(60, 108), mode="bilinear",
                               align_corners=False)[0].numpy()
    assert np.abs(got - ref).max() <= 1e-3 * np.abs(ref).max()


def test_warp_matches_grid_sample():
    rng = np.random.default_rng(3)
    c, h, w = 3, 40, 56
    img = _f16(rng.uniform(0, 1, (c, h, w)))
    flow = _f16(rng.uniform(-12, 12, (2, h, w)))
    got = oracle.warp(img, flow).astype(np.float32)
    ys, xs = np.meshgrid(np.arange(h, dtype=np.float32), np.arange(w, dtype=np.float32), indexing="ij")
    gx = (xs + flow[0].astype(np.float32)) / (w - 1) * 2 - 1
    gy = (ys + flow[1].astype(np.float32)) / (h - 1) * 2 - 1
    grid = torch.from_numpy(np.stack([gx, gy], -1))[None]
    ref = F.grid_sample(torch.from_numpy(img.astype(np.float32))[None], grid, mode="bilinear", padding_mode="border",
                        align_corners=True)[0].numpy()
    assert np.abs(got - ref).max() < 2e-3
