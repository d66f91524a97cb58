"""The camera warp on the GPU (fh_warp_*, fh_stream_mouse / _warp; crates/flyhigh-engine/src/warp/gpu.rs): each kernel
against the oracle's restatement on the same inputs (cell grids, every level's search and minimum, the lock mask, its
growth, the render), then the reference's own GPU tests (crates/flyhigh-engine/tests/warp.rs:230-463) on the same
synthetic scenes: panned shifts measured past the weapon, a flat picture unmeasured, the weapon masked, the render
turning the world, and a Stream learning the mouse and presenting a late frame where the camera is now."""
import json

import numpy as np
import pytest

from warp_scenes import FPS, GAIN, H, LAG, LOCK, W, frame, play, region_error

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


@pytest.fixture(scope="module")
def engine(torch_cuda):
    import flyhigh_engine_b200 as fh
    return fh.Engine()


def _dev(torch, rgba):
    t = torch.from_numpy(np.ascontiguousarray(rgba)).cuda()
    torch.cuda.synchronize()
    return t


class _DeviceFrame:
    """An rgba8 frame at a raw device pointer, as torch reads it (__cuda_array_interface__)."""

    def __init__(self, ptr, h, w):
        self.__cuda_array_interface__ = {"shape": (h, w, 4), "typestr": "|u1", "data": (int(ptr), False),
                                         "version": 2, "strides": None}


def _read(torch, ptr, w, h):
    torch.cuda.synchronize()  # the warp renders on a stream of its own
    return torch.as_tensor(_DeviceFrame(ptr, h, w), device="cuda").cpu().numpy()


def _scaled_lock(w, h):
    return (LOCK[0] * w // W, LOCK[1] * h // H, LOCK[2] * w // W, LOCK[3] * h // H)


@pytest.mark.parametrize("w,h", [(640, 360), (1920, 1080)])
def test_kernels_match_oracle(torch_cuda, engine, w, h):
    """One measured pair and a render: the cell grids within the last-bit differences of the trigonometric functions,
    each level's search and minimum from the GPU's own grids to 1e-4 px, the lock mask equal wherever its score is not
    within 1e-4 of the threshold, the grown mask and the rendered bytes equal."""
    import flyhigh_engine_b200 as fh
    from oracle import oracle as orc
    torch = torch_cuda
    lock = _scaled_lock(w, h)
    a, b = frame((0.0, 0.0), w, h, lock), frame((23.4 * w / W, 3.0 * h / H), w, h, lock)
    da, db = _dev(torch, a), _dev(torch, b)
    with fh.Warp(engine, w, h) as wp:
        wp.frame(da.data_ptr(), 0.0)
        wp.frame(db.data_ptr(), 16.7)
        wp.collect(wait=True)
        gbest = wp.tensor("best").reshape(3, 4)
        mgw, mgh = (w + 7) // 8, (h + 7) // 8
        for lv, (gw, gh, *_rest) in enumerate(orc.WARP_LEVELS):
            ga = wp.tensor(f"prev_cells{lv}").reshape(gh, gw)
            gb = wp.tensor(f"cells{lv}").reshape(gh, gw)
            for got, src in ((ga, a), (gb, b)):
                want = orc.warp_cells(src, w, h, lv)
                assert np.array_equal(got < 0, want < 0), f"level {lv}: cells outside the frame differ"
                # the device's and the host's tanf / cosf differ in the last bit: a sample point moves by up to
                # f * 2 ulp (about 1e-4 px at 1080p), a cell's luma by that times its slope (at most 1 per px)
                assert np.abs(got - want).max() <= 1e-4, (lv, float(np.abs(got - want).max()))
            coarse = gbest[lv - 1] if lv else np.zeros(4, np.float32)
            _, want_best = orc.warp_level(lv, ga, gb, w, h, coarse, np.zeros((mgh, mgw), np.float32))
            assert gbest[lv][2] == want_best[2], (lv, gbest[lv], want_best)
            assert np.abs(gbest[lv][:2] - want_best[:2]).max() <= 1e-4, (lv, gbest[lv], want_best)
            assert abs(gbest[lv][3] - want_best[3]) <= 1e-6, (lv, gbest[lv], want_best)
        # the whole chain from the frames alone
        obest, _, _, _ = orc.warp_measure(a, b, w, h)
        assert np.abs(obest[2][:2] - gbest[2][:2]).max() <= 1e-3 and obest[2][2] == gbest[2][2]
        # the lock on the GPU's result, the dilate on the GPU's mask
        gmask = wp.read_mask()
        omask, score = orc.warp_lock(a, b, w, h, gbest[2], np.zeros((mgh, mgw), np.float32))
        decided = ~(np.abs(score) < 1e-4)
        assert np.array_equal(gmask[decided], omask[decided])
        assert gmask.sum() > 0, "the weapon was locked"
        grown = wp.tensor("grown").reshape(mgh, mgw)
        np.testing.assert_array_equal(grown, orc.warp_dilate(gmask))
        # the render, bytes for bytes
        for sx, sy in ((30.0, 0.0), (-12.5, 6.25), (400.0, -150.0)):
            ptr = wp.render_shift(db.data_ptr(), sx, sy)
            got = _read(torch, ptr, w, h)
            want = orc.warp_render(b, w, h, grown, sx, sy)
            diff = np.abs(got.astype(np.int32) - want.astype(np.int32))
            assert diff.max() == 0, f"shift ({sx}, {sy}): {int((diff > 0).sum())} bytes differ, largest {diff.max()}"
        rep = wp.report()
        # cells of the first frame; cells, three searches, lock and dilate of the second; three renders
        assert rep["width"] == w and rep["height"] == h and rep["launches"] == 1 + 6 + 3


def test_the_shift_of_a_panned_frame_is_measured_past_the_screen_locked_weapon(torch_cuda, engine):
    """warp.rs:230-276"""
    import flyhigh_engine_b200 as fh
    torch = torch_cuda
    pans = [(40.0, 0.0), (23.4, 0.0), (-61.0, 0.0), (3.2, 0.0), (0.0, 0.0), (-1.4, 0.0), (140.0, 0.0), (-144.2, 0.0),
            (0.0, 6.0), (0.0, -25.0), (0.0, 1.5)]
    with fh.Warp(engine, W, H) as wp:
        at = (0.0, 0.0)
        keep = [_dev(torch, frame(at))]
        wp.frame(keep[0].data_ptr(), 0.0)
        for i, pan in enumerate(pans):
            at = (at[0] + pan[0], at[1] + pan[1])
            keep.append(_dev(torch, frame(at)))
            wp.frame(keep[-1].data_ptr(), 16.7 * (i + 1))
            torch.cuda.synchronize()
            wp.collect()
            s = wp.last_shift()
            assert s is not None, f"pan {pan}: no shift measured"
            tol = 0.75 if pan[1] == 0.0 else 0.75 + 0.04 * abs(pan[1])
            assert abs(s[0] - pan[0]) < tol and abs(s[1] - pan[1]) < tol, f"pan {pan} measured {s}"


def test_a_flat_picture_has_no_shift(torch_cuda, engine):
    """warp.rs:278-292"""
    import flyhigh_engine_b200 as fh
    torch = torch_cuda
    grey = _dev(torch, np.full((H, W, 4), 128, np.uint8))
    grey2 = _dev(torch, np.full((H, W, 4), 128, np.uint8))
    with fh.Warp(engine, W, H) as wp:
        wp.frame(grey.data_ptr(), 0.0)
        wp.frame(grey2.data_ptr(), 16.7)
        torch.cuda.synchronize()
        wp.collect()
        assert wp.last_shift() is None, "nothing to measure is not a still camera"


def _measure(torch, engine, a, b):
    import flyhigh_engine_b200 as fh
    wp = fh.Warp(engine, W, H)
    ta, tb = _dev(torch, frame(a)), _dev(torch, frame(b))
    wp.frame(ta.data_ptr(), 0.0)
    wp.frame(tb.data_ptr(), 16.7)
    torch.cuda.synchronize()
    wp.collect()
    return wp, (ta, tb)


def test_the_weapon_is_masked_and_the_world_is_not(torch_cuda, engine):
    """warp.rs:294-318"""
    wp, _keep = _measure(torch_cuda, engine, (0.0, 0.0), (23.4, 0.0))
    m = wp.read_mask().reshape(-1)
    gw = (W + 7) // 8
    inside, outside = [], []
    for i, v in enumerate(m):
        bx, by = (i % gw) * 8, (i // gw) * 8
        if bx >= LOCK[0] and bx + 8 <= LOCK[2] and by >= LOCK[1] and by + 8 <= LOCK[3]:
            inside.append(v)
        elif bx + 16 <= LOCK[0] or by + 16 <= LOCK[1]:
            outside.append(v)
    assert np.mean(inside) > 0.9, "the weapon is locked to the screen"
    assert np.mean(outside) < 0.02, "the world is not"
    wp.close()


def test_the_render_turns_the_world_by_the_shift_and_keeps_the_weapon(torch_cuda, engine):
    """warp.rs:320-340"""
    torch = torch_cuda
    pan = (23.4, 0.0)
    wp, _keep = _measure(torch, engine, (0.0, 0.0), pan)
    src = frame(pan)
    tb = _dev(torch, src)
    out = _read(torch, wp.render_shift(tb.data_ptr(), 30.0, 0.0), W, H)
    want = frame((pan[0] + 30.0, pan[1]))
    cx, cy = W // 2, H // 2
    turned = region_error(out, want, cx - 40, cy - 40, cx + 40, cy + 40)
    kept = region_error(out, src, cx - 40, cy - 40, cx + 40, cy + 40)
    weapon = region_error(out, src, LOCK[0] + 16, LOCK[1] + 16, LOCK[2] - 16, LOCK[3])
    assert turned < 3.0 and kept > 15.0, "the centre shows the world turned the right way"
    assert weapon < 1.0, "the weapon keeps its own pixels"
    # render_into another buffer: the same bytes
    dst = torch.zeros((H, W, 4), dtype=torch.uint8, device="cuda")
    wp.render_into(tb.data_ptr(), dst.data_ptr(), 30.0, 0.0)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(dst.cpu().numpy(), out)
    wp.close()


def test_the_stream_learns_the_mouse_and_shows_a_late_frame_where_the_camera_is_now(torch_cuda, synth_model_dir):
    """warp.rs:342-463: 5 s of synthetic play through a realtime Stream (each push runs its pair on the network); once
    calibrated, the frame before the newest, presented now, shows the camera where the mouse has it now."""
    import flyhigh_engine_b200 as fh
    torch = torch_cuda
    eng = fh.Engine()
    st = fh.Stream(eng, fh.Model(synth_model_dir), W, H)
    assert st.report()["camera_warp"] is None and st.camera_warp() is None
    assert not st.warp(0, 0, 0.0), "no mouse input: the warp is off"
    secs = 5.0
    counts, _ = play(secs)
    cam = np.concatenate(([0.0], np.cumsum(counts * GAIN)))
    next_frame = 0.0
    last = None
    checked = 0
    for i, k in enumerate(counts):
        t = float(i)
        st.mouse(t, float(k), 0.0)
        if t < next_frame:
            continue
        next_frame += 1000.0 / FPS
        slot = st.next_input()
        st.write(slot, frame((cam[int(max(t - LAG, 0.0))], 0.0)))
        st.push(slot, t)
        if last is not None and t > 3500.0 and abs(cam[i] - cam[int(t - 1000.0 / FPS - LAG)]) > 8.0 and checked < 6:
            prev = last[0]
            torch.cuda.synchronize()
            assert st.warp(prev, 0, t), f"the warp is on at {t} ms"
            out = np.frombuffer(st.read(0), np.uint8).reshape(H, W, 4)
            now_cam = cam[i + 1]  # the mouse event at t itself is in
            shown = cam[int(t - 1000.0 / FPS - LAG)]
            cx, cy = W // 2, H // 2
            to_now = region_error(out, frame((now_cam, 0.0)), cx - 120, cy - 80, cx + 80, cy + 40)
            to_late = region_error(out, frame((shown, 0.0)), cx - 120, cy - 80, cx + 80, cy + 40)
            assert to_now < 1.0 and to_now < 0.05 * to_late, (t, now_cam, shown, to_now, to_late)
            checked += 1
        last = (slot, t)
    r = st.report()["camera_warp"]
    assert r["on"] and abs(r["lag_ms"] - LAG) <= 5.0 and abs(r["gain_x"] / GAIN - 1.0) < 0.05, r
    assert checked >= 3, f"enough turning frames were checked ({checked})"
    assert st.report()["counters"]["warped"] == checked
    # a released mouse: nothing written, the frame is presented as it is
    st.set_mouse_captured(False)
    slot, t = last
    assert not st.warp(slot, 0, t + 10.0)
    assert st.report()["camera_warp"]["captured"] is False
    st.close()


def test_stream_warp_of_an_output_slot(torch_cuda, synth_model_dir):
    """A generated frame turned into another output slot and into its own slot (stream/mod.rs:548-562): the same bytes,
    those of the warp's render of that frame; `out` once turned is not turned again; a reset stops the measurement
    until a new pair."""
    import flyhigh_engine_b200 as fh
    torch = torch_cuda
    eng = fh.Engine()
    st = fh.Stream(eng, fh.Model(synth_model_dir), W, H, outputs=3)
    # teach the calibrator a plain relation: each frame shows the counts of 45 ms before, 0.138 px per count
    counts, _ = play(4.0)
    cam = np.concatenate(([0.0], np.cumsum(counts * GAIN)))
    next_frame, t = 0.0, 0.0
    for i, k in enumerate(counts):
        t = float(i)
        st.mouse(t, float(k), 0.0)
        if t >= next_frame:
            next_frame += 1000.0 / FPS
            slot = st.next_input()
            st.write(slot, frame((cam[int(max(t - LAG, 0.0))], 0.0)))
            st.push(slot, t)
    torch.cuda.synchronize()
    wp = st.camera_warp()
    assert wp is not None and st.report()["camera_warp"]["on"]
    assert st.generate(0.5, 0)
    base = np.frombuffer(st.read(0), np.uint8).reshape(H, W, 4)
    now = t + 5.0
    st.mouse(now, 40.0, 0.0)  # a turn the mouse made after the frame: 5.5 px at the calibrated gain
    assert st.warp(0, 1, now, output=True)
    one = np.frombuffer(st.read(1), np.uint8).reshape(H, W, 4)
    assert st.warp(0, 0, now, output=True)  # its own slot: through the warp's buffer
    own = np.frombuffer(st.read(0), np.uint8).reshape(H, W, 4)
    np.testing.assert_array_equal(one, own)
    assert region_error(one, base, 0, 0, W, H) > 1.0, "the frame was turned"
    assert not st.warp(0, 2, now, output=True), "slot 0 holds a turned frame: it has no moment any more"
    rep = st.report()
    assert rep["counters"]["warped"] == 2
    assert set(rep["camera_warp"]) == {"on", "captured", "r", "lag_ms", "gain_x", "gain_y"}
    # a reset: the next frame is measured against nothing
    st.reset()
    slot = st.next_input()
    st.write(slot, frame((0.0, 0.0)))
    st.push(slot, t + 500.0)
    torch.cuda.synchronize()
    wp.collect()
    assert wp.last_shift() is None
    json.dumps(wp.report())
    st.close()
