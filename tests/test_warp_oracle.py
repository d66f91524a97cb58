"""The camera warp's CPU restatement (oracle/oracle.cpp camwarp) held to the reference's own GPU expectations
(crates/flyhigh-engine/tests/warp.rs:230-340) on the same synthetic scenes: the shift of a panned frame measured past
the screen-locked weapon, none for a flat picture, the weapon masked and the world not, and the render turning the
world by the shift while the weapon keeps its pixels. The GPU kernels are then compared with this restatement
(tests/test_gpu_warp.py)."""
import numpy as np
import pytest

from oracle import oracle as orc
from warp_scenes import H, LOCK, W, frame, region_error


def test_geometry_is_the_default_view():
    f, ha, he = orc.warp_geometry(W, H)
    assert abs(f - 0.5 * W / np.tan(np.radians(53.0))) < 1e-3
    assert abs(ha - np.radians(53.0)) < 1e-6
    assert abs(he - np.arctan(0.5 * H / f)) < 1e-6


def test_the_shift_of_a_panned_frame_is_measured_past_the_screen_locked_weapon():
    # warp.rs:232-276: the first turn teaches the mask; back to level yaw before the pitch steps
    pans = [(40.0, 0.0), (23.4, 0.0), (-61.0, 0.0), (3.2, 0.0), (0.0, 0.0), (-1.4, 0.0), (140.0, 0.0), (-144.2, 0.0),
            (0.0, 6.0), (0.0, -25.0), (0.0, 1.5)]
    at = (0.0, 0.0)
    prev = frame(at)
    mask = None
    for pan in pans:
        at = (at[0] + pan[0], at[1] + pan[1])
        cur = frame(at)
        best, mask, _, _ = orc.warp_measure(prev, cur, W, H, mask)
        prev = cur
        sx, sy, valid = best[2][:3]
        assert valid > 0.5, f"pan {pan}: no shift measured"
        # the angular grid is exact for yaw; pitch bends its rows a little away from the centre
        tol = 0.75 if pan[1] == 0.0 else 0.75 + 0.04 * abs(pan[1])
        assert abs(sx - pan[0]) < tol and abs(sy - pan[1]) < tol, f"pan {pan} measured ({sx:.2f}, {sy:.2f})"


def test_a_flat_picture_has_no_shift():
    grey = np.full((H, W, 4), 128, np.uint8)
    best, _, _, _ = orc.warp_measure(grey, grey, W, H)
    assert best[0][2] == 0.0 and best[2][2] == 0.0, "nothing to measure is not a still camera"


def _weapon_and_world(mask):
    gw = (W + 7) // 8
    inside, outside = [], []
    for i, v in enumerate(mask.reshape(-1)):
        bx, by = (i % gw) * 8, (i // gw) * 8
        if bx >= LOCK[0] and bx + 8 <= LOCK[2] and by >= LOCK[1] and by + 8 <= LOCK[3]:
            inside.append(v)
        elif bx + 16 <= LOCK[0] or by + 16 <= LOCK[1]:
            outside.append(v)
    return float(np.mean(inside)), float(np.mean(outside))


def test_the_weapon_is_masked_and_the_world_is_not():
    _, mask, _, _ = orc.warp_measure(frame((0.0, 0.0)), frame((23.4, 0.0)), W, H)
    inside, outside = _weapon_and_world(mask)
    assert inside > 0.9, "the weapon is locked to the screen"
    assert outside < 0.02, "the world is not"


def test_the_render_turns_the_world_by_the_shift_and_keeps_the_weapon():
    pan = (23.4, 0.0)
    _, _, grown, _ = orc.warp_measure(frame((0.0, 0.0)), frame(pan), W, H)
    src = frame(pan)
    out = orc.warp_render(src, W, H, grown, 30.0, 0.0)
    want = frame((pan[0] + 30.0, pan[1]))
    cx, cy = W // 2, H // 2
    assert region_error(out, want, cx - 40, cy - 40, cx + 40, cy + 40) < 3.0
    assert region_error(out, src, cx - 40, cy - 40, cx + 40, cy + 40) > 15.0
    assert region_error(out, src, LOCK[0] + 16, LOCK[1] + 16, LOCK[2] - 16, LOCK[3]) < 1.0


@pytest.mark.parametrize("level", [0, 1, 2])
def test_a_level_alone_agrees_with_the_whole_measurement(level):
    """or_warp_level (one level from given grids) is the step or_warp_measure chains: the GPU tests compare each level
    through it."""
    a, b = frame((0.0, 0.0)), frame((23.4, 3.0))
    best, _, _, _ = orc.warp_measure(a, b, W, H)
    ca, cb = orc.warp_cells(a, W, H, level), orc.warp_cells(b, W, H, level)
    coarse = best[level - 1] if level else np.zeros(4, np.float32)
    _, got = orc.warp_level(level, ca, cb, W, H, coarse, np.zeros(((H + 7) // 8, (W + 7) // 8), np.float32))
    np.testing.assert_array_equal(got, best[level])
