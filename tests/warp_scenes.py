"""Synthetic scenes of the reference's camera-warp tests (crates/flyhigh-engine/tests/warp.rs), restated in numpy: a
smooth non-periodic world seen by a camera turned by a yaw / pitch (pixels at the centre times the focal length of the
default 106 degree view), a screen-locked "weapon" block drawn over it, and the synthetic play of mouse counts (flicks
and tracking, 45 ms picture lag, 0.138 px per count)."""
import math

import numpy as np

W, H = 640, 360
# the weapon in hand: a block in the lower right that stays put while the world pans (warp.rs:139-140)
LOCK = (440, 230, 600, 360)
FPS, LAG, GAIN = 60.0, 45.0, 0.138


def focal(w=W):
    return 0.5 * w / math.tan(math.radians(53.0))


def world(x, y):
    """warp.rs:155-162: the world's colour at angular position (x, y) (radians times the focal length)."""
    u, v = x * 0.043, y * 0.061
    return (128.0 + 60.0 * np.sin(u + 0.7 * v) + 40.0 * np.cos(2.3 * u - 1.1 * v),
            128.0 + 70.0 * np.cos(1.7 * u) * np.sin(0.9 * v) + 30.0 * np.sin(3.1 * v + u),
            128.0 + 50.0 * np.sin(0.6 * u - 1.9 * v) + 45.0 * np.cos(2.9 * u + 0.3 * v))


def frame(turn, w=W, h=H, lock=LOCK):
    """warp.rs:168-197: the world seen by a camera turned by `turn` (px at the centre; positive moves the content right
    and down), with the screen-locked block drawn over it; rgba8 [h][w][4]."""
    f = focal(w)
    ty, tp = turn[0] / f, turn[1] / f
    y, x = np.mgrid[0:h, 0:w].astype(np.float64)
    dx, dy, dz = x + 0.5 - 0.5 * w, y + 0.5 - 0.5 * h, np.full_like(x, f)
    dx, dz = dx * math.cos(ty) - dz * math.sin(ty), dx * math.sin(ty) + dz * math.cos(ty)
    dy, dz = dy * math.cos(tp) - dz * math.sin(tp), dy * math.sin(tp) + dz * math.cos(tp)
    az = np.arctan2(dx, dz)
    el = np.arctan2(dy, np.sqrt(dx * dx + dz * dz))
    c = np.stack(world(az * f, el * f), -1)
    if lock is not None:
        # not periodic: a periodic weapon would match itself shifted by a period
        u, v = x * 0.05, y * 0.07
        k = np.sin(u * u * 0.3 + v) * np.cos(1.3 * v - 0.2 * u * v)
        weapon = np.stack((90.0 + 80.0 * k, 70.0 + 60.0 * k, 60.0 - 40.0 * k), -1)
        inside = (x >= lock[0]) & (x < lock[2]) & (y >= lock[1]) & (y < lock[3])
        c = np.where(inside[..., None], weapon, c)
    out = np.empty((h, w, 4), np.uint8)
    out[..., :3] = np.clip(c, 0.0, 255.0).astype(np.uint8)  # `as u8` after the clamp: truncation
    out[..., 3] = 255
    return out


class Lcg:
    """warp.rs:10-19"""

    def __init__(self, seed):
        self.s = seed

    def f(self):
        self.s = (self.s * 6364136223846793005 + 1442695040888963407) & 0xFFFFFFFFFFFFFFFF
        return (self.s >> 11) / float(1 << 53)

    def n(self):
        return sum(self.f() for _ in range(6)) - 3.0


def play(secs, menu=(1e9, 1e9)):
    """warp.rs:22-51: mouse counts per millisecond over `secs`, and whether the camera follows them each ms."""
    r = Lcg(7)
    n = int(secs * 1000.0)
    t = np.arange(n, dtype=np.float64)
    rate = np.zeros(n)
    for _ in range(int(secs * 1.6)):
        t0 = 500.0 + r.f() * (secs * 1000.0 - 1000.0)
        d = 40.0 + 80.0 * r.f()
        sign = -1.0 if r.f() < 0.5 else 1.0
        amp = sign * (2.0 + 9.0 * r.f())
        on = (t >= t0) & (t < t0 + d)
        rate[on] += amp * np.sin(math.pi * (t[on] - t0) / d)
    for i in range(n):
        rate[i] += 0.2 * r.n()
    if menu[0] < secs * 1000.0:
        tt = t - (menu[0] + 300.0)
        on = (tt >= 0.0) & (tt < 100.0)
        rate[on] += 8.0 * np.sin(math.pi * tt[on] / 100.0)
    follows = ~((t >= menu[0]) & (t < menu[1]))
    return rate, follows


def region_error(a, b, x0, y0, x1, y1):
    """Mean absolute rgb difference over [y0, y1) x [x0, x1) (warp.rs:289-302)."""
    return float(np.abs(a[y0:y1, x0:x1, :3].astype(np.float64) - b[y0:y1, x0:x1, :3].astype(np.float64)).mean())
