"""Seeded synthetic RGBA8 frames with the shapes and statistics of the benchmark configurations.

No public image or video set is used: the reference's quality sets are not distributed with it. These generators stand
in for them:
  - texture(): a sum of 8 random 2-D sinusoids with periods 8..128 px, plus uniform noise of +-10, clamped to 0..255;
  - pair_c0(): config 0, frame b = frame a under an integer global pan in [-12, 12]^2 plus 3 rectangles of 20..80 px
    that move independently by up to 24 px;
  - sequence_c2(): config 2, a moving sequence whose pan velocity random-walks by +-2 px per frame, with 5 moving
    rectangles and a static 300 x 60 high-contrast HUD overlay at the bottom-left (noise-free, like a rendered HUD);
  - sequence_c3(): config 3, a camera pan of up to +-40 px per frame over a texture and a fence (a 32-px-period grid of
    bars) covering 30 % of the frame, the periodic structure the repair stage exists for;
  - stream_c4(): config 4's frame order for one stream: scenes of `cut_every` frames (a new seeded scene at each cut),
    2-frame held runs every `hold_every` frames (the frame after a run's first repeats it, anime on twos).
Every frame is (h, w, 4) uint8 with alpha 255.
"""
from __future__ import annotations

import numpy as np


def texture(w: int, h: int, rng: np.random.Generator, margin: int = 0) -> np.ndarray:
    """An RGB float texture of (h + 2 margin) x (w + 2 margin), values 0..255 before noise."""
    H, W = h + 2 * margin, w + 2 * margin
    y = np.arange(H, dtype=np.float32)[:, None]
    x = np.arange(W, dtype=np.float32)[None, :]
    img = np.zeros((H, W, 3), np.float32)
    for _ in range(8):
        period = rng.uniform(8.0, 128.0)
        ang = rng.uniform(0.0, np.pi)
        phase = rng.uniform(0.0, 2 * np.pi)
        amp = rng.uniform(10.0, 30.0, size=3).astype(np.float32)
        kx, ky = np.cos(ang) * 2 * np.pi / period, np.sin(ang) * 2 * np.pi / period
        wave = np.sin(kx * x + ky * y + phase).astype(np.float32)
        img += wave[..., None] * amp
    return img + 128.0


def _finish(rgb: np.ndarray, rng: np.random.Generator) -> np.ndarray:
    noisy = rgb + rng.uniform(-10.0, 10.0, size=rgb.shape).astype(np.float32)
    out = np.empty(rgb.shape[:2] + (4,), np.uint8)
    out[..., :3] = np.clip(noisy, 0, 255).astype(np.uint8)
    out[..., 3] = 255
    return out


def _rects(n, w, h, rng):
    rs = []
    for _ in range(n):
        rw, rh = int(rng.integers(20, 81)), int(rng.integers(20, 81))
        rs.append(dict(x=int(rng.integers(0, max(1, w - rw))), y=int(rng.integers(0, max(1, h - rh))), w=rw, h=rh,
                       color=rng.integers(0, 256, size=3).astype(np.float32)))
    return rs


def _paint(img, r, dx=0, dy=0):
    H, W = img.shape[:2]
    x0, y0 = r["x"] + dx, r["y"] + dy
    xa, ya, xb, yb = max(0, x0), max(0, y0), min(W, x0 + r["w"]), min(H, y0 + r["h"])
    if xa < xb and ya < yb:
        img[ya:yb, xa:xb, :] = r["color"]


def pair_c0(w: int = 640, h: int = 360, seed: int = 0):
    """Config 0: (frame a, frame b, (dx, dy))."""
    rng = np.random.default_rng(seed)
    m = 12
    base = texture(w, h, rng, margin=m)
    dx, dy = (int(v) for v in rng.integers(-12, 13, size=2))
    a = base[m:m + h, m:m + w].copy()
    b = base[m - dy:m - dy + h, m - dx:m - dx + w].copy()
    for r in _rects(3, w, h, rng):
        _paint(a, r)
        _paint(b, r, int(rng.integers(-24, 25)), int(rng.integers(-24, 25)))
    return _finish(a, rng), _finish(b, rng), (dx, dy)


def sequence_c2(n: int = 120, w: int = 1920, h: int = 1080, seed: int = 0, hud: bool = True):
    """Config 2: n frames. The pan velocity random-walks by +-2 px/frame (clamped to +-24), 5 rectangles move, a
    300 x 60 HUD stays fixed at the bottom-left."""
    rng = np.random.default_rng(seed)
    m = 24 * n // 4 + 64
    m = min(m, 1024)
    base = texture(w, h, rng, margin=m)
    rects = _rects(5, w, h, rng)
    vel = [rng.integers(-3, 4, size=2).astype(np.int64) for _ in rects]
    hud_img = np.zeros((60, 300, 3), np.float32)
    hud_img[:, :] = 16.0
    hud_img[10:50, 10:290] = 240.0
    hud_img[20:40, 40:260:20] = 16.0
    px, py, vx, vy = 0, 0, 0, 0
    frames = []
    for i in range(n):
        vx = int(np.clip(vx + rng.integers(-2, 3), -24, 24))
        vy = int(np.clip(vy + rng.integers(-2, 3), -24, 24))
        px = int(np.clip(px + vx, -m, m))
        py = int(np.clip(py + vy, -m, m))
        img = base[m + py:m + py + h, m + px:m + px + w].copy()
        for r, v in zip(rects, vel):
            r["x"] += int(v[0])
            r["y"] += int(v[1])
            _paint(img, r)
        f = _finish(img, rng)
        if hud:  # an overlay: composited after the sensor noise, identical in every frame
            f[h - 60 - 20:h - 20, 20:320, :3] = hud_img.astype(np.uint8)
        frames.append(f)
    return frames


def sequence_c3(n: int = 60, w: int = 3840, h: int = 2160, seed: int = 0):
    """Config 3: n frames of a pan whose velocity is drawn once per frame within +-40 px (x) and +-12 px (y); a region
    of 30 % of the frame shows a fence (dark 6-px bars every 32 px in both directions over a lit backdrop) that moves
    with the pan, as a camera panning past it would see it."""
    rng = np.random.default_rng(seed)
    m = min(40 * n + 64, 2048)
    base = texture(w, h, rng, margin=m)
    # the fence: a band of the frame's full width and 30 % of its height, centred vertically
    fh = int(round(0.3 * h))
    f0 = (h - fh) // 2
    yy = np.arange(h + 2 * m)[:, None]
    xx = np.arange(w + 2 * m)[None, :]
    bars = ((yy % 32) < 6) | ((xx % 32) < 6)
    fence = np.where(bars[..., None], 24.0, 200.0 + 0.2 * (base - 128.0)).astype(np.float32)
    px, py = 0, 0
    frames = []
    for _ in range(n):
        px = int(np.clip(px + rng.integers(-40, 41), -m, m))
        py = int(np.clip(py + rng.integers(-12, 13), -m, m))
        img = base[m + py:m + py + h, m + px:m + px + w].copy()
        img[f0:f0 + fh] = fence[m + py + f0:m + py + f0 + fh, m + px:m + px + w]
        frames.append(_finish(img, rng))
    return frames


def stream_c4(n: int = 240, cut_every: int = 48, hold_every: int = 30, scenes: int = 5, offset: int = 0):
    """Config 4's frame order for one stream: [(scene, frame within the scene)] for its n frames. Scene changes (cuts)
    every `cut_every` frames, starting at scene `offset`; frame i with i % hold_every == 1 repeats frame i - 1 (a 2-frame
    held run). The frames themselves come from per-scene sequences (sequence_c2 with the scene as seed)."""
    order = []
    for i in range(n):
        j = i - 1 if i % hold_every == 1 else i
        order.append(((j // cut_every + offset) % scenes, j % cut_every))
    return order


def sinusoid_pair(w: int, h: int, dx: float):
    """The reference's known-answer pattern (tests/core.rs:67-99): a soft pattern shifted dx px to the right."""
    v = np.zeros((h, w, 4), np.uint8)
    y = np.arange(h, dtype=np.float32)[:, None]
    x = np.arange(w, dtype=np.float32)[None, :]
    u = (x - np.float32(dx)) * np.float32(0.07)
    ww = y * np.float32(0.05)
    v[..., 0] = (128 + 100 * np.sin(u)).astype(np.uint8)
    v[..., 1] = (128 + 100 * np.cos(u * np.float32(0.7) + ww)).astype(np.uint8)
    v[..., 2] = (128 + 90 * np.sin(u + ww)).astype(np.uint8)
    v[..., 3] = 255
    return v
