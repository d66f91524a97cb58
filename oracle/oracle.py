"""TEST INFRASTRUCTURE — ctypes front of the CPU oracle (oracle/oracle.cpp).

The oracle restates the reference's Session::pair / Session::mid (the FlyHighFG Core graph, its WGSL kernels and the
net/build.rs planner semantics) on the host cores. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
legs use it, as the checker and as the timed CPU baseline; the product never imports this module.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from ctypes import POINTER, c_char_p, c_float, c_int, c_long, c_uint8, c_uint16, c_void_p

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")


def build() -> str:
    """Compile liboracle.so with the Makefile beside this file (a few seconds)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        L = ctypes.CDLL(LIB)
        L.or_error.restype = c_char_p
        L.or_threads.restype = c_int
        L.or_threads.argtypes = [c_int]
        L.or_model_load.restype = c_void_p
        L.or_model_load.argtypes = [c_char_p]
        L.or_model_free.argtypes = [c_void_p]
        L.or_model_cubic.argtypes = [c_void_p]
        L.or_session_new.restype = c_void_p
        L.or_session_new.argtypes = [c_void_p, POINTER(c_int)]
        L.or_session_free.argtypes = [c_void_p]
        L.or_pair.argtypes = [c_void_p, POINTER(c_uint8), POINTER(c_uint8)]
        L.or_mid.argtypes = [c_void_p, c_float, POINTER(c_uint8)]
        L.or_write_mask.argtypes = [c_void_p, POINTER(c_uint8)]
        L.or_tensor.restype = c_long
        L.or_tensor.argtypes = [c_void_p, c_int, c_char_p, POINTER(c_float), c_long, POINTER(c_int)]
        L.or_session_dims.argtypes = [c_void_p, POINTER(c_int), POINTER(c_float)]
        L.or_render_planes.argtypes = [POINTER(c_uint8), POINTER(c_uint8), c_int, c_int, POINTER(c_float),
                                       POINTER(c_float), c_int, c_int, POINTER(c_float), POINTER(c_float),
                                       POINTER(c_int), POINTER(c_uint8)]
        L.or_render_tex_planes.argtypes = L.or_render_planes.argtypes
        L.or_render_diag.argtypes = L.or_render_planes.argtypes[:-1] + [c_int, POINTER(c_int), POINTER(c_float)]
        L.or_render_diag_size.restype = c_int
        L.or_gmhs_select.argtypes = [c_void_p, POINTER(c_float), c_int, c_int, POINTER(c_float)]
        L.or_classify.argtypes = [POINTER(c_uint8), POINTER(c_uint8), c_int, c_int, c_int, c_int, POINTER(ctypes.c_uint32)]
        L.or_pan_search.argtypes = [POINTER(c_uint8), POINTER(c_uint8), c_int, c_int, POINTER(c_float)]
        F, U8 = POINTER(c_float), POINTER(c_uint8)
        L.or_warp_geometry.argtypes = [c_int, c_int, ctypes.c_double, F]
        L.or_warp_cells.argtypes = [U8, c_int, c_int, c_int, ctypes.c_double, F]
        L.or_warp_level.argtypes = [c_int, F, F, c_int, c_int, ctypes.c_double, F, F, F, F]
        L.or_warp_measure.argtypes = [U8, U8, c_int, c_int, ctypes.c_double, c_float, c_float, F, F, F, F]
        L.or_warp_lock.argtypes = [U8, U8, c_int, c_int, ctypes.c_double, F, c_float, c_float, F, F]
        L.or_warp_dilate.argtypes = [F, c_int, c_int, F]
        L.or_warp_render.argtypes = [U8, c_int, c_int, ctypes.c_double, F, c_float, c_float, U8]
        L.or_pan_apply.argtypes = [POINTER(c_uint8), POINTER(c_uint8), c_int, c_int, POINTER(c_float), c_float,
                                   POINTER(c_float), c_int, c_float, POINTER(c_uint8)]
        L.or_tex_down.argtypes = [POINTER(c_uint8), c_int, c_int, c_int, c_int, POINTER(c_uint16)]
        L.or_interp.argtypes = [POINTER(c_uint16), c_int, c_int, c_int, c_int, c_int, c_int, c_float, POINTER(c_uint16)]
        L.or_warp.argtypes = [POINTER(c_uint16), c_int, c_int, c_int, POINTER(c_uint16), c_float, POINTER(c_uint16)]
        L.or_conv.argtypes = [POINTER(c_uint16), c_int, c_int, c_int, POINTER(c_float), POINTER(c_float),
                              POINTER(c_float), c_int, c_int, POINTER(c_uint16), POINTER(c_uint16)]
        _lib = L
    return _lib


def _u8(a: np.ndarray):
    return a.ctypes.data_as(POINTER(c_uint8))


class OracleModel:
    """graph.json + flyhighfg.json + flyhighfg.bin from a model directory."""

    def __init__(self, directory: str):
        self.h = lib().or_model_load(directory.encode())
        if not self.h:
            raise RuntimeError(lib().or_error().decode())

    @property
    def cubic(self) -> bool:
        return bool(lib().or_model_cubic(self.h))

    def __del__(self):
        if getattr(self, "h", None):
            lib().or_model_free(self.h)
            self.h = None


class OracleSession:
    """The reference session semantics on the CPU: defaults of SessionOptions::new (session.rs:118-135) with the
    still test on (options.rs:296-298)."""

    def __init__(self, model: OracleModel, width: int, height: int, internal=(0, 0), k: int = 1, repair: int = 1,
                 cubic: int = -1, keep_static: bool = True, static_frames: int = 8, static_tolerance: int = 4,
                 still: bool = True, decisive: bool = False, protection_mask: bool = False, fast_render: bool = False,
                 linear_t: bool = False):
        self.model = model
        self.w, self.h = width, height
        o = (c_int * 15)(width, height, internal[0], internal[1], k, repair, cubic, int(keep_static), static_frames,
                         static_tolerance, int(still), int(decisive), int(protection_mask), int(fast_render),
                         int(linear_t))
        self.s = lib().or_session_new(model.h, o)
        if not self.s:
            raise RuntimeError(lib().or_error().decode())

    def pair(self, a: np.ndarray, b: np.ndarray) -> None:
        a = np.ascontiguousarray(a, dtype=np.uint8)
        b = np.ascontiguousarray(b, dtype=np.uint8)
        assert a.size == self.w * self.h * 4 and b.size == a.size
        if lib().or_pair(self.s, _u8(a), _u8(b)) != 0:
            raise RuntimeError(lib().or_error().decode())

    def mid(self, t: float) -> np.ndarray:
        out = np.zeros(self.w * self.h * 4, np.uint8)
        if lib().or_mid(self.s, c_float(t), _u8(out)) != 0:
            raise RuntimeError(lib().or_error().decode())
        return out

    def write_mask(self, mask: np.ndarray) -> None:
        m = np.ascontiguousarray(mask, dtype=np.uint8)
        assert m.size == self.w * self.h
        if lib().or_write_mask(self.s, _u8(m)) != 0:
            raise RuntimeError("the session was built without protection_mask")

    def tensor(self, name: str, stage: int = 0) -> np.ndarray:
        """A tensor of the last pair (stage 0) or mid (stage 1), f32 [c][h][w] with its view applied."""
        dims = (c_int * 3)()
        n = lib().or_tensor(self.s, stage, name.encode(), None, 0, dims)
        if n < 0:
            raise KeyError(name)
        out = np.zeros(n, np.float32)
        lib().or_tensor(self.s, stage, name.encode(), out.ctypes.data_as(POINTER(c_float)), n, dims)
        return out.reshape(dims[0], dims[1], dims[2])

    def gmhs_select(self, flow_pre: np.ndarray) -> dict:
        """The repair stage's decisions on the last pair's frames for a given pre-repair flow [4][h8][w8]: "sel" (1 where
        the affine flow replaces the network's) and the margins of its three conditions "m_cost" (cm - ca), "m_dv"
        (dv - dmin), "m_sd" (sd - tex), each [h8][w8]; a cell is selected exactly when all three are positive."""
        f = np.ascontiguousarray(flow_pre, np.float32)
        _, h8, w8 = f.shape
        out = np.zeros(4 * h8 * w8, np.float32)
        P = lambda a: a.ctypes.data_as(POINTER(c_float))
        if lib().or_gmhs_select(self.s, P(f), h8, w8, P(out)) != 0:
            raise RuntimeError(lib().or_error().decode())
        r = out.reshape(h8, w8, 4)
        return {"sel": r[..., 0], "m_cost": r[..., 1], "m_dv": r[..., 2], "m_sd": r[..., 3]}

    def dims(self) -> dict:
        iv = (c_int * 9)()
        fv = (c_float * 4)()
        lib().or_session_dims(self.s, iv, fv)
        return dict(hp=iv[0], wp=iv[1], ihp=iv[2], iwp=iv[3], internal=bool(iv[4]), r_blk=iv[5], r_dwin=iv[6],
                    hc=iv[7], wc=iv[8], dmin=fv[0], delta=fv[1], fsx=fv[2], fsy=fv[3])

    def __del__(self):
        if getattr(self, "s", None):
            lib().or_session_free(self.s)
            self.s = None


def threads(n: int = 0) -> int:
    """The host threads the oracle's OpenMP loops use; n > 0 sets them (a launcher may have set OMP_NUM_THREADS=1)."""
    return int(lib().or_threads(int(n)))


def conv(x: np.ndarray, w: np.ndarray, bias: np.ndarray, slope, stride: int, resid=None) -> np.ndarray:
    """One conv of the tensor-core path on CHW f16 x ([cin][h][w]) with torch-layout weights; f16 output."""
    x = np.ascontiguousarray(x, dtype=np.float16)
    cin, h, wd = x.shape
    cout = w.shape[0]
    ho, wo = (h - 1) // stride + 1, (wd - 1) // stride + 1
    W = np.ascontiguousarray(w, dtype=np.float32)
    B = np.ascontiguousarray(bias, dtype=np.float32)
    Sl = None if slope is None else np.ascontiguousarray(slope, dtype=np.float32)
    out = np.zeros((cout, ho, wo), np.float16)
    R = None if resid is None else np.ascontiguousarray(resid, dtype=np.float16)
    f = lambda a: a.ctypes.data_as(POINTER(c_float))
    u = lambda a: a.ctypes.data_as(POINTER(c_uint16))
    lib().or_conv(u(x), cin, h, wd, f(W), f(B), f(Sl) if Sl is not None else None, cout, stride,
                  u(R) if R is not None else None, u(out))
    return out


def render_planes(fa, fb, w, h, up7, rt, age, fsx, fsy, min_age, static_thr, cubic=True, flags=2):
    """The render alone on given network outputs (up7 [7][hq][wq], R_t [3][hq][wq], age [hp][wp] or None)."""
    fa = np.ascontiguousarray(fa, np.uint8)
    fb = np.ascontiguousarray(fb, np.uint8)
    up7 = np.ascontiguousarray(up7, np.float32)
    rt = np.ascontiguousarray(rt, np.float32)
    hq, wq = up7.shape[1], up7.shape[2]
    ag = None if age is None else np.ascontiguousarray(age, np.float32)
    fv = np.array([fsx, fsy, min_age, static_thr], np.float32)
    iv = np.array([int(cubic), int(flags)], np.int32)
    out = np.zeros(w * h * 4, np.uint8)
    f = lambda a: a.ctypes.data_as(POINTER(c_float))
    rc = lib().or_render_planes(_u8(fa), _u8(fb), w, h, f(up7), f(rt), hq, wq, f(ag) if ag is not None else None,
                                f(fv), iv.ctypes.data_as(POINTER(c_int)), _u8(out))
    if rc != 0:
        raise RuntimeError(lib().or_error().decode())
    return out


DIAG_FIELDS = ["gxa", "gya", "gxb", "gyb", "sa", "sb", "stillw", "ramp", "es", "bwa", "bwb", "rk", "raw", "range_a",
               "range_b", "ca0", "ca1", "ca2", "cb0", "cb1", "cb2", "cr0", "cr1", "cr2", "own0", "own1", "own2", "age"]


def render_diag(fa, fb, w, h, up7, rt, age, fsx, fsy, min_age, xs, ys, cubic=True, flags=2):
    """The render's decision record at pixels (xs[i], ys[i]) on given network outputs, as render_planes evaluates them:
    a dict of DIAG_FIELDS -> float32 arrays (source positions, static-rule hits, still weight and its ramp input, blend
    weights, tap value ranges, the blended terms, the age)."""
    fa = np.ascontiguousarray(fa, np.uint8)
    fb = np.ascontiguousarray(fb, np.uint8)
    up7 = np.ascontiguousarray(up7, np.float32)
    rt = np.ascontiguousarray(rt, np.float32)
    hq, wq = up7.shape[1], up7.shape[2]
    ag = None if age is None else np.ascontiguousarray(age, np.float32)
    fv = np.array([fsx, fsy, min_age, 0.0], np.float32)
    iv = np.array([int(cubic), int(flags)], np.int32)
    xy = np.ascontiguousarray(np.stack([np.asarray(xs, np.int32), np.asarray(ys, np.int32)], 1).reshape(-1))
    n = xy.size // 2
    k = lib().or_render_diag_size()
    assert k == len(DIAG_FIELDS)
    out = np.zeros(max(n, 1) * k, np.float32)
    f = lambda a: a.ctypes.data_as(POINTER(c_float))
    rc = lib().or_render_diag(_u8(fa), _u8(fb), w, h, f(up7), f(rt), hq, wq, f(ag) if ag is not None else None,
                              f(fv), iv.ctypes.data_as(POINTER(c_int)), n, xy.ctypes.data_as(POINTER(c_int)), f(out))
    if rc != 0:
        raise RuntimeError(lib().or_error().decode())
    out = out[:n * k].reshape(n, k)
    return {name: out[:, i] for i, name in enumerate(DIAG_FIELDS)}


def interp(x, oh: int, ow: int, aa: bool, scale: float = 1.0):
    """interp.wgsl on [c][h][w] f16 values (bilinear align_corners=False, or the antialias triangle filter)."""
    x = np.ascontiguousarray(x, dtype=np.float16)
    c, h, w = x.shape
    out = np.zeros((c, oh, ow), np.float16)
    u = lambda a: a.ctypes.data_as(POINTER(c_uint16))
    lib().or_interp(u(x), c, h, w, oh, ow, int(aa), c_float(scale), u(out))
    return out


def warp(img, flow, flow_scale: float = 1.0):
    """warp.wgsl: backward bilinear warp with border clamp of [c][h][w] by flow [2][h][w] (px, x flow_scale)."""
    img = np.ascontiguousarray(img, dtype=np.float16)
    flow = np.ascontiguousarray(flow, dtype=np.float16)
    c, h, w = img.shape
    out = np.zeros((c, h, w), np.float16)
    u = lambda a: a.ctypes.data_as(POINTER(c_uint16))
    lib().or_warp(u(img), c, h, w, u(flow), c_float(flow_scale), u(out))
    return out


def render_tex_planes(fa, fb, w, h, up7, rt, age, fsx, fsy, min_age, cubic=True, flags=2, sa=1.0, sb=1.0, sr=1.0):
    """The fast render (render_tex.wgsl) alone on given network outputs (up7 [7][hq][wq], R_t [3][hq][wq], age
    [hp][wp] or None); rgba8 out."""
    fa = np.ascontiguousarray(fa, np.uint8)
    fb = np.ascontiguousarray(fb, np.uint8)
    up7 = np.ascontiguousarray(up7, np.float32)
    rt = np.ascontiguousarray(rt, np.float32)
    hq, wq = up7.shape[1], up7.shape[2]
    ag = None if age is None else np.ascontiguousarray(age, np.float32)
    fv = np.array([fsx, fsy, min_age, sa, sb, sr], np.float32)
    iv = np.array([int(cubic), int(flags)], np.int32)
    out = np.zeros(w * h * 4, np.uint8)
    f = lambda a: a.ctypes.data_as(POINTER(c_float))
    rc = lib().or_render_tex_planes(_u8(fa), _u8(fb), w, h, f(up7), f(rt), hq, wq, f(ag) if ag is not None else None,
                                    f(fv), iv.ctypes.data_as(POINTER(c_int)), _u8(out))
    if rc != 0:
        raise RuntimeError(lib().or_error().decode())
    return out


def tex_down(frame, w, h, oh, ow):
    """tex_down.wgsl alone: the padded frame's antialiased downscale to [3][oh][ow] (B, G, R) as f16 bits."""
    f = np.ascontiguousarray(frame, np.uint8)
    out = np.zeros(3 * oh * ow, np.uint16)
    if lib().or_tex_down(_u8(f), w, h, oh, ow, out.ctypes.data_as(POINTER(c_uint16))) != 0:
        raise RuntimeError(lib().or_error().decode())
    return out.reshape(3, oh, ow)


# ---- the Stream's pair classifier (crates/flyhigh-engine/src/stream/classify.rs) ----

CLASSIFY_GRID = (48, 27)


def classify_stats(fa, fb, w, h, grid=CLASSIFY_GRID):
    """classify.wgsl on two rgba8 frames: (sum of the cells' rgb differences in 1/255 steps, the largest cell, the
    strongest coherent tile luma change)."""
    fa = np.ascontiguousarray(fa, np.uint8)
    fb = np.ascontiguousarray(fb, np.uint8)
    out = (ctypes.c_uint32 * 3)()
    if lib().or_classify(_u8(fa), _u8(fb), w, h, grid[0], grid[1], out) != 0:
        raise RuntimeError(lib().or_error().decode())
    return int(out[0]), int(out[1]), int(out[2])


class Classification:
    """classify.rs's Classification: kind, mean and max in 0..1 (f32 values), black, motion (the Pacer's units)."""

    def __init__(self, kind, mean, mx):
        self.kind, self.mean, self.max = kind, np.float32(mean), np.float32(mx)
        self.black = bool(self.max == 0.0)
        self.motion = float(np.float64(self.mean) * 765.0)

    def as_dict(self):
        return {"kind": self.kind, "mean": float(self.mean), "max": float(self.max), "black": self.black,
                "motion": self.motion}


class Thresholds:
    """classify.rs:38-49: cut_mean (None = never), hold_mean (None = no held frames), hold_max, step_after_hold."""

    def __init__(self, cut_mean=0.08, hold_mean=None, hold_max=0.0, step_after_hold=False):
        self.cut = None if cut_mean is None else np.float32(cut_mean)
        self.hold = None if hold_mean is None else np.float32(hold_mean)
        self.hold_max = np.float32(hold_max)
        self.step_after_hold = step_after_hold


CELL_MAX = np.float32(765.0)
FLASH_LUMA, FLASH_MEAN, CUT_AFTER_CALM = 32, np.float32(0.045), np.float32(0.5)


def from_stats(s, mx, cells, th):
    """classify.rs:65-80: the kind from the kernel's sums (f32 as the reference divides)."""
    mean = np.float32(np.float32(np.float32(s) / np.float32(max(cells, 1))) / CELL_MAX)
    mxf = np.float32(np.float32(mx) / CELL_MAX)
    kind = "motion"
    if th.cut is not None and mean > th.cut:
        kind = "cut"
    elif th.hold is not None and mean < th.hold and mxf < th.hold_max:
        kind = "hold"
    return Classification(kind, mean, mxf)


def after_hold(c, held_before, th):
    """classify.rs:86-91: a change right after a held frame is shown as drawn (a cut)."""
    if th.step_after_hold and held_before and c.kind == "motion":
        return Classification("cut", c.mean, c.max)
    return c


def after(c, before, th):
    """classify.rs:95-102: a cut right after a moving pair (mean >= half the threshold) is a fast camera move."""
    if c.kind == "cut" and th.cut is not None and before is not None and np.float32(before) >= th.cut * CUT_AFTER_CALM:
        return Classification("motion", c.mean, c.max)
    return c


def with_history(c, tile_luma, before, th):
    """classify.rs:104-111: a coherent brightness step (a flash) is a cut, else after()."""
    if th.cut is not None and c.mean >= FLASH_MEAN and tile_luma >= FLASH_LUMA:
        return Classification("cut", c.mean, c.max)
    return after(c, before, th)


class Classifier:
    """classify.rs's Classifier bookkeeping (begin's readback closure, :196-207): each pair's decision from the
    kernel's sums with the last moving pair's mean and whether the last pair was held."""

    def __init__(self, scene_cut=0.08, held_frames=None, cadence=False):
        h = held_frames if isinstance(held_frames, dict) else {}
        self.th = Thresholds(cut_mean=scene_cut if scene_cut else None,
                             hold_mean=(h.get("mean") or 0.0033) if held_frames else None,
                             hold_max=(h.get("max") or 0.06) if held_frames else 0.0,
                             step_after_hold=bool(held_frames) and not cadence)
        self.last_moving = None
        self.last_held = False

    def decide(self, stats, cells=CLASSIFY_GRID[0] * CLASSIFY_GRID[1]):
        s, mx, tile = stats
        c = with_history(from_stats(s, mx, cells, self.th), tile, self.last_moving, self.th)
        held = c.kind == "hold"
        if not held:
            self.last_moving = c.mean
        c = after_hold(c, self.last_held, self.th)
        self.last_held = held
        return c.as_dict()

    def forget(self):
        self.last_moving = None
        self.last_held = False


# ---- repair level 2's pan stage (crates/flyhigh-engine/src/pan.rs) ----

def pan_search(fa, fb, w, h):
    """pan_search / pan_select.wgsl over the three levels: (shift x, shift y, confidence, still error)."""
    fa = np.ascontiguousarray(fa, np.uint8)
    fb = np.ascontiguousarray(fb, np.uint8)
    fit = np.zeros(4, np.float32)
    lib().or_pan_search(_u8(fa), _u8(fb), w, h, fit.ctypes.data_as(POINTER(c_float)))
    return fit


def pan_apply(fa, fb, w, h, fit, t, frame, age=None, min_age=0.0):
    """pan_apply.wgsl on a generated rgba8 frame (a copy is returned); age: the static age plane [hp][wp] or None."""
    fa = np.ascontiguousarray(fa, np.uint8)
    fb = np.ascontiguousarray(fb, np.uint8)
    out = np.ascontiguousarray(np.asarray(frame, np.uint8).copy())
    fit = np.ascontiguousarray(fit, np.float32)
    ag = None if age is None else np.ascontiguousarray(age, np.float32)
    pitch = 0 if ag is None else ag.shape[-1]
    f = lambda a: a.ctypes.data_as(POINTER(c_float))
    lib().or_pan_apply(_u8(fa), _u8(fb), w, h, f(fit), c_float(t), f(ag) if ag is not None else None, pitch,
                       c_float(min_age), _u8(out))
    return out


# ---- the camera warp (crates/flyhigh-engine/src/warp/gpu.rs and its warp_* shaders) --------------------------------

WARP_LEVELS = ((32, 18, 12, 6, 1), (128, 72, 6, 6, 1), (512, 288, 6, 6, 2))  # grid w, h, range x, y, stride
WARP_HFOV = 106.0
WARP_LOCK_MARGIN = 6.0 / 255.0
WARP_LOCK_REL = 0.3


def _f32p(a):
    return a.ctypes.data_as(POINTER(c_float))


def warp_geometry(w, h, hfov=WARP_HFOV):
    """(focal length, half horizontal angle, half vertical angle), f32 (gpu.rs:222-226)."""
    out = np.zeros(3, np.float32)
    lib().or_warp_geometry(w, h, hfov, _f32p(out))
    return out


def warp_cells(frame, w, h, level, hfov=WARP_HFOV):
    """warp_cells.wgsl: the frame's cell grid at pyramid level `level`, [gh][gw] f32 (-1 outside the frame)."""
    gw, gh = WARP_LEVELS[level][:2]
    out = np.zeros((gh, gw), np.float32)
    lib().or_warp_cells(_u8(np.ascontiguousarray(frame, np.uint8)), w, h, level, hfov, _f32p(out))
    return out


def warp_level(level, cells_a, cells_b, w, h, coarse, mask, hfov=WARP_HFOV):
    """warp_shift / warp_refine + warp_best of one level from given grids: (sad [cand][2], best [4])."""
    rx, ry = WARP_LEVELS[level][2:4]
    sad = np.zeros(((2 * rx + 1) * (2 * ry + 1), 2), np.float32)
    bst = np.zeros(4, np.float32)
    a = np.ascontiguousarray(cells_a, np.float32)
    b = np.ascontiguousarray(cells_b, np.float32)
    c = np.ascontiguousarray(coarse, np.float32)
    m = np.ascontiguousarray(mask, np.float32)
    lib().or_warp_level(level, _f32p(a), _f32p(b), w, h, hfov, _f32p(c), _f32p(m), _f32p(sad), _f32p(bst))
    return sad, bst


def warp_measure(prev, frame, w, h, mask=None, hfov=WARP_HFOV):
    """A whole measurement of (prev, frame): (best [3][4], mask after, grown, lock score). mask: the lock mask before
    (zeros by default), [ceil(h/8)][ceil(w/8)]."""
    mgw, mgh = (w + 7) // 8, (h + 7) // 8
    m = np.zeros((mgh, mgw), np.float32) if mask is None else np.array(mask, np.float32, copy=True)
    bst = np.zeros((3, 4), np.float32)
    grown = np.zeros((mgh, mgw), np.float32)
    score = np.zeros((mgh, mgw), np.float32)
    lib().or_warp_measure(_u8(np.ascontiguousarray(prev, np.uint8)), _u8(np.ascontiguousarray(frame, np.uint8)), w, h,
                          hfov, WARP_LOCK_MARGIN, WARP_LOCK_REL, _f32p(m), _f32p(bst), _f32p(grown), _f32p(score))
    return bst, m, grown, score


def warp_lock(prev, frame, w, h, best, mask, hfov=WARP_HFOV):
    """warp_lock.wgsl on a given result: (mask after, score = e_moved - e_still - max(margin, rel * e_moved); NaN where
    the lock did not run)."""
    m = np.array(mask, np.float32, copy=True)
    score = np.zeros_like(m)
    b = np.ascontiguousarray(best, np.float32)
    lib().or_warp_lock(_u8(np.ascontiguousarray(prev, np.uint8)), _u8(np.ascontiguousarray(frame, np.uint8)), w, h,
                       hfov, _f32p(b), WARP_LOCK_MARGIN, WARP_LOCK_REL, _f32p(m), _f32p(score))
    return m, score


def warp_dilate(mask):
    m = np.ascontiguousarray(mask, np.float32)
    out = np.zeros_like(m)
    lib().or_warp_dilate(_f32p(m), m.shape[1], m.shape[0], _f32p(out))
    return out


def warp_render(src, w, h, grown, sx, sy, hfov=WARP_HFOV):
    """warp_render.wgsl: src turned by (sx, sy) px at the centre, the grown mask's blocks kept; rgba8 [h][w][4]."""
    out = np.zeros((h, w, 4), np.uint8)
    g = np.ascontiguousarray(grown, np.float32)
    lib().or_warp_render(_u8(np.ascontiguousarray(src, np.uint8)), w, h, hfov, _f32p(g), sx, sy, _u8(out))
    return out
