"""Comparison helpers of the parity tests (tolerances from the north star: per layer relative L2 <= 1e-2; final rgba8
max |diff| <= 2 / 255 and PSNR >= 50 dB)."""
import numpy as np

LAYER_REL_L2 = 1e-2
FRAME_MAX_ABS = 2
FRAME_PSNR_DB = 50.0


def rel_l2(x, ref):
    x = np.asarray(x, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.linalg.norm(ref)
    num = np.linalg.norm(x - ref)
    return float(num / den) if den > 0 else float(num)


def psnr(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    mse = np.mean((a - b) ** 2)
    return float("inf") if mse == 0 else float(10 * np.log10(255.0 ** 2 / mse))


def frame_stats(got, ref):
    g = np.asarray(got, np.int32).reshape(-1, 4)[:, :3]
    r = np.asarray(ref, np.int32).reshape(-1, 4)[:, :3]
    return int(np.abs(g - r).max()), psnr(g, r)
