"""The oracle's restatement of repair level 2's pan stage (CPU only): on an exact camera pan it finds the translation
and trusts it, and the apply takes the translated pixels; on a still pair it rules the pan out (confidence -1); on
independent motion it does not trust it (pan_select.wgsl's conditions)."""
import os
import sys

import numpy as np

from oracle import oracle

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from test_gpu_stream import _pan_pair  # noqa: E402  (the frame maker only; no GPU needed)


def test_pan_finds_an_exact_translation():
    w, h = 320, 180
    for dx, dy in ((7, -3), (-6, 5)):  # within the first level's reach: 7 candidates of 1.25 px either way
        fa, fb = _pan_pair(w, h, dx, dy)
        fit = oracle.pan_search(fa, fb, w, h)
        assert fit[2] == 1.0 and abs(fit[0] + dx) < 0.5 and abs(fit[1] + dy) < 0.5, (dx, dy, fit)
        assert fit[3] > 0.016  # the zero shift did not explain the pair


def test_pan_still_pair_is_ruled_out():
    w, h = 320, 180
    fa, _ = _pan_pair(w, h, 0, 0)
    fit = oracle.pan_search(fa, fa, w, h)
    assert fit[2] == -1.0 and fit[3] == 0.0


def test_pan_apply_takes_translated_pixels():
    """At t = 0 the generated frame becomes frame a wherever frame b (shifted back) agrees with it."""
    w, h = 320, 180
    fa, fb = _pan_pair(w, h, 6, 0)
    fit = oracle.pan_search(fa, fb, w, h)
    grey = np.full((h * w * 4,), 128, np.uint8)
    out = oracle.pan_apply(fa, fb, w, h, fit, 0.0, grey).reshape(h, w, 4)
    inner = out[4:-4, 8:-8, :3].astype(np.int32)
    assert np.abs(inner - fa[4:-4, 8:-8, :3].astype(np.int32)).max() <= 1
    assert (out[..., 3] == 255).all()
