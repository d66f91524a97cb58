"""The oracle's restatement of the Stream's pair classifier (CPU only), pinned against the reference's own tests:
crates/flyhigh-engine/tests/stream.rs's pure threshold cases (classification_thresholds_are_pure) and its kernel cases
(the_classifier_tells_cuts_holds_and_motion_apart, a_local_flash_and_its_clear_frame_are_discontinuities) on the CPU
restatement of classify.wgsl."""
import numpy as np

from oracle import oracle
from oracle.oracle import CLASSIFY_GRID, Thresholds, after, after_hold, from_stats

W, H = 256, 192


def test_classification_thresholds_are_pure():
    th = Thresholds(cut_mean=0.08, hold_mean=0.0033, hold_max=0.06, step_after_hold=True)
    cells = CLASSIFY_GRID[0] * CLASSIFY_GRID[1]
    identical = from_stats(0, 0, cells, th)
    assert (identical.kind, identical.black) == ("hold", True)
    cut = from_stats(cells * 765 // 5, 765, cells, th)
    assert cut.kind == "cut"  # a mean difference of 0.2
    motion = from_stats(cells * 20, 400, cells, th)
    assert motion.kind == "motion" and abs(motion.motion - 20.0) < 0.01
    noise = from_stats(cells, 30, cells, th)
    assert noise.kind == "hold"  # codec noise on a held frame stays a hold
    off = Thresholds(cut_mean=None, hold_mean=None, hold_max=0.0, step_after_hold=False)
    assert from_stats(cells * 765, 765, cells, off).kind == "motion"
    assert after(cut, 0.02, th).kind == "cut"
    assert after(cut, None, th).kind == "cut"
    assert after(cut, 0.07, th).kind == "motion"
    assert after(motion, 0.2, th).kind == "motion"
    assert after_hold(motion, True, th).kind == "cut"
    assert after_hold(motion, False, th).kind == "motion"
    assert after_hold(noise, True, th).kind == "hold"
    assert after_hold(motion, True, off).kind == "motion"


def test_classifier_tells_cuts_holds_and_motion_apart():
    from flyhigh_engine_b200.synth_frames import sinusoid_pair
    flat = np.full((H, W, 4), 30, np.uint8)
    f0, f2 = sinusoid_pair(W, H, 0.0), sinusoid_pair(W, H, 2.0)
    cl = oracle.Classifier(held_frames=True)
    motion = cl.decide(oracle.classify_stats(f0, f2, W, H))
    hold = cl.decide(oracle.classify_stats(f0, f0, W, H))
    cut = cl.decide(oracle.classify_stats(f0, flat, W, H))
    assert motion["kind"] == "motion" and 0.0033 < motion["mean"] < 0.08 and not motion["black"]
    assert (hold["kind"], hold["black"]) == ("hold", True)
    assert cut["kind"] == "cut"


def test_a_local_flash_and_its_clear_frame_are_discontinuities():
    original = np.zeros((H, W, 4), np.uint8)
    original[..., :3], original[..., 3] = 48, 255
    flash = original.copy()
    flash[:, 3 * W // 4:, :3] = 112  # the right quarter of every row
    cl = oracle.Classifier()
    onset = cl.decide(oracle.classify_stats(original, flash, W, H))
    clear = cl.decide(oracle.classify_stats(flash, original, W, H))
    assert onset["mean"] < 0.08  # below the ordinary cut threshold
    assert (onset["kind"], clear["kind"]) == ("cut", "cut")


def test_classify_sums_of_a_uniform_step():
    """A uniform step of k levels in every channel: every cell differs by u32(3 * (k / 255) * 255), every tile changes
    its luma coherently."""
    for k in (0, 1, 17, 200):
        a = np.zeros((H, W, 4), np.uint8)
        a[..., 3] = 255
        b = a.copy()
        b[..., :3] = k
        s, mx, tile = oracle.classify_stats(a, b, W, H)
        d = np.float32(np.float32(k) / np.float32(255.0))
        cell = int(np.float32(np.float32(np.float32(d * np.float32(255.0)) + np.float32(d * np.float32(255.0)))
                              + np.float32(d * np.float32(255.0))))
        assert (s, mx) == (cell * CLASSIFY_GRID[0] * CLASSIFY_GRID[1], cell)
        assert tile == (k if k else 0)
