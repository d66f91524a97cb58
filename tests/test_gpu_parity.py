"""GPU parity: the CUDA path (through the C ABI) against the CPU oracle on the same seeded inputs and weights.

Tolerances (the north star's): every network layer within 1e-2 relative L2 of the oracle's tensor; final rgba8 frames
with max |diff| <= 2 levels and PSNR >= 50 dB.

The path has stages that turn continuous values into decisions: the GMHS repair's cost-margin selection, the
render's still test (a 1 / 0.04 ramp on |warped A - warped B|) and its static rules (1-px probes of the age plane).
The f32 accumulation order of the tensor-core convs differs from the oracle's, which moves the network outputs by a few
f16 ulps (~1e-3 relative); at a few pixels that is enough to switch a decision or, at a steep edge, to move a bicubic
sample by more than 2 levels. So:
  - each decision stage is checked on identical inputs (the oracle's own flow for GMHS, the GPU's own network
    outputs for the render): bit for bit, resp. max |diff| <= 1 level everywhere;
  - every end-to-end frame of the exact render goes through tests/frame_parity.check_frame: PSNR >= 50 dB, the render
    within 1 level of the oracle's render of the GPU's own network outputs, and each pixel beyond 2 levels explained
    by a threshold or a steep edge of the render in the oracle's run, none unexplained; flow_tq within 0.05 px L1 (the
    reference's own backend check, crates/flyhigh-cli/src/cli/selftest.rs:132-151);
  - the fast render's frames: PSNR >= 50 dB with at most 1e-3 of the channels beyond 2 levels (_frame_ok);
  - the integer static-protection state is checked exactly after every pair.
"""
import ctypes
from ctypes import POINTER, Structure, c_float, c_int, c_longlong, c_void_p

import numpy as np
import pytest

from tests.frame_parity import check_frame, flipped_cells, gmhs_records, layer_rel_l2
from tests.parity import FRAME_MAX_ABS, FRAME_PSNR_DB, LAYER_REL_L2, frame_stats, rel_l2

pytestmark = pytest.mark.gpu


class ConvSrc(Structure):  # include/flyhigh_kernels.h FhConvSrc
    _fields_ = [("p", c_void_p), ("bs", c_longlong), ("cs", c_int), ("nc", c_int), ("scale", c_float), ("slot", c_int)]


class ConvParams(Structure):
    _fields_ = [("src", ConvSrc * 6), ("nsrc", c_int), ("h", c_int), ("w", c_int), ("ho", c_int), ("wo", c_int),
                ("cp", c_int), ("cout", c_int), ("wpack", c_void_p), ("bias", c_void_p), ("slope", c_void_p),
                ("epi", c_int), ("out", c_void_p), ("out_cs", c_int), ("out_bs", c_longlong), ("res", c_void_p),
                ("res_cs", c_int), ("res_bs", c_longlong), ("n", c_int), ("wm", c_int), ("ngroups", c_int),
                ("wsmem", c_int), ("wait_cycles", c_longlong), ("test_extra_tx", c_int)]


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _up8(c):
    return (c + 7) // 8 * 8


def run_conv(torch, x_chw, w, bias, slope, stride, resid_chw=None, wm=0, ngroups=0, wait_cycles=0, extra_tx=0,
             umma=False, pad_fill=0.0):
    """One conv through fhk_conv3x3 on NHWC device buffers; returns CHW f16. pad_fill: the value of the input's
    channels past cin (the pixel pitch rounds cin up to 8, or 4)."""
    import flyhigh_engine_b200 as fh
    L = fh.lib()
    cin, h, wd = x_chw.shape
    cout = w.shape[0]
    cs = 4 if cin <= 4 else _up8(cin)
    ho, wo = (h - 1) // stride + 1, (wd - 1) // stride + 1
    x = torch.full((h, wd, cs), pad_fill, dtype=torch.float16)
    x[:, :, :cin] = torch.from_numpy(np.ascontiguousarray(x_chw.transpose(1, 2, 0)))
    x = x.cuda()
    cp = (_up8(cin) + 15) // 16 * 16
    cmap = np.full(cp, -1, np.int32)
    cmap[:cin] = np.arange(cin)
    n_pack = L.fhk_conv_packed_elems_umma(cout, cp) if umma else L.fhk_conv_packed_elems(cout, cp)
    packed = np.zeros(n_pack, np.uint16)
    wbits = np.ascontiguousarray(w.astype(np.float16)).view(np.uint16)
    pack = L.fhk_conv_pack_weights_umma if umma else L.fhk_conv_pack_weights
    assert pack(wbits.ctypes.data, cin, cout, cmap.ctypes.data, cp, packed.ctypes.data) == 0
    wp = torch.from_numpy(packed.view(np.int16)).cuda()
    b = torch.from_numpy(bias.astype(np.float32)).cuda()
    s = torch.from_numpy(slope.astype(np.float32)).cuda() if slope is not None else None
    ocs = _up8(cout)
    out = torch.zeros((ho, wo, ocs), dtype=torch.float16, device="cuda")
    r = None
    if resid_chw is not None:
        r = torch.zeros((ho, wo, ocs), dtype=torch.float16)
        r[:, :, :cout] = torch.from_numpy(np.ascontiguousarray(resid_chw.transpose(1, 2, 0)))
        r = r.cuda()
    p = ConvParams()
    p.src[0] = ConvSrc(x.data_ptr(), 0, cs, cin, 1.0, 0)
    p.nsrc, p.h, p.w, p.ho, p.wo, p.cp, p.cout = 1, h, wd, ho, wo, cp, cout
    p.wpack, p.bias, p.slope = wp.data_ptr(), b.data_ptr(), (s.data_ptr() if s is not None else None)
    p.epi, p.out, p.out_cs, p.out_bs = 0, out.data_ptr(), ocs, 0
    p.res, p.res_cs, p.res_bs, p.n = (r.data_ptr() if r is not None else None), ocs, 0, 1
    p.wm, p.ngroups, p.wait_cycles, p.test_extra_tx = wm, ngroups, wait_cycles, extra_tx
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = L.fhk_conv3x3_umma(ctypes.byref(p), st) if umma else L.fhk_conv3x3(ctypes.byref(p), stride, st)
    assert rc == 0, rc
    torch.cuda.synchronize()
    return out[:, :, :cout].permute(2, 0, 1).cpu().numpy()


# config 1: fp16 activations ~N(0,1), weights ~N(0, 1/sqrt(9 cin)), bias + leaky ReLU(0.1), with and
# without a residual; the model's own shapes at their network sizes
CONV_CASES = [
    # (h, w, cin, cout, stride, residual)
    (270, 480, 16, 16, 1, False),
    (270, 480, 32, 64, 2, False),
    (270, 480, 64, 64, 1, True),
    (270, 480, 48, 32, 2, True),
    (540, 960, 16, 32, 1, False),
    (120, 216, 3, 36, 2, False),
    (60, 108, 36, 36, 1, True),
    (60, 108, 36, 72, 2, False),
    (30, 54, 72, 72, 1, True),
    (30, 54, 279, 96, 1, False),
    (30, 54, 96, 12, 1, False),
    (60, 108, 155, 48, 1, False),
    (60, 108, 48, 7, 1, True),
    (60, 108, 48, 36, 1, False),
    (120, 216, 14, 24, 1, False),
    (120, 216, 24, 3, 1, False),
    (37, 29, 24, 24, 1, True),  # ragged: partial tiles in both directions
    (24, 40, 400, 40, 1, True),  # a weight slice streamed through the ring in many chunks
]


@pytest.mark.parametrize("h,w,cin,cout,stride,res", CONV_CASES)
@pytest.mark.parametrize("split", [(0, 0), (1, 2), (4, 1), (2, 1)])
def test_conv_matches_oracle(torch_cuda, h, w, cin, cout, stride, res, split):
    from oracle import oracle
    rng = np.random.default_rng(h * 1000 + cin * 10 + cout + stride)
    x = rng.standard_normal((cin, h, w)).astype(np.float16)
    wt = (rng.standard_normal((cout, cin, 3, 3)) / np.sqrt(9 * cin)).astype(np.float16).astype(np.float32)
    bias = rng.standard_normal(cout).astype(np.float16).astype(np.float32) * 0.1
    slope = np.full(cout, 0.1, np.float32)
    ho, wo = (h - 1) // stride + 1, (w - 1) // stride + 1
    resid = rng.standard_normal((cout, ho, wo)).astype(np.float16) if res else None
    ref = oracle.conv(x, wt, bias, slope, stride, resid).astype(np.float32)
    wm, ng = split
    ng = min(ng, (cout + 7) // 8)
    got = run_conv(torch_cuda, x, wt, bias, slope, stride, resid, wm, ng).astype(np.float32)
    assert got.shape == ref.shape
    assert rel_l2(got, ref) < 2e-3
    # f32 accumulation order differs from the oracle's: a few f16 ulps at most
    assert np.abs(got - ref).max() <= 4e-3 * max(1.0, np.abs(ref).max())


@pytest.mark.parametrize("cin,stride", [(155, 1), (14, 1), (3, 2), (36, 2), (279, 1)])
@pytest.mark.parametrize("kernel", ["mma", "umma", "umma_persistent"])
def test_conv_never_reads_padding_channels(torch_cuda, cin, stride, kernel):
    """The channels past cin in an input pixel (its pitch rounds cin up to 8, or 4) hold NaN here: the halo copies read
    only the valid channels of a partial 8-channel chunk and zero-fill the rest, so the output equals the one with
    zeros there, bit for bit (a NaN read would reach every output through its zero weight)."""
    import flyhigh_engine_b200 as fh
    umma = kernel != "mma"
    wm = 1 if kernel == "umma_persistent" else 0
    cp = (_up8(cin) + 15) // 16 * 16
    if umma and (stride != 1 or not fh.lib().fhk_conv_umma_fits(cp, 48, 1)):
        pytest.skip("the tcgen05 kernel takes stride 1 only")
    if wm == 1 and not fh.lib().fhk_conv_umma_persistent_fits(cp, 48):
        pytest.skip("no persistent variant for this shape")
    rng = np.random.default_rng(cin * 7 + stride)
    h, w, cout = 60, 108, 48
    x = rng.standard_normal((cin, h, w)).astype(np.float16)
    wt = (rng.standard_normal((cout, cin, 3, 3)) / np.sqrt(9 * cin)).astype(np.float16).astype(np.float32)
    bias = rng.standard_normal(cout).astype(np.float16).astype(np.float32) * 0.1
    slope = np.full(cout, 0.1, np.float32)
    ref = run_conv(torch_cuda, x, wt, bias, slope, stride, wm=wm, umma=umma, pad_fill=0.0)
    got = run_conv(torch_cuda, x, wt, bias, slope, stride, wm=wm, umma=umma, pad_fill=float("nan"))
    assert np.isfinite(got).all()
    assert np.array_equal(got.view(np.uint16), ref.view(np.uint16))


UMMA_CASES = [c for c in CONV_CASES if c[4] == 1] + [(30, 54, 96, 96, 1, True), (120, 216, 24, 24, 1, True)]


@pytest.mark.parametrize("h,w,cin,cout,stride,res", UMMA_CASES)
@pytest.mark.parametrize("wm", [0, 1])
def test_conv_umma_matches_oracle(torch_cuda, h, w, cin, cout, stride, res, wm):
    """The tcgen05 kernel (wm 1: its persistent variant) on the stride-1 shapes that fit it, against the oracle (f32
    accumulation in another order: a few f16 ulps at most)."""
    import flyhigh_engine_b200 as fh
    from oracle import oracle
    cp = (_up8(cin) + 15) // 16 * 16
    if not fh.lib().fhk_conv_umma_fits(cp, cout, 1):
        pytest.skip("weights and halo tile exceed shared memory: conv3x3_mma takes this layer")
    if wm == 1 and not fh.lib().fhk_conv_umma_persistent_fits(cp, cout):
        pytest.skip("two halo buffers and the weights exceed shared memory: no persistent variant")
    rng = np.random.default_rng(h * 1000 + cin * 10 + cout + 7)
    x = rng.standard_normal((cin, h, w)).astype(np.float16)
    wt = (rng.standard_normal((cout, cin, 3, 3)) / np.sqrt(9 * cin)).astype(np.float16).astype(np.float32)
    bias = rng.standard_normal(cout).astype(np.float16).astype(np.float32) * 0.1
    slope = np.full(cout, 0.1, np.float32)
    resid = rng.standard_normal((cout, h, w)).astype(np.float16) if res else None
    ref = oracle.conv(x, wt, bias, slope, 1, resid).astype(np.float32)
    got = run_conv(torch_cuda, x, wt, bias, slope, 1, resid, wm=wm, umma=True).astype(np.float32)
    assert rel_l2(got, ref) < 2e-3
    assert np.abs(got - ref).max() <= 4e-3 * max(1.0, np.abs(ref).max())
    assert fh.lib().fhk_conv_wait_timeouts(0) == 0


@pytest.mark.parametrize("h,w,cin,cout,res", [(60, 108, 48, 48, False), (60, 108, 48, 7, True), (37, 29, 24, 24, True),
                                              (30, 54, 96, 96, True), (120, 216, 14, 24, False), (17, 9, 3, 36, False),
                                              (60, 108, 155, 48, False)])
def test_conv_umma_persistent_is_bit_exact(torch_cuda, h, w, cin, cout, res):
    """The persistent variant (a CTA looping over tiles, accumulators double-buffered, the halo too where two buffers
    fit beside the weights: 155 -> 48 has one) gives the bytes of the one-tile-per-CTA kernel, over a batch of 5
    entries (tiles of several entries per CTA)."""
    import flyhigh_engine_b200 as fh
    from flyhigh_engine_b200.kernels import Conv3x3
    torch = torch_cuda
    cp = (_up8(cin) + 15) // 16 * 16
    if not fh.lib().fhk_conv_umma_persistent_fits(cp, cout):
        pytest.skip("no persistent variant for this shape")
    rng = np.random.default_rng(cin * 31 + cout)
    cs = 4 if cin <= 4 else _up8(cin)
    x = torch.zeros((5, h, w, cs), dtype=torch.float16)
    x[..., :cin] = torch.from_numpy(rng.standard_normal((5, h, w, cin)).astype(np.float16))
    x = x.cuda()
    wt = (rng.standard_normal((cout, cin, 3, 3)) / np.sqrt(9 * cin)).astype(np.float32)
    bias = (0.1 * rng.standard_normal(cout)).astype(np.float32)
    slope = np.full(cout, 0.1, np.float32)
    outs = []
    for wm in (0, 1):
        conv = Conv3x3(wt, bias, slope, kernel="umma", wm=wm)
        r = None
        if res:
            torch.manual_seed(3)
            r = torch.randn(conv.out_shape(5, h, w), dtype=torch.float16, device="cuda")
        outs.append(conv(x, r).cpu().numpy())
    assert np.array_equal(outs[0].view(np.uint16), outs[1].view(np.uint16))
    assert fh.lib().fhk_conv_wait_timeouts(0) == 0


@pytest.mark.parametrize("h,w,cin,cout,umma,wm", [(60, 108, 48, 48, False, 0), (30, 54, 279, 96, False, 0),
                                                  (60, 108, 48, 48, True, 0), (60, 108, 48, 48, True, 1),
                                                  (30, 54, 279, 96, True, 0)])
def test_conv_weight_wait_runs_out(torch_cuda, h, w, cin, cout, umma, wm):
    """Failure detection without a fault: the weight staging's mbarrier is made to expect 16 bytes that no copy brings
    (whole slice: 48 -> 48; streamed ring: 279 -> 96, on both kernels), so every wait runs out after its bound; the
    kernel counts the timeouts, finishes and leaves the context usable, and the next normal launch is exact again."""
    import flyhigh_engine_b200 as fh
    from oracle import oracle
    L = fh.lib()
    rng = np.random.default_rng(5)
    x = rng.standard_normal((cin, h, w)).astype(np.float16)
    wt = (rng.standard_normal((cout, cin, 3, 3)) / np.sqrt(9 * cin)).astype(np.float16).astype(np.float32)
    bias = np.zeros(cout, np.float32)
    slope = np.full(cout, 0.1, np.float32)
    assert L.fhk_conv_wait_timeouts(1) >= 0
    run_conv(torch_cuda, x, wt, bias, slope, 1, wm=wm, wait_cycles=200000, extra_tx=16, umma=umma)
    assert L.fhk_conv_wait_timeouts(1) > 0
    got = run_conv(torch_cuda, x, wt, bias, slope, 1, wm=wm, umma=umma).astype(np.float32)
    assert L.fhk_conv_wait_timeouts(0) == 0
    ref = oracle.conv(x, wt, bias, slope, 1).astype(np.float32)
    assert rel_l2(got, ref) < 2e-3


def _session_pair(model_dir, w, h, frames, t=0.5, check_age=False, mask=None, **opts):
    """(gpu session, oracle session, [(gpu frame, oracle frame, frame report)], keep-alive) after the same pairs;
    frames is a list of (a, b). Each frame report is tests/frame_parity.check_frame's; with the repair stage on, a
    second session without it yields the GPU's pre-repair flow, from which the oracle tells the GPU run's repair
    decisions. check_age: the age plane equals the oracle's after every pair; mask: a protection mask for both."""
    import flyhigh_engine_b200 as fh
    from oracle.oracle import OracleModel, OracleSession
    still = opts.pop("still", True)
    eng = fh.Engine()
    model = fh.Model(model_dir)
    s = fh.Session(eng, model, w, h, **opts)
    a, b, out = s.add_input(), s.add_input(), s.add_output()
    s0 = fh.Session(eng, model, w, h, **dict(opts, repair=0)) if opts.get("repair", 1) > 0 else None
    a0, b0 = (s0.add_input(), s0.add_input()) if s0 else (None, None)
    pp = model.plan_params(w, h, **opts)
    om = OracleModel(model_dir)
    okw = dict(k=opts.get("k", 1), repair=opts.get("repair", 1), still=still,
               cubic={"model": -1, "bilinear": 0, "bicubic": 1}[opts.get("render", "model")],
               keep_static=opts.get("static_protection", True) is not False,
               protection_mask=opts.get("protection_mask", False), fast_render=opts.get("fast_render", False),
               linear_t=opts.get("linear_t", False))
    if isinstance(opts.get("internal"), tuple):
        okw["internal"] = opts["internal"]
    o = OracleSession(om, w, h, **okw)
    if mask is not None:
        for x in (s, s0):
            if x:
                x.write_mask(mask)
        o.write_mask(mask)
    results = []
    for i, (fa, fb) in enumerate(frames):
        s.write(a, fa)
        s.write(b, fb)
        s.pair(a, b)
        s.mid(t, out)
        got = np.frombuffer(s.read(out), np.uint8)
        o.pair(fa, fb)
        ref = o.mid(t)
        gm = None
        if s0:
            s0.write(a0, fa)
            s0.write(b0, fb)
            s0.pair(a0, b0)
            gm = gmhs_records(o, s0.tensor("flow"))
        age = s.tensor("age") if pp["protects"] else None
        if check_age:
            assert np.array_equal(age, o.tensor("age")), f"age differs after pair {i + 1}"
        rep = check_frame(got, ref, fa, fb, w, h, pp, (s.tensor("up7"), s.tensor("R_t")),
                          (o.tensor("up7", 1), o.tensor("R_t", 1)), age, gm)
        rep["flipped"] = flipped_cells(gm)  # the repair cells decided differently (for the layer checks)
        results.append((got, ref, rep))
    return s, o, results, (eng, model, om, s0)


PAIR_LAYERS = ["A", "B", "aq", "bq", "i8a", "i8b", "i16a", "i16b", "f8a", "f8b", "f16a", "f16b", "cv", "ch1", "ch2",
               "ch3r", "hc", "o", "wa", "wb", "ia", "ib", "fcv", "fr1", "fr2", "fr3", "flow", "vis"]
MID_LAYERS = ["hm", "fh1", "fh2", "dfilm", "ft_vt", "up7", "rx", "rq1", "rq2", "rq3", "R_t"]


def _check_layers(s, o, names, stage, tol=LAYER_REL_L2, flipped=None):
    """Each layer within tol relative L2 of the oracle's; a layer after the repair stage leaves out what the repair
    cells in `flipped` (decided differently by the two runs, at a threshold) reach."""
    worst = {}
    h8 = s.tensor("flow").shape[1]
    fl = np.zeros((0, 2), np.int64) if flipped is None else flipped
    for n in names:
        got = s.tensor(n)
        ref = o.tensor(n, stage)
        assert got.shape == ref.shape, (n, got.shape, ref.shape)
        worst[n] = layer_rel_l2(n, got, ref, fl, h8)
    bad = {k: v for k, v in worst.items() if v > tol}
    assert not bad, f"layers above {tol}: {bad} (all: {worst})"
    return worst


def test_session_c0_layers_and_frame(synth_model_dir):
    """Config 0: 640 x 360 (internal = frame), pair(a, b) + mid(0.5); every layer and the final frame."""
    from flyhigh_engine_b200 import synth_frames
    fa, fb, _ = synth_frames.pair_c0(640, 360, seed=0)
    s, o, res, _keep = _session_pair(synth_model_dir, 640, 360, [(fa, fb)])
    _check_layers(s, o, PAIR_LAYERS, 0, flipped=res[0][2]["flipped"])
    _check_layers(s, o, MID_LAYERS, 1, flipped=res[0][2]["flipped"])
    got, ref, rep = res[0]
    mx, p = frame_stats(got, ref)
    assert mx <= FRAME_MAX_ABS and p >= FRAME_PSNR_DB, (mx, p)
    assert rep["ok"], rep


def _flow_tq_l1(s, o):
    """Mean |flow_tq difference| in quarter-resolution px (the reference's selftest bound is 0.05 px)."""
    return float(np.abs(s.tensor("up7")[:4] - o.tensor("up7", 1)[:4]).mean())


def test_session_1080p_frame(synth_model_dir, monkeypatch):
    """Config 2's size: 1920 x 1080 (internal 856 x 480 -> 864 x 480), two intervals, in the reference's own parity
    configuration (NetOpts::new: no static protection, no still test; FH_STILL=0 as options.rs:296-298 reads it)
    with the repair stage off (it has its own exact test)."""
    from flyhigh_engine_b200 import synth_frames
    monkeypatch.setenv("FH_STILL", "0")
    frames = synth_frames.sequence_c2(3, 1920, 1080, seed=1)
    s, o, res, _keep = _session_pair(synth_model_dir, 1920, 1080, [(frames[0], frames[1]), (frames[1], frames[2])],
                                     static_protection=False, still=False, repair=0)
    _check_layers(s, o, ["A", "aq", "f16a", "ch1", "o", "fr3", "flow", "vis"], 0)
    _check_layers(s, o, MID_LAYERS, 1)
    assert _flow_tq_l1(s, o) <= 0.05
    for _got, _ref, rep in res:
        assert rep["ok"], rep


def _frame_ok(got, ref, keep=None):
    """The fast render's end-to-end criterion (its own render has no decision record in the oracle): PSNR >= 50 dB and
    at most 1e-3 of the channels beyond 2 levels, over the pixels `keep` (default all: the ones no repair cell flipped
    at a threshold reaches); returns (ok, (PSNR, fraction beyond 2 levels, max |diff|)). The fast render on identical
    inputs is checked to 1 level separately; the exact render's frames go through check_frame."""
    g = np.asarray(got, np.int32).reshape(-1, 4)[:, :3]
    r = np.asarray(ref, np.int32).reshape(-1, 4)[:, :3]
    if keep is not None:
        g, r = g[keep.reshape(-1)], r[keep.reshape(-1)]
    over = float((np.abs(g - r) > FRAME_MAX_ABS).mean())
    mx = int(np.abs(g - r).max())
    mse = float(((g - r).astype(np.float64) ** 2).mean())
    p = float("inf") if mse == 0 else 10 * np.log10(255.0 ** 2 / mse)
    return p >= FRAME_PSNR_DB and over <= 1e-3, (p, over, mx)


def test_session_1080p_default_options(synth_model_dir):
    """The same at the Session defaults (static protection and the still test on): exact static-age state."""
    from flyhigh_engine_b200 import synth_frames
    frames = synth_frames.sequence_c2(3, 1920, 1080, seed=1)
    s, o, res, _keep = _session_pair(synth_model_dir, 1920, 1080, [(frames[0], frames[1]), (frames[1], frames[2])])
    _check_layers(s, o, ["o", "fr1", "fr3"], 0)  # the layers before the repair stage
    assert np.array_equal(s.tensor("age"), o.tensor("age"))
    for _got, _ref, rep in res:
        assert rep["ok"], rep


def test_static_protection_sequence(synth_model_dir):
    """Static protection over 12 consecutive pairs of a sequence with a fixed HUD: the age state machine matches
    exactly after every pair, and every generated frame passes the frame check."""
    from flyhigh_engine_b200 import synth_frames
    frames = synth_frames.sequence_c2(13, 640, 360, seed=2)
    s, o, res, _keep = _session_pair(synth_model_dir, 640, 360, list(zip(frames[:-1], frames[1:])),
                                     check_age=True)
    for i, (_got, _ref, rep) in enumerate(res):
        assert rep["ok"], (i, rep)
    assert int((s.tensor("age") >= 8).sum()) > 1000, "the HUD should be protected after 8+ pairs"


@pytest.mark.parametrize("opts", [
    dict(k=2), dict(k=3, repair=0), dict(repair=2), dict(render="bilinear"), dict(static_protection=False),
    dict(internal=(320, 192)),
])
def test_session_options(synth_model_dir, opts):
    from flyhigh_engine_b200 import synth_frames
    fa, fb, _ = synth_frames.pair_c0(640, 360, seed=3)
    s, o, res, _keep = _session_pair(synth_model_dir, 640, 360, [(fa, fb)], t=0.25, **opts)
    _check_layers(s, o, ["o", "fr3"], 0)
    assert res[0][2]["ok"], (opts, res[0][2])


def test_odd_size_and_mask(synth_model_dir):
    """A frame size that is not a multiple of 32 (replicate padding) and the host's protection mask."""
    from flyhigh_engine_b200 import synth_frames
    w, h = 333, 197
    fa, fb, _ = synth_frames.pair_c0(w, h, seed=4)
    mask = np.zeros((h, w), np.uint8)
    mask[150:180, 20:120] = 1
    s, o, res, _keep = _session_pair(synth_model_dir, w, h, [(fa, fb)], check_age=True, mask=mask,
                                     protection_mask=True)
    got, _ref, rep = res[0]
    assert rep["ok"], rep
    # masked pixels take the sources' mean (keep_static apply at age 255)
    g = got.reshape(h, w, 4)[155:175, 30:110, :3].astype(np.int32)
    src = (fa.astype(np.int32) + fb.astype(np.int32))[155:175, 30:110, :3] / 2.0
    assert np.abs(g - src).max() <= 1.0


def test_pipelined_host_io_matches_sequential(synth_model_dir):
    """Host uploads and readbacks run on their own streams. The reference call sequence with a lagging readback (two
    output slots, each read while the next interval runs) and one reused pinned upload buffer (write_rgba returns
    once the buffer has been copied) gives bit-identical frames to the plain write / pair / mid / read loop, static
    protection state included."""
    import torch
    import flyhigh_engine_b200 as fh
    from flyhigh_engine_b200 import synth_frames
    w, h, n = 320, 192, 7
    frames = synth_frames.sequence_c2(n, w, h, seed=3)
    model = fh.Model(synth_model_dir)

    def run(pipelined):
        s = fh.Session(fh.Engine(), model, w, h)
        ins, outs = [s.add_input(), s.add_input()], [s.add_output(), s.add_output()]
        up = torch.empty((h, w, 4), dtype=torch.uint8).pin_memory()
        up_np = up.numpy()
        got, prev = [], None
        up_np[:] = frames[0]
        s.write(ins[0], up_np)
        for i in range(1, n):
            up_np[:] = frames[i]  # reused right after the previous write returned
            s.write(ins[i % 2], up_np)
            s.pair(ins[(i - 1) % 2], ins[i % 2])
            o = outs[i % 2] if pipelined else outs[0]
            s.mid(0.5, o)
            if not pipelined:
                got.append(np.frombuffer(s.read(o), np.uint8).copy())
                continue
            if prev is not None:
                got.append(np.frombuffer(s.read(prev), np.uint8).copy())
            prev = o
        if pipelined:
            got.append(np.frombuffer(s.read(prev), np.uint8).copy())
        return got

    a, b = run(False), run(True)
    assert len(a) == len(b) == n - 1
    for i, (x, y) in enumerate(zip(a, b)):
        assert np.array_equal(x, y), i


@pytest.mark.parametrize("batch,size,opts", [(4, (320, 192), {}), (3, (384, 160), dict(repair=2, k=2)),
                                             (4, (1920, 1080), {})])
def test_batched_session_matches_single(synth_model_dir, batch, size, opts):
    """A batched session (pair / mid calls queued, `batch` chained intervals per launch) gives bit-identical frames
    and static-protection state whether its intervals run `batch` at a time (reads at the end) or one at a time (a read
    after every mid runs the queued interval alone): full batches, a partial queue run by a read, and a further mid of
    the newest interval after a batch. The one-interval session is checked against the oracle elsewhere; a batched
    session runs its stride-1 convs on the tcgen05 kernel (another f32 summation order), so it is compared to itself."""
    import flyhigh_engine_b200 as fh
    from flyhigh_engine_b200 import synth_frames
    w, h = size
    model = fh.Model(synth_model_dir)
    frames = synth_frames.sequence_c2(2 * batch + 2, w, h, seed=11)

    def run(n, read_each):
        s = fh.Session(fh.Engine(), model, w, h, batch=batch, **opts)
        ins = [s.add_input(), s.add_input()]
        outs = [s.add_output() for _ in range(n)]
        got = {}
        s.write(ins[0], frames[0])
        for i in range(1, n):
            s.write(ins[i % 2], frames[i])
            s.pair(ins[(i - 1) % 2], ins[i % 2])
            s.mid(0.25 + 0.5 * (i % 2), outs[i])
            if read_each:
                got[i] = np.frombuffer(s.read(outs[i]), np.uint8).copy()
        for i in range(1, n):
            if i not in got:
                got[i] = np.frombuffer(s.read(outs[i]), np.uint8).copy()
        extra = s.add_output()
        s.mid(0.75, extra)  # a further mid of the newest pair
        return [got[i] for i in range(1, n)] + [np.frombuffer(s.read(extra), np.uint8).copy()], s.tensor("age")

    # 2 * batch intervals: two full batches, then a mid of the newest one; one more: a partial queue run by a read
    for n in (2 * batch + 1, 2 * batch + 2):
        single, age1 = run(n, True)
        batched, ageb = run(n, False)
        for i, (x, y) in enumerate(zip(single, batched)):
            assert np.array_equal(x, y), (n, i)
        assert np.array_equal(age1, ageb), n


@pytest.mark.parametrize("sets,size,n", [(2, (384, 160), 11), (3, (384, 160), 14), (3, (1920, 1080), 14)])
def test_batch_streams_match_one_stream_and_count_launches(synth_model_dir, monkeypatch, sets, size, n):
    """A batched session runs each batch as four graphs on streams of their own, so that consecutive batches overlap
    (the frame stage, the static pass, the network, the render), over `sets` render sets (FH_SETS; three keep one more
    batch in flight). The frames and the static state must not depend on that: the same intervals with every batch
    serialised on the session stream (FH_OVERLAP=0, read when the session is built) give the same bytes, at a small
    size and at the benchmarked one. fh_session_kernel_launches counts the session's kernels: the same calls launch
    the same number, the same on both schedules."""
    import flyhigh_engine_b200 as fh
    from flyhigh_engine_b200 import synth_frames
    (w, h), batch = size, 4
    model = fh.Model(synth_model_dir)
    frames = synth_frames.sequence_c2(n, w, h, seed=23)
    monkeypatch.setenv("FH_SETS", str(sets))

    def run(overlap):
        monkeypatch.setenv("FH_OVERLAP", "1" if overlap else "0")
        s = fh.Session(fh.Engine(), model, w, h, batch=batch)
        ins = [s.add_input(), s.add_input()]
        outs = [s.add_output() for _ in range(n - 1)]
        k0 = s.kernel_launches()
        s.write(ins[0], frames[0])
        for i in range(1, n):
            s.write(ins[i % 2], frames[i])
            s.pair(ins[(i - 1) % 2], ins[i % 2])
            s.mid(0.5, outs[i - 1])
        got = [np.frombuffer(s.read(o), np.uint8).copy() for o in outs]
        s.join()
        return got, s.tensor("age"), s.kernel_launches() - k0

    a, age_a, ka = run(True)
    b, age_b, kb = run(False)
    for i, (x, y) in enumerate(zip(a, b)):
        assert np.array_equal(x, y), i
    assert np.array_equal(age_a, age_b)
    assert ka == kb and ka > 2 * 40, (ka, kb)


def test_batch_profile(synth_model_dir):
    """fh_session_profile_batch_json: one batch's kernels timed eagerly, each stage once (the frame stage for all
    batch + 1 frames in one launch per kernel); refused for a one-interval session and before any batch ran."""
    import flyhigh_engine_b200 as fh
    from flyhigh_engine_b200 import synth_frames
    w, h, batch = 384, 160, 4
    model = fh.Model(synth_model_dir)
    frames = synth_frames.sequence_c2(batch + 1, w, h, seed=5)
    one = fh.Session(fh.Engine(), model, w, h)
    with pytest.raises(fh.FlyHighError, match="not a batched session"):
        one.profile_batch()
    s = fh.Session(fh.Engine(), model, w, h, batch=batch)
    ins = [s.add_input(), s.add_input()]
    outs = [s.add_output() for _ in range(batch)]
    with pytest.raises(fh.FlyHighError, match="no batch has run"):
        s.profile_batch()
    s.write(ins[0], frames[0])
    for i in range(1, batch + 1):
        s.write(ins[i % 2], frames[i])
        s.pair(ins[(i - 1) % 2], ins[i % 2])
        s.mid(0.5, outs[i - 1])
    first = np.frombuffer(s.read(outs[0]), np.uint8).copy()
    prof = s.profile_batch()
    names = [k["kernel"] for k in prof]
    for k in ("frame_to_input", "input_pyramid", "pair_planes", "static_age", "render", "mid_combine"):
        assert names.count(k) == 1, (k, names)
    assert sum(1 for k in names if k.startswith("conv ")) >= 20
    assert all(k["ms"] >= 0 for k in prof) and sum(k["ms"] for k in prof) > 0
    # the profile rewrites the arena, not the output slots the batch already filled
    assert np.array_equal(first, np.frombuffer(s.read(outs[0]), np.uint8))


def test_errors_and_reports(synth_model_dir):
    """The C ABI's error behaviour (core.rs): -1 / NULL with fh_last_error, never a crash."""
    import flyhigh_engine_b200 as fh
    eng = fh.Engine()
    info = eng.info()
    assert info["class"] == "tc-f16" and info["sm"].startswith("10.")
    model = fh.Model(synth_model_dir)
    s = fh.Session(eng, model, 256, 192)
    with pytest.raises(fh.FlyHighError, match="pair two input slots first"):
        s.add_output()
        s.mid(0.5, 0)
    with pytest.raises(fh.FlyHighError, match="bad input slot"):
        s.pair(0, 1)
    a, b = s.add_input(), s.add_input()
    with pytest.raises(fh.FlyHighError, match="bytes"):
        s.write(a, b"\x00" * 10)
    with pytest.raises(fh.FlyHighError, match="bad output slot"):
        s.pair(a, b)
        s.mid(0.5, 7)
    s.warm_up()
    r = s.report()
    assert r["pair_steps"] > 10 and r["mid_steps"] > 5 and r["inputs"] == 2 and r["outputs"] == 1
    assert s.pair_timed(a, b) > 0 and s.mid_timed(0.5, 0) > 0
    with pytest.raises(fh.FlyHighError, match="k"):
        fh.Session(eng, model, 256, 192, k=4)
    with pytest.raises(fh.FlyHighError, match="64x64"):
        fh.Session(eng, model, 32, 32)
    assert eng.report()["tensor_bytes"] > 0


@pytest.mark.parametrize("size,opts", [((1920, 1080), {}), ((333, 197), dict(protection_mask=True)),
                                       ((640, 360), dict(render="bilinear"))])
def test_render_on_identical_inputs(synth_model_dir, size, opts):
    """The fused full-resolution render (render.wgsl + its static variant, keep_static apply, rgba out) against the
    oracle's on the GPU's own network outputs (up7, R_t, age): the still test and the static rules see identical
    inputs, so the frames agree to within one level everywhere."""
    import flyhigh_engine_b200 as fh
    from flyhigh_engine_b200 import synth_frames
    from oracle import oracle
    w, h = size
    frames = synth_frames.sequence_c2(10, w, h, seed=5)
    eng = fh.Engine()
    model = fh.Model(synth_model_dir)
    s = fh.Session(eng, model, w, h, **opts)
    slots = [s.add_input(), s.add_input()]
    out = s.add_output()
    if opts.get("protection_mask"):
        m = np.zeros((h, w), np.uint8)
        m[h - 60:h - 20, 20:200] = 1
        s.write_mask(m)
    pp = model.plan_params(w, h, **opts)
    s.write(slots[0], frames[0])
    for i in range(1, len(frames)):  # enough pairs for ages to reach the protecting age
        a, b = slots[(i - 1) % 2], slots[i % 2]
        s.write(b, frames[i])
        s.pair(a, b)
        s.mid(0.5, out)
    got = np.frombuffer(s.read(out), np.uint8)
    age = s.tensor("age")[0] if pp["protects"] else None
    ref = oracle.render_planes(frames[-2], frames[-1], w, h, s.tensor("up7"), s.tensor("R_t"), age, pp["fsx"],
                               pp["fsy"], pp["min_age"], pp["static_thr"], cubic=bool(pp["cubic"]),
                               flags=pp["render_flags"])
    d = np.abs(got.astype(np.int32) - ref.astype(np.int32)).reshape(-1, 4)[:, :3]
    assert d.max() <= 1, (int(d.max()), int((d > 1).sum()))


@pytest.mark.parametrize("size,opts,t", [((1280, 720), dict(fast_render=True), 0.5),
                                         ((1280, 720), dict(fast_render=True, linear_t=True), 0.25),
                                         ((640, 360), dict(fast_render=True, linear_t=True, render="bilinear"), 0.75),
                                         ((333, 197), dict(fast_render=True, protection_mask=True), 0.5)])
def test_render_tex_on_identical_inputs(synth_model_dir, size, opts, t):
    """The fast render (render_tex.wgsl: rgba8 texels, linear-t scales, its own still test and static rules) against
    the oracle's on the GPU's own maps and age plane: within one level everywhere."""
    import flyhigh_engine_b200 as fh
    from flyhigh_engine_b200 import synth_frames
    from oracle import oracle
    w, h = size
    frames = synth_frames.sequence_c2(10, w, h, seed=6)
    eng = fh.Engine()
    model = fh.Model(synth_model_dir)
    s = fh.Session(eng, model, w, h, **opts)
    slots = [s.add_input(), s.add_input()]
    out = s.add_output()
    if opts.get("protection_mask"):
        m = np.zeros((h, w), np.uint8)
        m[h - 60:h - 20, 20:200] = 1
        s.write_mask(m)
    pp = model.plan_params(w, h, **opts)
    s.write(slots[0], frames[0])
    for i in range(1, len(frames)):
        a, b = slots[(i - 1) % 2], slots[i % 2]
        s.write(b, frames[i])
        s.pair(a, b)
        s.mid(t, out)
    got = np.frombuffer(s.read(out), np.uint8)
    age = s.tensor("age")[0] if pp["protects"] else None
    sa, sb, sr = (2 * t, 2 * (1 - t), 1 - abs(2 * t - 1)) if opts.get("linear_t") else (1.0, 1.0, 1.0)
    ref = oracle.render_tex_planes(frames[-2], frames[-1], w, h, s.tensor("up7"), s.tensor("R_t"), age, pp["fsx"],
                                   pp["fsy"], pp["min_age"], cubic=bool(pp["cubic"]), flags=pp["render_flags"],
                                   sa=np.float32(2) * np.float32(t) if opts.get("linear_t") else 1.0,
                                   sb=np.float32(2) * (np.float32(1) - np.float32(t)) if opts.get("linear_t") else 1.0,
                                   sr=sr)
    d = np.abs(got.astype(np.int32) - ref.astype(np.int32)).reshape(-1, 4)[:, :3]
    assert d.max() <= 1, (int(d.max()), int((d > 1).sum()), (sa, sb, sr))


@pytest.mark.parametrize("size,opts", [((640, 360), dict(fast_render=True)),
                                       ((1280, 720), dict(fast_render=True, linear_t=True))])
def test_fast_session_matches_oracle(synth_model_dir, size, opts):
    """The fast render session end to end (tex_down or tex_in, the age pass on texels, the mid maps, render_tex; with
    linear_t the maps once per pair at t = 0.5) against the oracle's: the network input and the maps per layer, the
    age state inside the frame exactly, and every phase's frame."""
    import flyhigh_engine_b200 as fh
    from flyhigh_engine_b200 import synth_frames
    from oracle.oracle import OracleModel, OracleSession
    from tests.frame_parity import reach_mask
    w, h = size
    frames = synth_frames.sequence_c2(4, w, h, seed=7)
    model = fh.Model(synth_model_dir)
    pp = model.plan_params(w, h, **opts)
    s = fh.Session(fh.Engine(), model, w, h, **opts)
    s0 = fh.Session(fh.Engine(), model, w, h, repair=0, **opts)  # the GPU's pre-repair flow
    slots, slots0 = [s.add_input(), s.add_input()], [s0.add_input(), s0.add_input()]
    out = s.add_output()
    o = OracleSession(OracleModel(synth_model_dir), w, h, **opts)
    s.write(slots[0], frames[0])
    s0.write(slots0[0], frames[0])
    for i in range(1, len(frames)):
        for ss, sl in ((s, slots), (s0, slots0)):
            ss.write(sl[i % 2], frames[i])
            ss.pair(sl[(i - 1) % 2], sl[i % 2])
        o.pair(frames[i - 1], frames[i])
        fl = flipped_cells((o.gmhs_select(o.tensor("flow_pre")), o.gmhs_select(s0.tensor("flow"))))
        keep = ~reach_mask(fl, w, h, pp) if len(fl) else None
        _check_layers(s, o, ["A", "B", "o", "fr3"], 0)
        assert np.array_equal(s.tensor("age")[:, :h, :w], o.tensor("age")[:, :h, :w]), f"age differs after pair {i}"
        for t in (0.25, 0.5, 0.75):
            s.mid(t, out)
            got = np.frombuffer(s.read(out), np.uint8)
            ref = o.mid(t)
            ok, info = _frame_ok(got, ref, keep)
            assert ok, (i, t, info, len(fl))
        _check_layers(s, o, ["up7", "R_t"], 1, flipped=fl)


def test_batched_fast_matches_single(synth_model_dir):
    """A batched fast_render + linear_t session gives the same frames whether its intervals run four at a time or one
    at a time, including further phases of the newest pair after a batch."""
    import flyhigh_engine_b200 as fh
    from flyhigh_engine_b200 import synth_frames
    w, h, batch = 384, 160, 4
    model = fh.Model(synth_model_dir)
    frames = synth_frames.sequence_c2(batch + 2, w, h, seed=8)

    def run(read_each):
        s = fh.Session(fh.Engine(), model, w, h, batch=batch, fast_render=True, linear_t=True)
        ins = [s.add_input(), s.add_input()]
        outs = [s.add_output() for _ in range(batch + 3)]
        got = {}
        s.write(ins[0], frames[0])
        for i in range(1, batch + 1):
            s.write(ins[i % 2], frames[i])
            s.pair(ins[(i - 1) % 2], ins[i % 2])
            s.mid(0.2 * i, outs[i])
            if read_each:
                got[i] = np.frombuffer(s.read(outs[i]), np.uint8).copy()
        for i in range(1, batch + 1):
            if i not in got:
                got[i] = np.frombuffer(s.read(outs[i]), np.uint8).copy()
        s.mid(0.6, outs[0])  # a further phase of the newest pair: its t = 0.5 maps are reused
        return [got[i] for i in range(1, batch + 1)] + [np.frombuffer(s.read(outs[0]), np.uint8).copy()]

    single, batched = run(True), run(False)
    for i, (x, y) in enumerate(zip(single, batched)):
        assert np.array_equal(x, y), i


class GmhsParams(Structure):
    _fields_ = [("flow", c_void_p), ("flow_bs", c_longlong), ("h8", c_int), ("w8", c_int), ("a", c_void_p),
                ("b", c_void_p), ("ab_bs", c_longlong), ("h", c_int), ("w", c_int), ("full_w", c_int),
                ("level", c_int), ("scratch", c_void_p), ("n", c_int)]


def nhwc(torch, chw, cs):
    """[c][h][w] float values of f16 tensors -> a device [h][w][cs] f16 buffer (pad channels zero)."""
    c, h, w = chw.shape
    t = torch.zeros((h, w, cs), dtype=torch.float16)
    t[:, :, :c] = torch.from_numpy(np.ascontiguousarray(chw.transpose(1, 2, 0))).to(torch.float16)
    return t.cuda()


def run_gmhs(torch, a_chw, b_chw, flow_chw, full_w, level):
    import flyhigh_engine_b200 as fh
    L = fh.lib()
    _, h, w = a_chw.shape
    _, h8, w8 = flow_chw.shape
    A, B, F = nhwc(torch, a_chw, 4), nhwc(torch, b_chw, 4), nhwc(torch, flow_chw, 8)
    scratch = torch.zeros(L.fhk_gmhs_scratch_floats(h, w), dtype=torch.float32, device="cuda")
    p = GmhsParams(F.data_ptr(), 0, h8, w8, A.data_ptr(), B.data_ptr(), 0, h, w, full_w, level, scratch.data_ptr(), 1)
    rc = L.fhk_gmhs(ctypes.byref(p), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, rc
    torch.cuda.synchronize()
    return F[:, :, :4].permute(2, 0, 1).float().cpu().numpy()


@pytest.mark.parametrize("size,level", [((1920, 1080), 1), ((640, 360), 2), ((1280, 720), 1)])
def test_gmhs_on_identical_inputs(torch_cuda, synth_model_dir, size, level):
    """The repair stage (IRLS affine fit with the shader's reduction tree, cost maps, box windows, select) on the
    oracle's own inputs: the rewritten flow matches the oracle's bit for bit."""
    from flyhigh_engine_b200 import synth_frames
    from oracle.oracle import OracleModel, OracleSession
    w, h = size
    fa, fb, _ = synth_frames.pair_c0(w, h, seed=7)
    o = OracleSession(OracleModel(synth_model_dir), w, h, repair=level)
    o.pair(fa, fb)
    pre, post = o.tensor("flow_pre"), o.tensor("flow")
    got = run_gmhs(torch_cuda, o.tensor("A"), o.tensor("B"), pre, o.dims()["wp"], level)
    changed = int((pre != post).any(axis=0).sum())
    assert np.array_equal(got, post), (changed, int((got != post).any(axis=0).sum()))
