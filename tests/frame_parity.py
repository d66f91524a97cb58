"""End-to-end frame parity with an explanation for every pixel beyond the north star's 2 levels.

The GPU's network outputs differ from the oracle's by the f32 summation order of the tensor-core convs: a few f16 ulps
(about 1e-3 relative L2, checked per layer). The render turns some of those differences into more than 2 levels at a
few pixels, in four ways, each a threshold or a steep slope of the render in the oracle's own run:

  gmhs   the repair stage's select (gm_select.wgsl: ca + eps < cm, dv > dmin, sd > tex) decided a cell differently
         because one of its conditions sat within GMHS_TOL of its threshold in both runs, or because the two runs'
         pre-repair flows, within POS_ULPS f16 ulps of each other around the cell, moved a cost condition across its
         threshold (a cost moves by the local luma gradient times the flow difference: several 1e-3 per f16 ulp at a
         sharp edge; both decisions come from the oracle's own rule, only the flows differ); the cell's flow then
         differs by more than dmin (several px), and so does every pixel the cell reaches through the mid network and
         the render (within GMHS_REACH E8 cells);
  static a static rule's probe (render.wgsl's `round()` of the source position, then the 3 x 3 protected-age test)
         rounded to another pixel: the source positions of the two runs agree (to POS_ULPS f16 ulps of the flow or
         POS_ABS network px), but lie on either side of a half-pixel boundary;
  still  the still test's weight (a ramp of slope 1 / 0.04 on ef - es) moved: the positions agree, and the ramp input
         of at least one run lies on the ramp;
  edge   no decision moved, the positions agree, and the bicubic samples' own change accounts for the
         difference (at most EDGE_SLACK levels besides): a steep edge under the tap window, whose slope bound
         (2.0625 x the taps' value range per px: max sum |w| = 1.375 times half of max sum |w'| = 3 of the Keys
         a = -0.75 kernel) covers the sample change.

Everything else is "unexplained" and fails the check. The PSNR bound (50 dB) holds over the pixels that no flipped
repair cell reaches: two repairs that choose differently at a threshold differ there by as much as their choices do. The classifier evaluates both renders with the oracle's decision
record (oracle.render_diag), on the oracle's own network outputs and on the GPU's: the render is the same code on both,
so any difference between those two records comes from the network outputs alone. Separately, the GPU frame must equal
the oracle's render of the GPU's own network outputs within RENDER_GAP level everywhere (the render on identical
inputs).
"""
from __future__ import annotations

import numpy as np

from oracle import oracle
from tests.parity import FRAME_MAX_ABS, FRAME_PSNR_DB, frame_stats

# The source positions of the two runs agree when each flow component (network px: the render scales flow_tq by
# fsx / fsy) differs by at most POS_ULPS f16 ulps of the oracle's flow value there, or by at most POS_ABS network px.
POS_ULPS = 4
POS_ABS = 2e-2
# a flipped repair cell: a condition whose sign differs between the runs, within this of its threshold in both runs
# (cm - ca in luma units, dv - dmin in E8 px; sd - tex depends on frame A alone, identical in both runs)
GMHS_TOL = {"m_cost": 1e-3, "m_dv": 1e-2}
GMHS_REACH = 5       # E8 cells: how far a flipped cell's flow reaches (convex upsample, refine convs, render bilinear)
EDGE_SLACK = 3       # levels: the render gap (1), rounding (1), blend-weight and residual changes (1)
RENDER_GAP = 1       # levels between the GPU frame and the oracle's render of the GPU's network outputs
KEYS_SLOPE = 2.0625  # Keys a = -0.75: max sum |w| (1.375) x max sum |w'| (3) / 2


# layers the repair stage's flow reaches: the repaired E8 flow and everything the mid network derives from it
POST_REPAIR = {"flow", "vis", "hm", "fh1", "fh2", "dfilm", "ft_vt", "up7", "rx", "rq1", "rq2", "rq3", "R_t"}


def flipped_cells(gmhs):
    """The E8 cells whose repair decision differs between the two runs' records ((oracle, gpu) gmhs_select)."""
    if gmhs is None:
        return np.zeros((0, 2), np.int64)
    return np.argwhere(gmhs[0]["sel"] != gmhs[1]["sel"])


def layer_rel_l2(name, got, ref, flipped, h8):
    """Relative L2 of a layer, leaving out the positions that a flipped repair cell reaches (GMHS_REACH E8 cells, at
    the layer's own resolution) when the layer comes after the repair stage: two repairs that choose differently at a
    threshold differ there by more than dmin px of flow, as much as their choices do."""
    from tests.parity import rel_l2
    got, ref = np.asarray(got), np.asarray(ref)
    if name not in POST_REPAIR or len(flipped) == 0:
        return rel_l2(got, ref)
    _, h, w = ref.shape
    scale = max(1, int(round(h / h8)))  # E8 layers 1, quarter-resolution layers 2
    keep = np.ones((h, w), bool)
    r = GMHS_REACH * scale
    for i, j in flipped.tolist():
        ci, cj = i * scale, j * scale
        keep[max(ci - r, 0):ci + r + scale, max(cj - r, 0):cj + r + scale] = False
    return rel_l2(got[:, keep], ref[:, keep])


def reach_mask(flipped, w, h, pp):
    """The frame's pixels (h x w bool) within GMHS_REACH E8 cells of a flipped repair cell."""
    yy, xx = np.mgrid[0:h, 0:w]
    ci, cj = _e8_of(xx.reshape(-1), yy.reshape(-1), pp["fsx"], pp["fsy"], pp["w8"], pp["h8"])
    reach = np.zeros(h * w, bool)
    for (i, j) in np.asarray(flipped).tolist():
        reach |= (np.abs(ci - i) <= GMHS_REACH) & (np.abs(cj - j) <= GMHS_REACH)
    return reach.reshape(h, w)


def _e8_of(xs, ys, fsx, fsy, w8, h8):
    """The E8 cell (i, j) under full-resolution pixels: full -> internal (/ fs) -> E8 (/ 8)."""
    j = np.clip(np.floor((xs + 0.5) / fsx / 8.0).astype(np.int64), 0, w8 - 1)
    i = np.clip(np.floor((ys + 0.5) / fsy / 8.0).astype(np.int64), 0, h8 - 1)
    return i, j


def _pre_flow_tol(go, gg, i, j):
    """The largest pre-repair flow difference of the two runs over E8 cell (i, j)'s reach (GMHS_REACH cells), in units
    of max(POS_ULPS f16 ulps of the oracle's flow, POS_ABS); None when the records carry no flows ("flow")."""
    if "flow" not in go or "flow" not in gg:
        return None
    fo, fg = np.asarray(go["flow"], np.float64), np.asarray(gg["flow"], np.float64)
    sl = (slice(None), slice(max(i - GMHS_REACH, 0), i + GMHS_REACH + 1), slice(max(j - GMHS_REACH, 0), j + GMHS_REACH + 1))
    a, b = fo[sl], fg[sl]
    ulp = np.spacing(np.abs(a).astype(np.float16)).astype(np.float64)
    return float((np.abs(a - b) / np.maximum(POS_ULPS * ulp, POS_ABS)).max())


def gmhs_records(o, gpu_pre_flow):
    """(oracle, gpu) repair decision records on the oracle's current pair: the oracle's repair rule over its own
    pre-repair flow and over the GPU's, each with the flow it was given ("flow")."""
    ora = np.asarray(o.tensor("flow_pre"))
    go, gg = o.gmhs_select(ora), o.gmhs_select(gpu_pre_flow)
    go["flow"], gg["flow"] = ora, np.asarray(gpu_pre_flow)
    return go, gg


def check_frame(got, ref, fa, fb, w, h, pp, gpu_maps, ora_maps, age, gmhs=None, max_over=None):
    """Frame parity of one generated frame. got / ref: the GPU's and the oracle's rgba8 frames; fa, fb: the interval's
    source frames; pp: the session's plan parameters (Model.plan_params); gpu_maps / ora_maps: (up7, R_t) of each run;
    age: the (common, exactly checked) age plane or None; gmhs: None, or (ora, gpu), the OracleSession.gmhs_select
    records of both runs' pre-repair flows (gmhs_records: with the flows, so that a flip away from a threshold is
    accepted where the two pre-repair flows agree within POS_ULPS f16 ulps around the cell). Returns a report dict;
    report["ok"] says whether the frame passes: PSNR (over the pixels that no accepted repair flip reaches), the render
    gap, no repair cell flipped unexplained, and no unexplained pixel."""
    H, W = h, w
    g = np.asarray(got, np.int32).reshape(H, W, 4)[..., :3]
    r = np.asarray(ref, np.int32).reshape(H, W, 4)[..., :3]
    mx, psnr = frame_stats(got, ref)
    cubic, flags = bool(pp["cubic"]), int(pp["render_flags"])
    age2 = None if age is None else np.asarray(age, np.float32).reshape(age.shape[-2], age.shape[-1])
    rep = oracle.render_planes(fa, fb, W, H, gpu_maps[0], gpu_maps[1], age2, pp["fsx"], pp["fsy"], pp["min_age"],
                               pp["static_thr"], cubic=cubic, flags=flags)
    gap = int(np.abs(g - np.asarray(rep, np.int32).reshape(H, W, 4)[..., :3]).max())
    dch = np.abs(g - r)
    d = dch.max(-1)
    ys, xs = np.nonzero(d > FRAME_MAX_ABS)
    cats = {"gmhs": 0, "static": 0, "still": 0, "edge": 0, "unexplained": 0}
    rep_out = {"max": mx, "psnr": psnr, "render_gap": gap, "over": int(len(xs)), "cats": cats, "unexplained": [],
               "max_pos_shift": 0.0}
    # the repair cells decided differently, and whether each sat at a threshold
    flipped = np.zeros((0, 2), np.int64)
    gm_bad = []
    if gmhs is not None:
        go, gg = gmhs
        fl = np.argwhere(go["sel"] != gg["sel"])
        flipped = fl
        margins = []
        for (i, j) in fl:
            # the conditions whose sign differs between the runs, with their larger |margin|
            flips = {k: max(abs(float(go[k][i, j])), abs(float(gg[k][i, j]))) for k in GMHS_TOL
                     if (float(go[k][i, j]) > 0) != (float(gg[k][i, j]) > 0)}
            near = {k: m for k, m in flips.items() if m <= GMHS_TOL[k]}
            ft = _pre_flow_tol(go, gg, i, j)
            if near:
                margins.append(near)
            elif ft is not None and ft <= 1.0:
                # both records come from the oracle's own repair rule, so the flip is the pre-repair flows' doing;
                # those agree within POS_ULPS f16 ulps (or POS_ABS) over the cell's reach: rounding amplified by a
                # cost that moves by the luma gradient times the flow (a few 1e-3 per f16 ulp at a sharp edge)
                margins.append({"pre_flow_tol": ft})
            else:
                gm_bad.append((int(i), int(j), dict(flips, pre_flow_tol=ft)))
        rep_out["gmhs_flipped"] = int(len(fl))
        rep_out["gmhs_margins"] = margins
        rep_out["gmhs_not_adjacent"] = gm_bad
    if len(xs):
        kw = dict(cubic=cubic, flags=flags)
        Do = oracle.render_diag(fa, fb, W, H, ora_maps[0], ora_maps[1], age2, pp["fsx"], pp["fsy"], pp["min_age"],
                                xs, ys, **kw)
        Dg = oracle.render_diag(fa, fb, W, H, gpu_maps[0], gpu_maps[1], age2, pp["fsx"], pp["fsy"], pp["min_age"],
                                xs, ys, **kw)
        dpos_a = np.abs(Do["gxa"] - Dg["gxa"]) + np.abs(Do["gya"] - Dg["gya"])
        dpos_b = np.abs(Do["gxb"] - Dg["gxb"]) + np.abs(Do["gyb"] - Dg["gyb"])
        dpos = np.maximum.reduce([np.abs(Do[k] - Dg[k]) for k in ("gxa", "gya", "gxb", "gyb")])
        # each component's difference in units of its tolerance: POS_ULPS f16 ulps of the oracle's flow value (network
        # px) at the pixel, at least POS_ABS
        ulps, rel = [], []
        for k, base, fs in (("gxa", xs, pp["fsx"]), ("gya", ys, pp["fsy"]), ("gxb", xs, pp["fsx"]),
                            ("gyb", ys, pp["fsy"])):
            flow = (Do[k] - base) / fs
            ulp = np.spacing(np.abs(flow).astype(np.float16)).astype(np.float64)
            dn = np.abs(Do[k] - Dg[k]) / fs
            ulps.append(dn / np.maximum(ulp, 2.0 ** -24))
            rel.append(dn / np.maximum(POS_ULPS * ulp, POS_ABS))
        dulp = np.maximum.reduce(ulps)
        dtol = np.maximum.reduce(rel)
        near_flip = np.zeros(len(xs), bool)
        if len(flipped):
            ci, cj = _e8_of(xs, ys, pp["fsx"], pp["fsy"], pp["w8"], pp["h8"])
            bad = {(a, b) for a, b, _ in gm_bad}
            good = [(i, j) for (i, j) in flipped.tolist() if (i, j) not in bad]
            for (i, j) in good:
                near_flip |= (np.abs(ci - i) <= GMHS_REACH) & (np.abs(cj - j) <= GMHS_REACH)
        static_flip = (Do["sa"] != Dg["sa"]) | (Do["sb"] != Dg["sb"])
        # a flipped static rule: the rounded probe position moved on the side that flipped
        rnd = lambda v: np.rint(v)  # round half to even, as WGSL round()
        moved_a = (rnd(Do["gxa"]) != rnd(Dg["gxa"])) | (rnd(Do["gya"]) != rnd(Dg["gya"]))
        moved_b = (rnd(Do["gxb"]) != rnd(Dg["gxb"])) | (rnd(Do["gyb"]) != rnd(Dg["gyb"]))
        static_ok = static_flip & (((Do["sa"] != Dg["sa"]) & moved_a) | ((Do["sb"] != Dg["sb"]) & moved_b))
        still_flip = np.abs(Do["stillw"] - Dg["stillw"]) > 1e-6
        on_ramp = lambda v: (v > 0.0) & (v < 0.04)
        still_ok = still_flip & (on_ramp(Do["ramp"]) | on_ramp(Dg["ramp"]) | (np.sign(Do["ramp"]) != np.sign(Dg["ramp"]))
                                 | (np.sign(Do["ramp"] - 0.04) != np.sign(Dg["ramp"] - 0.04)))
        # bicubic sample change per channel, and the slope bound it must respect
        # (its share of the output: the still mix, the static source mix and the keep_static ramp scale it down)
        kk = np.clip((Dg["age"] - pp["min_age"] + 2.0) / 2.0, 0.0, 1.0) if age2 is not None else 0.0
        share = (1.0 - Dg["stillw"]) * (1.0 - Dg["raw"]) * (1.0 - kk)
        samp = np.stack([Dg["bwa"] * np.abs(Dg[f"ca{c}"] - Do[f"ca{c}"]) + Dg["bwb"] * np.abs(Dg[f"cb{c}"] - Do[f"cb{c}"])
                         for c in range(3)], 1) * (255.0 * share)[:, None]
        rng_a = np.maximum(Do["range_a"], Dg["range_a"])
        rng_b = np.maximum(Do["range_b"], Dg["range_b"])
        bound = KEYS_SLOPE * 255.0 * share * (Dg["bwa"] * rng_a * dpos_a + Dg["bwb"] * rng_b * dpos_b) + 0.5
        dpx = dch[ys, xs]  # [n][3]
        need = np.where(dpx > FRAME_MAX_ABS, dpx - EDGE_SLACK, -1e9).max(1)
        edge_ok = (samp.max(1) >= need) & (samp.max(1) <= bound)
        close = dtol <= 1.0
        for k in range(len(xs)):
            if close[k] and static_ok[k]:
                c = "static"
            elif close[k] and still_ok[k] and not static_flip[k]:
                c = "still"
            elif close[k] and edge_ok[k] and not static_flip[k] and not still_flip[k]:
                c = "edge"
            elif near_flip[k]:
                c = "gmhs"
            else:
                c = "unexplained"
                if len(rep_out["unexplained"]) < 20:
                    rep_out["unexplained"].append(dict(
                        x=int(xs[k]), y=int(ys[k]), d=int(d[ys[k], xs[k]]), dpos=float(dpos[k]), dulp=float(dulp[k]),
                        dtol=float(dtol[k]),
                        static=bool(static_flip[k]), still=bool(still_flip[k]), samp=float(samp[k].max()),
                        need=float(need[k]), bound=float(bound[k])))
            cats[c] += 1
        rep_out["max_pos_shift"] = float(dpos[close].max()) if close.any() else 0.0
        rep_out["max_pos_ulps"] = float(dulp[close].max()) if close.any() else 0.0
        rep_out["max_pos_tol"] = float(dtol[close].max()) if close.any() else 0.0
    # PSNR over the pixels that no threshold-adjacent repair flip reaches (a flipped cell's flow differs by more than
    # dmin px, so the frame there differs as much as two repairs' choices do); the whole frame's PSNR is reported too
    psnr_rest = psnr
    if len(flipped) and not gm_bad:
        reach = reach_mask(flipped, W, H, pp)
        keep = ~reach
        diff = (g - r).astype(np.float64)[keep]
        mse = float((diff ** 2).mean()) if diff.size else 0.0
        psnr_rest = float("inf") if mse == 0 else float(10 * np.log10(255.0 ** 2 / mse))
        rep_out["gmhs_reach_px"] = int(reach.sum())
    rep_out["psnr_outside_repair_flips"] = psnr_rest
    rep_out["ok"] = bool(psnr_rest >= FRAME_PSNR_DB and gap <= RENDER_GAP and cats["unexplained"] == 0
                         and not gm_bad and (max_over is None or len(xs) <= max_over))
    return rep_out
