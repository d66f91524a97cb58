"""Extracts the parameter words of the reference's golden plan dumps into tests/golden/plan_params.json.

The reference pins its planner with text dumps of every dispatch (crates/flyhigh-engine/tests/golden/<config>.tc-f16.txt,
written by tests/golden_plans.rs: pipeline, workgroups, binding sizes, uniform words). This script keeps, for the
configurations the exact-render Session builds (fast render is not part of this build), the words that fix sizes and
parameters: every conv's (cin, h, w, hout, wout, stride, cout), every interp, sad, warp, the GMHS windows and
thresholds, and the render's scales, sampler and protecting age. Run it with a checkout of the reference repository:
    python tests/golden/make_plan_params.py <reference checkout>    (or FLYHIGH_REFERENCE=<checkout>)
"""
import json
import os
import struct
import sys

CONFIGS = ["rt-720p-default", "rt-720p-repair0", "rt-720p-repair2", "rt-480p-k2"]
CONV_PIPES = {"fused", "fused2", "fdirect", "fdirect32", "fdirect64", "tconv", "tconv8", "tconv88", "tconv8p"}


def f32(word):
    return struct.unpack("<f", struct.pack("<I", int(word, 16)))[0]


def parse(path):
    out = {"header": None, "pair": [], "mid": []}
    stage = None
    for line in open(path):
        line = line.rstrip("\n")
        if line.startswith("# rt") or line.startswith("# cpu"):
            out["header"] = line[2:]
            continue
        if line == "# pair":
            stage = "pair"
            continue
        if line == "# mid":
            stage = "mid"
            continue
        parts = line.split()
        if len(parts) < 3 or stage is None:
            continue
        pipe = parts[1]
        words = [p for p in parts if len(p) == 8 and all(c in "0123456789abcdef" for c in p)]
        out[stage].append((pipe, words))
    return out


def extract(path):
    d = parse(path)
    hdr = d["header"].split()
    kv = dict(x.split("=") for x in hdr[2:] if "=" in x)
    w, h = (int(v) for v in hdr[1].split("x"))
    rec = {"config": hdr[0], "width": w, "height": h, "k": int(kv["k"]), "repair": int(kv["repair"]),
           "internal": [int(v) for v in kv["internal"].split("x")], "pair_dispatches": len(d["pair"]),
           "mid_dispatches": len(d["mid"]), "convs": [], "interps": [], "sads": [], "warps": [], "gm": {},
           "render": None}
    for stage in ("pair", "mid"):
        for pipe, wd in d[stage]:
            u = [int(x, 16) for x in wd]
            if pipe in CONV_PIPES:
                # ImplicitGemmParams: cin, h, w, hout, wout, stride, pad, k, kp, n, ...
                rec["convs"].append({"stage": stage, "cin": u[0], "h": u[1], "w": u[2], "hout": u[3], "wout": u[4],
                                     "stride": u[5], "cout": u[9]})
            elif pipe == "interp":
                rec["interps"].append({"stage": stage, "c": u[0], "ih": u[1], "iw": u[2], "oh": u[3], "ow": u[4],
                                       "aa": u[5], "c0": u[6], "scale": f32(wd[7])})
            elif pipe == "sad":
                rec["sads"].append({"stage": stage, "h": u[0], "w": u[1], "radius": u[2]})
            elif pipe == "warp":
                rec["warps"].append({"stage": stage, "c": u[0], "h": u[1], "w": u[2], "f0": u[3], "i0": u[4],
                                     "fs": f32(wd[5]), "is": f32(wd[6])})
            elif pipe == "gm_fit_reduce":
                rec["gm"]["delta"] = f32(wd[4])
                rec["gm"]["h8"], rec["gm"]["w8"] = u[0], u[1]
            elif pipe == "gm_cost":
                rec["gm"]["h"], rec["gm"]["w"], rec["gm"]["hc"], rec["gm"]["wc"] = u[2], u[3], u[4], u[5]
            elif pipe == "gm_box_h":
                rec["gm"].setdefault("radii", []).append(u[3])
            elif pipe == "gm_select":
                rec["gm"]["dmin"] = f32(wd[5])
                rec["gm"]["tex"] = f32(wd[6])
            elif pipe in ("render", "render_static"):
                rec["render"] = {"H": u[0], "W": u[1], "hq": u[2], "wq": u[3], "f0": u[4], "v0": u[5],
                                 "fsx": f32(wd[6]), "fsy": f32(wd[7]), "vs": f32(wd[8]), "cubic": u[9],
                                 "min_age": u[10], "flags": u[11]}
    return rec


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FLYHIGH_REFERENCE", "")
    if not ref:
        sys.exit("usage: make_plan_params.py <reference checkout>")
    gdir = os.path.join(ref, "crates", "flyhigh-engine", "tests", "golden")
    out = [extract(os.path.join(gdir, f"{c}.tc-f16.txt")) for c in CONFIGS]
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "plan_params.json")
    with open(dst, "w") as f:
        json.dump(out, f, indent=1)
    print(dst)


if __name__ == "__main__":
    main()
