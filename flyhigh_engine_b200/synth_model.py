"""A FlyHighFG model directory with seeded synthetic weights.

The shipped weights (models/flyhighfg.bin of the reference) are CC BY-NC 4.0 and are not redistributed with this
package. Where they are absent (the GPU hosts, CI), a model directory with the same graph and tensor shapes and seeded
N(0, 0.05) f16 weights stands in for them; the engine loads either the same way.

The graph below is the FlyHighFG operation list in the reference's graph.json format (format_version 1; the op
vocabulary of crates/flyhigh-engine/src/net/build.rs:191-475, the op order of models/graph.json). It is written out
here op by op so the engine, its tests and its benchmark run where the reference's files are not present; a CPU test
checks it against the reference's own graph.json and manifest shapes wherever those are readable.
"""
from __future__ import annotations

import json
import os
from typing import Dict, List, Tuple

import numpy as np

# channel widths of the shipped checkpoint (flyhighfg.json meta.cfg)
C8, C16, CC, CR, CQ = 36, 72, 96, 48, 24


def graph_ops() -> List[dict]:
    ops: List[dict] = []

    def op(kind, ins, outs, **kw):
        d = {"in": ins, "out": outs}
        d.update(kw)
        d["op"] = kind
        ops.append(d)
        return d

    def conv(x, y, prefix, stride=1, **kw):
        op("conv", [x], [y], w=[f"{prefix}.0.weight", f"{prefix}.0.bias", f"{prefix}.1.weight"], stride=stride, **kw)

    def conv2d(x, y, prefix, **kw):
        op("conv2d", [x], [y], w=[f"{prefix}.weight", f"{prefix}.bias"], **kw)

    interp = dict(scale=0.25, mode="bilinear", align_corners=False, antialias=True)
    op("interpolate", ["A"], ["aq"], **interp)
    op("interpolate", ["B"], ["bq"], **interp)
    for s in "ab":
        conv(f"{s}q", f"{s}_e1", "enc.e1", 2)
        conv(f"{s}_e1", f"{s}_e2", "enc.e2", 1)
        op("add", [f"{s}_e2", f"{s}_e1"], [f"f8{s}"])
        conv(f"f8{s}", f"{s}_e3", "enc.e3", 2)
        conv(f"{s}_e3", f"{s}_e4", "enc.e4", 1)
        op("add", [f"{s}_e4", f"{s}_e3"], [f"f16{s}"])
    op("avgpool", ["aq"], ["i8a"], k=2)
    op("avgpool", ["bq"], ["i8b"], k=2)
    op("avgpool", ["i8a"], ["i16a"], k=2)
    op("avgpool", ["i8b"], ["i16b"], k=2)
    op("concat", ["i16a", "i16b"], ["img16"], axis=1)
    op("zeros", ["f16a"], ["side"], ch=4)
    op("zeros", ["f16a"], ["state"], ch=76)
    op("slice", ["img16"], ["img16a"], a=0, b=3)
    op("slice", ["img16"], ["img16b"], a=3, b=6)
    op("luma", ["img16a"], ["la"])
    op("luma", ["img16b"], ["lb"])
    op("sad_volume", ["la", "lb"], ["cv"], radius=3)
    op("concat", ["f16a", "f16b", "img16", "side", "state", "cv"], ["cin"], axis=1)
    conv("cin", "ch1", "coarse.c1")
    conv("ch1", "ch2", "coarse.c2")
    conv("ch2", "ch3", "coarse.c3")
    op("add", ["ch3", "ch1"], ["ch3r"])
    conv("ch3r", "hc", "coarse.c4")
    conv2d("hc", "o", "coarse.head")
    op("slice", ["o"], ["o04"], a=0, b=4)
    op("scale", ["o04"], ["flow16"], factor=16.0)
    op("slice", ["o"], ["vis16"], a=4, b=7)
    op("slice", ["o"], ["conf"], a=7, b=8, output=True)
    op("slice", ["o"], ["gate"], a=8, b=9, output=True)
    op("slice", ["o"], ["sal"], a=9, b=10, output=True)
    up2 = dict(scale=2, mode="bilinear", align_corners=False)
    op("interpolate", ["flow16"], ["flow"], **up2)
    op("interpolate", ["vis16"], ["vis"], **up2)
    op("zeros", ["flow"], ["h"], ch=CR)

    body_start = len(ops)
    op("scale", ["flow"], ["flow8"], factor=0.125)
    op("slice", ["flow8"], ["flow8f"], a=0, b=2)
    op("slice", ["flow8"], ["flow8b"], a=2, b=4)
    op("warp", ["f8a", "flow8f"], ["wa"])
    op("warp", ["f8b", "flow8b"], ["wb"])
    op("warp", ["i8a", "flow8f"], ["ia"])
    op("warp", ["i8b", "flow8b"], ["ib"])
    op("luma", ["ia"], ["fla"])
    op("luma", ["ib"], ["flb"])
    op("sad_volume", ["fla", "flb"], ["fcv"], radius=2)
    op("concat", ["wa", "wb", "ia", "ib", "flow8", "h", "fcv"], ["fx"], axis=1)
    conv("fx", "fr1", "fine.r1")
    conv("fr1", "fr2", "fine.r2")
    conv("fr2", "fr3", "fine.r3")
    conv2d("fr3", "d", "fine.out")
    op("slice", ["d"], ["d04"], a=0, b=4)
    op("add", ["flow", "d04"], ["flow"])
    op("slice", ["d"], ["d47"], a=4, b=7)
    op("add", ["vis", "d47"], ["vis"])
    op("copy", ["fr3"], ["h"])
    body = ops[body_start:]
    del ops[body_start:]
    ops.append({"op": "repeat", "times": "K", "carry": ["flow", "vis", "h"], "body": body})

    op("concat", ["f16b", "flow16"], ["state_out"], axis=1, output=True)
    op("slice", ["flow"], ["flowf"], a=0, b=2)
    op("slice", ["flow"], ["flowb"], a=2, b=4)
    op("mul_t", ["flowf"], ["linf"], mode="fwd")
    op("mul_t", ["flowb"], ["linb"], mode="bwd")
    op("concat", ["linf", "linb"], ["lin"], axis=1)
    film = dict(cond="use_film")
    op("film_mlp", ["t"], ["g"], w=["film.film.0.weight", "film.film.0.bias", "film.film.2.weight",
                                   "film.film.2.bias"], **film)
    op("film_modulate", ["h", "g"], ["hm"], cr=CR, **film)
    conv("hm", "fh1", "film.h1", **film)
    conv("fh1", "fh2", "film.h2", **film)
    conv2d("fh2", "dfilm", "film.out", **film)
    op("slice", ["dfilm"], ["d_flow"], a=0, b=4, **film)
    op("slice", ["dfilm"], ["d_mask"], a=4, b=5, **film)
    op("add", ["lin", "d_flow"], ["flow_t"], else_alias={"flow_t": "lin"}, **film)
    op("neg", ["d_mask"], ["nd"], **film)
    op("zeros_like", ["d_mask"], ["zd"], **film)
    op("concat", ["d_mask", "nd", "zd"], ["dvis"], axis=1, **film)
    op("add", ["vis", "dvis"], ["vis_t"], else_alias={"vis_t": "vis"}, **film)
    op("concat", ["flow_t", "vis_t"], ["ft_vt"], axis=1)
    op("convex_upsample", ["h", "ft_vt"], ["up7"], w=["up.w.weight", "up.w.bias"])
    op("slice", ["up7"], ["flow_tq"], a=0, b=4, output=True)
    op("slice", ["up7"], ["vis_tq"], a=4, b=7, output=True)
    ref = dict(cond="use_refine")
    op("scale", ["flow_tq"], ["flow_tq4"], factor=0.25, **ref)
    op("slice", ["flow_tq4"], ["ftq4f"], a=0, b=2, **ref)
    op("slice", ["flow_tq4"], ["ftq4b"], a=2, b=4, **ref)
    op("warp", ["aq", "ftq4f"], ["rwa"], **ref)
    op("warp", ["bq", "ftq4b"], ["rwb"], **ref)
    op("blend_weights", ["vis_tq"], ["bwA", "bwB"], **ref)
    op("mul", ["rwa", "bwA"], ["bt1"], **ref)
    op("mul", ["rwb", "bwB"], ["bt2"], **ref)
    op("add", ["bt1", "bt2"], ["blend"], **ref)
    op("scale", ["flow_tq"], ["flow_tq20"], factor=0.05, **ref)
    op("luma_grad", ["blend"], ["lg"], **ref)
    op("concat", ["rwa", "rwb", "vis_tq", "flow_tq20", "lg"], ["rx"], axis=1, **ref)
    conv("rx", "rq1", "refine.q1", **ref)
    conv("rq1", "rq2", "refine.q2", **ref)
    conv("rq2", "rq3", "refine.q3", **ref)
    conv2d("rq3", "rr", "refine.q4", **ref)
    op("affine_out", ["rr"], ["R_t"], output=True, **ref)
    op("render_pix", ["A", "B", "flow_tq", "vis_tq", "R_t"], ["render"], output=True)
    return ops


def tensor_shapes() -> List[Tuple[str, List[int]]]:
    """Every weight tensor in manifest order with its shape (conv weights are torch [cout][cin][3][3])."""
    t: List[Tuple[str, List[int]]] = []

    def conv(prefix, cin, cout, act=True):
        if act:
            t.extend([(f"{prefix}.0.weight", [cout, cin, 3, 3]), (f"{prefix}.0.bias", [cout]), (f"{prefix}.1.weight", [cout])])
        else:
            t.extend([(f"{prefix}.weight", [cout, cin, 3, 3]), (f"{prefix}.bias", [cout])])

    conv("enc.e1", 3, C8)
    conv("enc.e2", C8, C8)
    conv("enc.e3", C8, C16)
    conv("enc.e4", C16, C16)
    conv("coarse.c1", 2 * C16 + 6 + 4 + 76 + 49, CC)
    conv("coarse.c2", CC, CC)
    conv("coarse.c3", CC, CC)
    conv("coarse.c4", CC, CC)
    conv("coarse.head", CC, 12, act=False)
    conv("fine.r1", 2 * C8 + 6 + 4 + CR + 25, CR)
    conv("fine.r2", CR, CR)
    conv("fine.r3", CR, CR)
    conv("fine.out", CR, 7, act=False)
    conv("up.w", CR, 36, act=False)
    t.extend([("film.film.0.weight", [64, 1]), ("film.film.0.bias", [64]), ("film.film.2.weight", [2 * CR, 64]),
              ("film.film.2.bias", [2 * CR])])
    conv("film.h1", CR, CR)
    conv("film.h2", CR, CR)
    conv("film.out", CR, 5, act=False)
    conv("refine.q1", 14, CQ)
    conv("refine.q2", CQ, CQ)
    conv("refine.q3", CQ, CQ)
    conv("refine.q4", CQ, 3, act=False)
    return t


def manifest(shapes: List[Tuple[str, List[int]]]) -> dict:
    tensors: Dict[str, dict] = {}
    off = 0
    for name, shape in shapes:
        tensors[name] = {"shape": shape, "offset": off, "dtype": "f16"}
        off += int(np.prod(shape))
    meta = {"model": "FlyHighFG", "format_version": 1, "source_checkpoint": "synthetic", "train_step": 0,
            "cfg": {"c8": C8, "c16": C16, "cc": CC, "cr": CR, "cq": CQ, "side_ch": 4, "k_default": 2,
                    "cost_radius": 3, "fine_cost_radius": 2},
            "default_K": 2, "K_range": [1, 3], "dtype": "f16", "bytes_per_elem": 2, "endian": "little",
            "n_tensors": len(shapes), "n_params": off, "render_sampling": "bicubic"}
    return {"meta": meta, "tensors": tensors}


def write(directory: str, seed: int = 0, std: float = 0.05) -> str:
    """Writes graph.json, flyhighfg.json and flyhighfg.bin (seeded N(0, std) f16 weights) into `directory`."""
    os.makedirs(directory, exist_ok=True)
    shapes = tensor_shapes()
    man = manifest(shapes)
    graph = {"meta": {"model": "FlyHighFG", "format_version": 1, "weights": "flyhighfg.bin/.json"}, "ops": graph_ops()}
    rng = np.random.default_rng(seed)
    total = man["meta"]["n_params"]
    w = (rng.standard_normal(total, dtype=np.float32) * np.float32(std)).astype("<f2")
    with open(os.path.join(directory, "graph.json"), "w") as f:
        json.dump(graph, f, indent=1)
    with open(os.path.join(directory, "flyhighfg.json"), "w") as f:
        json.dump(man, f, indent=1)
    w.tofile(os.path.join(directory, "flyhighfg.bin"))
    return directory


def default_dir(seed: int = 0) -> str:
    """A cached synthetic model directory under the user's cache (created on first use)."""
    base = os.environ.get("FLYHIGH_SYNTH_DIR") or os.path.join(os.path.expanduser("~"), ".cache", "flyhigh_b200")
    d = os.path.join(base, f"synthetic-seed{seed}")
    if not os.path.exists(os.path.join(d, "flyhighfg.bin")):
        write(d, seed)
    return d


if __name__ == "__main__":
    import sys
    print(write(sys.argv[1] if len(sys.argv) > 1 else "synthetic_model", int(sys.argv[2]) if len(sys.argv) > 2 else 0))
