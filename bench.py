"""Benchmark of the FlyHighFG Core hot path (Session::pair + Session::mid) on B200: 1080p generated frames/s.

Workload: a seeded 120-frame 1920 x 1080 sequence (pan random walk, 5 moving rectangles, a
static HUD), one pair() + one mid(0.5) per interval = 119 generated frames per step; default session options
(k 1, repair 1, bicubic render, static protection on, still test on), weights seeded N(0, 0.05) f16 of the FlyHighFG
shapes. One step = the whole sequence.

  value : frames/s with the 120 source frames resident in HBM when the timed region starts (each interval copies its
          new frame device-to-device into a session slot, then pair + mid); CUDA events on the session's stream.
  e2e   : the same through the C ABI with host buffers, every interval: the upload of its frame from pinned host
          memory (fh_session_write_rgba_async), fh_session_pair, fh_session_mid, the readback of a generated frame into
          pinned host memory (fh_session_read_rgba_async, waited for before its buffer is reused and by the end of the
          step). `e2e.blocking_calls` is the reference's own call pattern (fh_session_write_rgba / read_rgba, each
          returning once its copy has landed).
The sequence (1 GB) is larger than L2 (126 MB), so no explicit flush is needed between timed steps.

Further keys of the line: `strong` (one 120-frame stream split by interval over the ranks, each replaying the
static-age pass over its prefix: strong scaling), `config4_streams` (config 4: 64 streams through the Stream layer,
sharded by stream), `e2e.copy_ceiling` (the e2e loop's bytes with no compute, serial and
overlapped; e2e as a fraction of the overlapped ceiling, the blocking calls' of the serial one), `roofline` (k_render against HBM: algorithmic bytes, design
bytes, DRAM traffic from its ncu summary), `roofline_conv` (every conv of a batch against the tensor peak),
`conv_sweep` (config 1: each isolated conv shape on both conv kernels), `config3_4k` (3840 x 2160 latency of a pair
and three phases), `camera_warp` (the camera warp's measurement latency and render time at 1080p and 4K), `fast_render_linear_t`, `conv_kernels` (the autotuned kernel of each layer), `kernel_ms`.

Multi-GPU (torchrun, one process per GPU): every rank runs its own seeded sequence (weak scaling, no collective on
the data path); the step time is the max over ranks. --impl reference times the reference algorithm's CPU
restatement (oracle/; the reference itself cannot be built or run here) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "1080p generated frames/s (1 GPU and 1/2/4/8 box); device us per pair()/mid()"
W, H, NFRAMES = 1920, 1080, 120


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="b200", choices=["b200", "reference"])
    p.add_argument("--frames", type=int, default=NFRAMES)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-strong", action="store_true", help="skip the strong-scaling arm")
    p.add_argument("--no-c4", action="store_true", help="skip config 4 (the multi-stream Stream-layer run)")
    p.add_argument("--cpu-sample", type=int, default=3, help="intervals of the CPU baseline sample")
    p.add_argument("--batch", type=int, default=16,
                   help="intervals per launch (fh_session_create_batched); 1 = one interval per launch")
    p.add_argument("--e2e-ring", type=int, default=32, help="pinned host buffers the e2e loop reads generated frames into")
    p.add_argument("--e2e-lag", type=int, default=3,
                   help="the e2e loop reads each interval's frame this many batches after submitting it (3 measured "
                        "about 5 %% above 2: a third batch in flight covers the copy of the last one)")
    return p.parse_args()


class Clocks:
    """nvidia-smi samples of the SM clock and throttle reasons during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self._stop = threading.Event()
        self._t = None

    def __enter__(self):
        def run():
            q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap")
            while not self._stop.is_set():
                try:
                    out = subprocess.run(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits"], capture_output=True, text=True,
                                         timeout=5).stdout.strip()
                    if out:
                        self.samples.append([x.strip() for x in out.split(",")])
                except Exception:
                    pass
                self._stop.wait(0.2)

        self._t = threading.Thread(target=run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [v for v in (num(s[0]) for s in self.samples) if v is not None]
        mx = [v for v in (num(s[1]) for s in self.samples) if v is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4)
                          if len(s) > 3 + i and s[3 + i].strip() == "Active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


def dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


WORKLOAD = ("FlyHighFG Core 1920x1080, 120-frame sequence, pair + mid(0.5) per interval (config 2), internal 864x480, "
            "k 1, repair 1, bicubic, static protection on")


def host_threads() -> int:
    """All host cores this process may use for the oracle (torchrun sets OMP_NUM_THREADS=1 for its workers); returns
    the threads in force."""
    from oracle import oracle
    try:
        n = len(os.sched_getaffinity(0))
    except AttributeError:
        n = os.cpu_count() or 1
    return oracle.threads(n)


def cpu_baseline(model_dir, frames, n_intervals):
    """The oracle (the reference algorithm restated in C++, OpenMP over all host cores) on the first n intervals."""
    from oracle import oracle
    from oracle.oracle import OracleModel, OracleSession
    host_threads()
    om = OracleModel(model_dir)
    o = OracleSession(om, W, H)
    o.pair(frames[0], frames[1])  # warm the caches once
    o.mid(0.5)
    t0 = time.perf_counter()
    for i in range(1, n_intervals + 1):
        o.pair(frames[i - 1], frames[i])
        o.mid(0.5)
    dt = time.perf_counter() - t0
    return n_intervals / dt, dt


def cpu_baseline_warp(w=1920, h=1080):
    """The camera warp's CPU restatement (oracle camwarp) on the host cores at w x h: one measurement of a panned pair
    (cells, the three levels, lock, dilate; one thread) and one render (OpenMP over the cores), ms each."""
    from oracle import oracle
    from flyhigh_engine_b200 import synth_frames
    fr = synth_frames.sequence_c2(2, w, h, seed=5)
    t0 = time.perf_counter()
    best, _, grown, _ = oracle.warp_measure(fr[0], fr[1], w, h)
    t1 = time.perf_counter()
    oracle.warp_render(fr[1], w, h, grown, 30.0, -5.0)
    t2 = time.perf_counter()
    return {"measure_ms": (t1 - t0) * 1000.0, "render_ms": (t2 - t1) * 1000.0, "kind": "port",
            "cores": host_threads(), "sample": f"one config-2 pair at {w}x{h}"}


def run_reference(args):
    ws, rank, _ = dist()
    if rank != 0:
        return 0
    from flyhigh_engine_b200 import synth_frames, synth_model
    model_dir = synth_model.default_dir(0)
    frames = synth_frames.sequence_c2(max(args.cpu_sample + 1, 4), W, H, seed=0)
    cores = host_threads()
    times = []
    for _ in range(args.warmup):
        cpu_baseline(model_dir, frames, 1)
    for _ in range(args.steps):
        _fps, dt = cpu_baseline(model_dir, frames, args.cpu_sample)
        times.append(dt / args.cpu_sample)
    ms = float(np.max(times) * 1000.0)
    fps = 1000.0 / ms
    line = {"impl": "reference", "metric": METRIC, "value": fps, "unit": "generated frames/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms * args.cpu_sample,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (seeded config-2 frames, seeded N(0,0.05) weights)",
            "config": {"workload": WORKLOAD, "sample": f"{args.cpu_sample} intervals per step"},
            "cpu_baseline": {"value": fps, "unit": "generated frames/s", "cores": cores, "kind": "port",
                             "sample": f"{args.cpu_sample} consecutive 1080p intervals (pair + mid) per step; the "
                                       "reference (Rust + wgpu/WGSL) cannot be built or run here: no Rust toolchain, "
                                       "no graphics stack"},
            "e2e": {"value": fps, "unit": "generated frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    ws, rank, local = dist()
    import torch
    torch.cuda.set_device(local)
    pg = None
    if ws > 1:
        import datetime
        import torch.distributed as tdist
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
        pg = tdist
    import flyhigh_engine_b200 as fh
    from flyhigh_engine_b200 import synth_frames, synth_model

    model_dir = synth_model.default_dir(0)
    n = args.frames
    frames = synth_frames.sequence_c2(n, W, H, seed=100 + rank)
    fbytes = W * H * 4
    dev_frames = torch.from_numpy(np.stack(frames)).to(f"cuda:{local}")  # [n][h][w][4], resident in HBM
    engine = fh.Engine(adapter=f"#{local}")
    model = fh.Model(model_dir)
    s = fh.Session(engine, model, W, H, batch=args.batch)
    slots = [s.add_input(), s.add_input()]
    out = s.add_output()
    stream = torch.cuda.ExternalStream(s.cuda_stream(), device=f"cuda:{local}")
    base = dev_frames.data_ptr()

    def step_device():
        s.write_device(slots[0], base, fbytes)
        for i in range(1, n):
            a, b = slots[(i - 1) % 2], slots[i % 2]
            s.write_device(b, base + i * fbytes, fbytes)
            s.pair(a, b)
            s.mid(0.5, out)
        # a batched session renders on a stream of its own: the step's end event on the session stream comes after
        # every render issued in the step
        s.join()

    def barrier():
        torch.cuda.synchronize()
        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize()

    def timed(fn, k):
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(k):
            fn()
        e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / k
        barrier()
        if pg is not None:
            t = torch.tensor([ms], device=f"cuda:{local}")
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    warm = max(args.warmup, 3)
    for _ in range(warm):
        step_device()
    k0 = s.kernel_launches()
    with Clocks(local) as clk:
        ms = timed(step_device, args.steps)
    launches = s.kernel_launches() - k0  # this rank's kernels in the timed steps
    gen_per_rank = n - 1
    value = gen_per_rank * ws / (ms / 1000.0)

    # strong scaling: ONE 120-frame stream (the same seeded sequence on every rank) split into contiguous interval
    # shards; a rank whose shard starts at interval s first replays the static-age pass over intervals 1..s
    # (fh_session_advance_static), so its protection state equals a single GPU's; the replay is inside the timed region
    strong = None
    if not args.no_strong:
        from flyhigh_engine_b200.multi import shard
        one = synth_frames.sequence_c2(n, W, H, seed=100) if ws > 1 else frames
        one_dev = torch.from_numpy(np.stack(one)).to(f"cuda:{local}") if ws > 1 else dev_frames
        s0, e0 = shard(n - 1, ws, rank)
        ss = fh.Session(engine, model, W, H, batch=args.batch)
        sslots = [ss.add_input(), ss.add_input()]
        sout = ss.add_output()
        sbase = one_dev.data_ptr()

        def step_strong():
            ss.write_device(sslots[0], sbase, fbytes)
            for i in range(1, s0 + 1):
                ss.write_device(sslots[i % 2], sbase + i * fbytes, fbytes)
                ss.advance_static(sslots[(i - 1) % 2], sslots[i % 2])
            for i in range(s0 + 1, e0 + 1):
                ss.write_device(sslots[i % 2], sbase + i * fbytes, fbytes)
                ss.pair(sslots[(i - 1) % 2], sslots[i % 2])
                ss.mid(0.5, sout)
            ss.join()

        sstream = torch.cuda.ExternalStream(ss.cuda_stream(), device=f"cuda:{local}")

        def timed_on(fn, k, strm):
            barrier()
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record(strm)
            for _ in range(k):
                fn()
            ev1.record(strm)
            ev1.synchronize()
            t_ms = ev0.elapsed_time(ev1) / k
            barrier()
            if pg is not None:
                t = torch.tensor([t_ms], device=f"cuda:{local}")
                pg.all_reduce(t, op=pg.ReduceOp.MAX)
                t_ms = float(t.item())
            return t_ms

        for _ in range(warm):
            step_strong()
        strong_ms = timed_on(step_strong, args.steps, sstream)
        strong = {"value": (n - 1) / (strong_ms / 1000.0), "unit": "generated frames/s", "scaling": "strong",
                  "ms_per_step": strong_ms, "intervals": n - 1, "this_rank": [s0, e0],
                  "replayed_intervals_max": (ws - 1) * (n - 1) // ws,
                  "workload": "one 120-frame config-2 stream split by interval over the ranks, each replaying the "
                              "static-age pass over its prefix (device-resident frames)"}
        del ss
        if ws > 1:
            del one_dev

    # device ms per pair() and per mid() (the reference's pair_timed / mid_timed: min of 3 / 5 runs)
    pair_ms = s.pair_timed(slots[0], slots[1])
    mid_ms = s.mid_timed(0.5, out)

    # end to end through the C ABI with host buffers
    e2e = None
    if not args.no_e2e:
        pinned = torch.empty((n, H, W, 4), dtype=torch.uint8).pin_memory()
        pinned.copy_(torch.from_numpy(np.stack(frames)))
        pin_np = pinned.numpy()
        outbuf = torch.empty((H, W, 4), dtype=torch.uint8).pin_memory()
        out_np = outbuf.numpy()

        lag = 1 if args.batch <= 1 else args.e2e_lag * args.batch
        outs = [out] + [s.add_output() for _ in range(2 * lag - 1)]

        RING = args.e2e_ring  # host buffers of generated frames (32: a second of output at 30 fps, what a host queues)
        ring = torch.empty((RING, H, W, 4), dtype=torch.uint8).pin_memory()
        ring_np = [ring[k].numpy() for k in range(RING)]

        def step_host():
            # the reference's call sequence per interval (write, pair, mid, read), reading each interval's frame `lag`
            # intervals later (2 x lag output slots): the read overlaps the next intervals' compute; with a batched
            # session it reads the batch before the one on the GPU while the next one is queued. write_rgba and
            # read_rgba return once their copy has landed, so one host thread serialises the two directions.
            s.write(slots[0], pin_np[0])
            for i in range(1, n):
                a, b = slots[(i - 1) % 2], slots[i % 2]
                s.write(b, pin_np[i])
                s.pair(a, b)
                s.mid(0.5, outs[i % (2 * lag)])
                if i > lag:
                    s.read_into(outs[(i - lag) % (2 * lag)], out_np)
            for i in range(max(1, n - lag), n):
                s.read_into(outs[i % (2 * lag)], out_np)

        # the same calls with the asynchronous copies of flyhigh_b200.h: uploads from the pinned frames, readbacks into
        # a ring of pinned buffers, each frame waited for (in the host's hands) before its buffer is reused. Steps
        # follow each other as a stream's intervals do: the next step's uploads start while the last readbacks of
        # this one land; every step's copies are waited for inside the timed region (drain).
        ring_held = [None] * RING
        ring_n = [0]

        def read(slot):
            k = ring_n[0] % RING
            if ring_held[k] is not None:
                s.read_wait(ring_held[k])
            s.read_async(slot, ring_np[k])
            ring_held[k] = slot
            ring_n[0] += 1

        def drain():
            for k, slot in enumerate(ring_held):
                if slot is not None:
                    s.read_wait(slot)
                ring_held[k] = None

        def step_host_async():
            s.write_async(slots[0], pin_np[0])
            for i in range(1, n):
                a, b = slots[(i - 1) % 2], slots[i % 2]
                s.write_async(b, pin_np[i])
                s.pair(a, b)
                s.mid(0.5, outs[i % (2 * lag)])
                if i > lag:
                    read(outs[(i - lag) % (2 * lag)])
            for i in range(max(1, n - lag), n):
                read(outs[i % (2 * lag)])

        def timed(step, end=lambda: None):
            step()
            end()
            barrier()
            t0 = time.perf_counter()
            for _ in range(args.steps):
                step()
            end()
            torch.cuda.synchronize()
            ms = (time.perf_counter() - t0) * 1000.0 / args.steps
            if pg is not None:
                t = torch.tensor([ms], device=f"cuda:{local}")
                pg.all_reduce(t, op=pg.ReduceOp.MAX)
                ms = float(t.item())
            return ms

        e2e_ms = timed(step_host_async, drain)
        e2e = {"value": gen_per_rank * ws / (e2e_ms / 1000.0), "unit": "generated frames/s",
               "h2d_bytes_per_step": n * fbytes, "d2h_bytes_per_step": gen_per_rank * fbytes,
               "ms_per_step": e2e_ms,
               "calls": "write_rgba_async / pair / mid / read_rgba_async + read_wait (flyhigh_b200.h), pinned buffers; "
                        "steps back to back, every copy waited for inside the timed region"}
        blk_ms = timed(step_host)
        e2e["blocking_calls"] = {"value": gen_per_rank * ws / (blk_ms / 1000.0), "unit": "generated frames/s",
                                 "ms_per_step": blk_ms,
                                 "calls": "write_rgba / pair / mid / read_rgba (the reference's flyhigh.h), pinned"}

        # The copy ceiling of this call pattern: the same bytes between the same pinned buffers and the device with no
        # compute, one host thread per rank. "serial": each copy waited for before the next call, as write_rgba and
        # read_rgba wait for theirs; "overlapped": uploads and readbacks on two streams at once, what the link and host
        # memory allow. Max over ranks, wall clock as e2e.
        cin_dev = torch.empty((H, W, 4), dtype=torch.uint8, device=f"cuda:{local}")
        cout_dev = torch.empty_like(cin_dev)
        up_s, dn_s = torch.cuda.Stream(device=f"cuda:{local}"), torch.cuda.Stream(device=f"cuda:{local}")

        def step_copy(overlapped):
            for i in range(n):
                with torch.cuda.stream(up_s):
                    cin_dev.copy_(pinned[i], non_blocking=True)
                if not overlapped:
                    up_s.synchronize()
                if i > 0:
                    with torch.cuda.stream(dn_s):
                        outbuf.copy_(cout_dev, non_blocking=True)
                    if not overlapped:
                        dn_s.synchronize()
            up_s.synchronize()
            dn_s.synchronize()

        copy = {}
        for mode in ("serial", "overlapped"):
            step_copy(mode == "overlapped")
            barrier()
            t0 = time.perf_counter()
            for _ in range(args.steps):
                step_copy(mode == "overlapped")
            c_ms = (time.perf_counter() - t0) * 1000.0 / args.steps
            if pg is not None:
                t = torch.tensor([c_ms], device=f"cuda:{local}")
                pg.all_reduce(t, op=pg.ReduceOp.MAX)
                c_ms = float(t.item())
            copy[mode] = {"value": gen_per_rank * ws / (c_ms / 1000.0), "ms_per_step": c_ms,
                          "gb_per_s_per_rank": (n + gen_per_rank) * fbytes / (c_ms / 1000.0) / 1e9}
        e2e["copy_ceiling"] = copy
        e2e["frac_of_overlapped_copy_ceiling"] = e2e["value"] / copy["overlapped"]["value"]
        e2e["blocking_calls"]["frac_of_serial_copy_ceiling"] = e2e["blocking_calls"]["value"] / copy["serial"]["value"]

    # per-kernel device times on the session's own stream (min over 5 eager runs): one batch of `batch` intervals for a
    # batched session (the frame stage of its batch + 1 frames, its pairs and mids), else one pair + mid
    nb = max(args.batch, 1)
    prof = {}
    for _ in range(5):
        seen_this_run = {}
        run = s.profile_batch() if nb > 1 else s.profile(slots[0], slots[1], 0.5, out)
        for k in run:
            key = k["kernel"]
            if key in seen_this_run:  # launched again in the run (the second frame stage, k > 1): its own entry
                key = f"{key} #{seen_this_run[key] + 1}"
            seen_this_run[k["kernel"]] = seen_this_run.get(k["kernel"], 0) + 1
            prof[key] = min(prof.get(key, 1e9), k["ms"])
    roof, roof_conv = roofline_blocks(s, prof, nb)
    if rank == 0:
        total = sum(prof.values())
        for k, v in sorted(prof.items(), key=lambda x: -x[1]):
            print(f"# {v * 1000:8.1f} us {100 * v / total:5.1f}%  {k}", file=sys.stderr)
    # the fast render + linear_t session (texbench's configuration): device ms of one pair and of one further phase
    fast = None
    if not args.no_e2e:
        sf = fh.Session(engine, model, W, H, fast_render=True, linear_t=True)
        fs = [sf.add_input(), sf.add_input()]
        fo = sf.add_output()
        sf.write(fs[0], frames[0])
        sf.write(fs[1], frames[1])
        sf.pair(fs[0], fs[1])
        sf.mid(0.5, fo)
        fast = {"pair_ms": sf.pair_timed(fs[0], fs[1]), "mid_ms": sf.mid_timed(0.25, fo)}
        del sf
    # config 4 through the Stream layer, sharded by stream (every rank, every N)
    c4 = None
    if not args.no_c4:
        try:
            c4 = config4(engine, model, ws, rank, local, barrier, pg)
        except Exception as e:  # a side measurement: reported in the line, not a failed run
            c4 = {"error": str(e)}
            if pg is not None:
                raise
    # config 3's latency and config 1's per-conv sweep (rank 0 of a 1-GPU run; the scaling runs skip them)
    c3 = sweep = cwarp = None
    if rank == 0 and ws == 1 and not args.no_e2e:
        peaks = {}
        try:
            with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
                peaks = json.load(f)
        except Exception:
            pass
        try:  # side measurements: a failure is reported in the line, not as a failed run
            c3 = config3_latency(engine, model)
        except Exception as e:
            c3 = {"error": str(e)}
        try:
            sweep = conv_sweep(f"cuda:{local}", peaks.get("bf16_tflops"))
        except Exception as e:
            sweep = {"error": str(e)}
        try:
            cwarp = camera_warp_timing(engine, peaks.get("hbm_gbs"))
        except Exception as e:
            cwarp = {"error": str(e)}
    cpu = None
    if rank == 0 and ws == 1:
        fps_cpu, dt = cpu_baseline(model_dir, frames, args.cpu_sample)
        cpu = {"value": fps_cpu, "unit": "generated frames/s", "cores": host_threads(), "kind": "port",
               "sample": f"{args.cpu_sample} consecutive intervals of the same 1080p sequence (pair + mid(0.5)), "
                         f"{dt:.1f} s on the host cores"}
        if not args.no_e2e:
            try:  # beside the GPU's camera_warp numbers: the same stages restated on the host cores
                cpu["camera_warp"] = cpu_baseline_warp()
            except Exception as e:
                cpu["camera_warp"] = {"error": str(e)}
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "generated frames/s", "n_gpus": ws, "steps": args.steps,
                "warmup": warm, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f16",
                "data": "synthetic (seeded config-2 frames, seeded N(0,0.05) f16 weights of the FlyHighFG shapes)",
                "config": {"workload": WORKLOAD + "; the reference's per-interval calls on a batched session "
                                                  "(intervals queued and launched `batch` at a time, results identical "
                                                  "to one at a time)",
                           "frames_per_step": gen_per_rank, "l2": "inputs (1 GB of frames) larger than L2, no flush",
                           "batch": args.batch, "pair_ms": pair_ms, "mid_ms": mid_ms},
                "gpu_launches": launches * ws,
                "clocks": clk.summary(), "roofline": roof, "roofline_conv": roof_conv, "cpu_baseline": cpu,
                "e2e": e2e, "strong": strong, "config4_streams": c4, "fast_render_linear_t": fast, "config3_4k": c3,
                "camera_warp": cwarp, "conv_sweep": sweep,
                "conv_kernels": {k: v["kernel"] for k, v in s.report()["convs"].items()},
                "kernel_ms": {k: round(v, 5) for k, v in sorted(prof.items(), key=lambda x: -x[1])[:12]}}
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    return 0


def conv_sweep(device: str, peak_tflops):
    """Config 1: every implicit-GEMM 3x3 conv of the isolated sweep (480x270 and 960x540, Cin / Cout in {16, 32, 48,
    64}, stride 1 and 2, bias + PReLU(0.1), with and without an f16 residual) on both conv kernels where they apply
    (mma.sync at the rows-per-CTA rule; tcgen05 for stride 1), batch 1. Each timed as the mean of 20 back-to-back
    launches (CUDA events on the launching stream, min over 3 trials, after 3 warm-up launches). Returns the per-shape
    records [h, w, cin, cout, stride, residual, best kernel, us, TFLOP/s] and a summary against the tensor peak."""
    import torch
    from flyhigh_engine_b200.kernels import Conv3x3
    rng = np.random.default_rng(1)
    stream = torch.cuda.current_stream()
    rows = []
    for (h, w) in ((270, 480), (540, 960)):
        for cin in (16, 32, 48, 64):
            x = torch.from_numpy(rng.standard_normal((1, h, w, cin)).astype(np.float16)).to(device)
            for cout in (16, 32, 48, 64):
                wt = (rng.standard_normal((cout, cin, 3, 3)) / np.sqrt(9 * cin)).astype(np.float32)
                bias = (0.1 * rng.standard_normal(cout)).astype(np.float32)
                slope = np.full(cout, 0.1, np.float32)
                for stride in (1, 2):
                    for res in (False, True):
                        best = None
                        for kernel in ("mma", "umma") if stride == 1 else ("mma",):
                            conv = Conv3x3(wt, bias, slope, stride=stride, kernel=kernel, device=device)
                            out = torch.zeros(conv.out_shape(1, h, w), dtype=torch.float16, device=device)
                            r = torch.zeros_like(out) if res else None
                            prm = conv.params(x, out, r)
                            for _ in range(3):
                                conv.launch(prm, stream.cuda_stream)
                            ms = 1e9
                            for _ in range(3):
                                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                                e0.record(stream)
                                for _ in range(20):
                                    conv.launch(prm, stream.cuda_stream)
                                e1.record(stream)
                                e1.synchronize()
                                ms = min(ms, e0.elapsed_time(e1) / 20)
                            if best is None or ms < best[1]:
                                best = (kernel, ms)
                        ho, wo = (h - 1) // stride + 1, (w - 1) // stride + 1
                        tflops = 2.0 * ho * wo * 9 * cin * cout / (best[1] / 1000.0) / 1e12
                        rows.append([h, w, cin, cout, stride, int(res), best[0], round(best[1] * 1000, 2),
                                     round(tflops, 2)])
    top = max(rows, key=lambda r: r[8])
    return {"fields": ["h", "w", "cin", "cout", "stride", "residual", "kernel", "us", "tflops"], "rows": rows,
            "best": {"shape": top[:6], "kernel": top[6], "us": top[7], "tflops": top[8],
                     "frac": top[8] / peak_tflops if peak_tflops else None},
            "note": "batch 1, inputs L2-resident (<= 66 MB), mean of 20 back-to-back launches"}


def config3_latency(engine, model):
    """Config 3 (3840 x 2160, 4x: a pair and phases 0.25 / 0.5 / 0.75) on a session run one interval at a time: device
    ms of pair() and of each mid() (the reference's pair_timed / mid_timed: min of 3 / 5 runs) on seeded fence-pan
    frames, and ms per generated frame = (pair + three mids) / 3."""
    import flyhigh_engine_b200 as fh
    from flyhigh_engine_b200 import synth_frames
    w4, h4 = 3840, 2160
    fr = synth_frames.sequence_c3(2, w4, h4, seed=3)
    s = fh.Session(engine, model, w4, h4)
    a, b, out = s.add_input(), s.add_input(), s.add_output()
    s.write(a, fr[0])
    s.write(b, fr[1])
    s.pair(a, b)
    s.mid(0.5, out)
    pair_ms = s.pair_timed(a, b)
    mids = [s.mid_timed(t, out) for t in (0.25, 0.5, 0.75)]
    del s
    return {"workload": "3840x2160, pair + mid(0.25 / 0.5 / 0.75), one interval per launch, fence pan frames",
            "pair_ms": pair_ms, "mid_ms": mids, "ms_per_generated_frame": (pair_ms + sum(mids)) / 3.0}


def camera_warp_timing(engine, hbm_gbs):
    """The camera warp (fh_warp_*) at 1080p (config-2 frames) and 4K (config 3's fence pan): the latency of one frame's
    measurement (frame() to its shift in the host's hands: a cells launch, three search launches, lock, dilate, the
    16-byte readback; host clock, median of 8) and the device time of one render (k_warp_render, CUDA events on the
    warp's stream, mean of 20) with its bytes: the source frame read once and the turned frame written."""
    import torch
    import flyhigh_engine_b200 as fh
    from flyhigh_engine_b200 import synth_frames
    res = {}
    for w, h, frames in ((1920, 1080, synth_frames.sequence_c2(9, 1920, 1080, seed=5)),
                         (3840, 2160, synth_frames.sequence_c3(9, 3840, 2160, seed=5))):
        dev = torch.from_numpy(np.stack(frames)).cuda()
        dst = torch.empty_like(dev[0])
        torch.cuda.synchronize()
        with fh.Warp(engine, w, h) as wp:
            wp.frame(dev[0].data_ptr(), 0.0)
            wp.collect(True)
            lat = []
            for i in range(1, 9):
                torch.cuda.synchronize()
                t0 = time.perf_counter()
                wp.frame(dev[i].data_ptr(), 16.7 * i)
                wp.collect(True)
                lat.append((time.perf_counter() - t0) * 1000.0)
            st = torch.cuda.ExternalStream(wp.cuda_stream())
            for _ in range(3):
                wp.render_into(dev[8].data_ptr(), dst.data_ptr(), 30.0, -5.0)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            for _ in range(20):
                wp.render_into(dev[8].data_ptr(), dst.data_ptr(), 30.0, -5.0)
            e1.record(st)
            e1.synchronize()
            rms = e0.elapsed_time(e1) / 20
            gbs = 2 * w * h * 4 / (rms / 1000.0) / 1e9
            res[f"{w}x{h}"] = {"measure_ms": float(np.median(lat)), "render_ms": rms, "render_gb_per_s": gbs,
                               "render_frac_of_hbm": gbs / hbm_gbs if hbm_gbs else None,
                               "last_shift": wp.last_shift()}
        del dev, dst
    return res


def c4_pool(device, scenes=5, per_scene=48, seed=400):
    """Config 4's source frames, made on the GPU: `scenes` seeded scenes of `per_scene` 1080p frames each, with the
    statistics of the config-2 generator (a texture of 8 random sinusoids, periods 8-128 px, uniform noise of +-10; a pan
    whose velocity random-walks by +-2 px per frame; 5 rectangles of 20-80 px moving independently). [scenes *
    per_scene][H][W][4] uint8 on `device`."""
    import torch
    out = torch.empty((scenes * per_scene, H, W, 4), dtype=torch.uint8, device=device)
    m = 24 * per_scene // 4 + 64
    yy = torch.arange(H + 2 * m, device=device, dtype=torch.float32)[:, None]
    xx = torch.arange(W + 2 * m, device=device, dtype=torch.float32)[None, :]
    for k in range(scenes):
        rng = np.random.default_rng(seed + k)
        tex = torch.full((H + 2 * m, W + 2 * m, 3), 128.0, device=device)
        for _ in range(8):
            period, ang, phase = rng.uniform(8.0, 128.0), rng.uniform(0.0, np.pi), rng.uniform(0.0, 2 * np.pi)
            amp = torch.tensor(rng.uniform(10.0, 30.0, size=3), dtype=torch.float32, device=device)
            kx, ky = float(np.cos(ang) * 2 * np.pi / period), float(np.sin(ang) * 2 * np.pi / period)
            tex += torch.sin(kx * xx + ky * yy + phase)[..., None] * amp
        rects = [dict(x=int(rng.integers(0, W - 80)), y=int(rng.integers(0, H - 80)), w=int(rng.integers(20, 81)),
                      h=int(rng.integers(20, 81)), v=rng.integers(-3, 4, size=2),
                      c=torch.tensor(rng.integers(0, 256, size=3), dtype=torch.float32, device=device))
                 for _ in range(5)]
        gen = torch.Generator(device=device).manual_seed(seed + k)
        px = py = vx = vy = 0
        for i in range(per_scene):
            vx = int(np.clip(vx + rng.integers(-2, 3), -24, 24))
            vy = int(np.clip(vy + rng.integers(-2, 3), -24, 24))
            px, py = int(np.clip(px + vx, -m, m)), int(np.clip(py + vy, -m, m))
            img = tex[m + py:m + py + H, m + px:m + px + W].clone()
            for r in rects:
                r["x"] += int(r["v"][0])
                r["y"] += int(r["v"][1])
                x0, y0 = max(0, r["x"]), max(0, r["y"])
                x1, y1 = min(W, r["x"] + r["w"]), min(H, r["y"] + r["h"])
                if x0 < x1 and y0 < y1:
                    img[y0:y1, x0:x1] = r["c"]
            img += torch.rand(img.shape, generator=gen, device=device) * 20.0 - 10.0
            out[k * per_scene + i, ..., :3] = img.clamp_(0, 255).to(torch.uint8)
            out[k * per_scene + i, ..., 3] = 255
    return out


def config4(engine, model, ws, rank, local, barrier, pg, streams_total=64, frames=240, phases=(0.2, 0.4, 0.6, 0.8)):
    """Config 4: 64 independent 1080p streams of 240 source frames each (24 -> 120 fps: four mids per interval), a scene
    cut every 48 frames, 2-frame held runs every 30 frames, through the Stream layer (realtime, scene cuts at the
    default threshold, held frames on), sharded by stream over the ranks with no collective. Per frame and stream: the
    next input slot, the frame (device-resident pool), classify, push, and the four mids when the pair is motion (cuts
    and holds show source frames). One pass, wall clock from a barrier to the synchronize after the last call, max over
    ranks."""
    import torch
    import flyhigh_engine_b200 as fh
    from flyhigh_engine_b200 import synth_frames
    from flyhigh_engine_b200.multi import shard
    dev = f"cuda:{local}"
    pool = c4_pool(dev)
    fbytes = W * H * 4
    base = pool.data_ptr()
    s0, s1 = shard(streams_total, ws, rank)
    sts = [fh.Stream(engine, model, W, H, held_frames=True) for _ in range(s0, s1)]
    orders = [synth_frames.stream_c4(frames, 48, 30, scenes=5, offset=k) for k in range(s0, s1)]
    for st in sts:  # every graph built before the timed pass: the ring's four pairs, each into the four outputs
        prev_w = None
        for i in range(5):
            slot = st.next_input([] if prev_w is None else [prev_w])
            st.write_device(slot, base + i * fbytes, fbytes)
            if st.push(slot, float(i)).ready:
                for j, t in enumerate(phases):
                    st.generate(t, j)
            prev_w = slot
        st.reset()
    torch.cuda.synchronize()
    counts = {"motion": 0, "cut": 0, "hold": 0}
    mids = 0
    prev = [None] * len(sts)
    barrier()
    t0 = time.perf_counter()
    for f in range(frames):
        for k, st in enumerate(sts):
            sc, j = orders[k][f]
            slot = st.next_input([] if prev[k] is None else [prev[k]])
            st.write_device(slot, base + (sc * 48 + j) * fbytes, fbytes)
            kind = None
            if prev[k] is not None:
                c = st.classify(prev[k], slot)
                kind = c.kind if c is not None else "motion"
                counts[kind] += 1
            p = st.push(slot, f * 1000.0 / 24.0)
            if p.ready and kind == "motion":
                for j2, t in enumerate(phases):
                    st.generate(t, j2)
                mids += len(phases)
            prev[k] = slot
    torch.cuda.synchronize()
    ms = (time.perf_counter() - t0) * 1000.0
    tot = torch.tensor([ms, float(mids), float(frames * len(sts))], device=dev, dtype=torch.float64)
    if pg is not None:
        t = tot[:1].clone()
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        s = tot[1:].clone()
        pg.all_reduce(s, op=pg.ReduceOp.SUM)
        tot = torch.cat([t, s])
    ms, mids_all, src_all = float(tot[0]), float(tot[1]), float(tot[2])
    del sts, pool
    torch.cuda.empty_cache()
    return {"workload": "64 streams x 240 frames at 1920x1080, 24 -> 120 fps (mids at 0.2 / 0.4 / 0.6 / 0.8), scene cut "
                        "every 48 frames, 2-frame holds every 30, realtime Stream with held-frame detection, sharded by "
                        "stream", "streams": streams_total, "streams_this_rank": s1 - s0,
            "generated_frames_per_s": mids_all / (ms / 1000.0), "source_frames_per_s": src_all / (ms / 1000.0),
            "ms": ms, "generated": int(mids_all), "pairs_by_kind_this_rank": counts, "scaling": "strong",
            "timing": "wall clock from a barrier to the device synchronize after the last call, max over ranks"}


def conv_flops(s, nb: int) -> float:
    """2 * M * 9 * cin * cout summed over the convs of one profiled run at this session's sizes: the encoders of nb + 1
    frames (both frames of one pair when nb is 1, as the reference computes them every pair) and the pair + mid convs
    of nb intervals."""
    p = s._m.plan_params(W, H)
    q, e8, e16 = p["qh"] * p["qw"], p["h8"] * p["w8"], p["h16"] * p["w16"]
    encoder = [(e8, 3, 36), (e8, 36, 36), (e16, 36, 72), (e16, 72, 72)]  # (pixels, cin, cout)
    interval = [
        (e16, 279, 96), (e16, 96, 96), (e16, 96, 96), (e16, 96, 96), (e16, 96, 12),
        (e8, 155, 48), (e8, 48, 48), (e8, 48, 48), (e8, 48, 7),
        (e8, 48, 48), (e8, 48, 48), (e8, 48, 5), (e8, 48, 36),
        (q, 14, 24), (q, 24, 24), (q, 24, 24), (q, 24, 3)]

    def fl(cs):
        return float(sum(2 * m * 9 * ci * co for m, ci, co in cs))
    return fl(encoder) * (nb + 1) + fl(interval) * nb


def render_bytes(p) -> float:
    """Algorithmic bytes of one full-resolution render as the hot-path measurement defines them: the two source frames
    read once (B, G, R as f16, 12 B/px), the quarter-resolution flow / visibility (7 ch) and residual (3 ch) maps (f16)
    read once, the rgba8 frame written (4 B/px)."""
    q = p["qh"] * p["qw"]
    return float(W * H * (12 + 4) + q * (7 + 3) * 2)


def render_design_bytes(p) -> float:
    """Bytes this design's render reads beyond the algorithmic ones: the own-pixel word of the padded plane that
    k_static_planes writes (near, the keep_static ramp and the still test's mean in 32 bits, 4 B/px)."""
    return float(p["hp"] * p["wp"] * 4)


RENDER_PROFILE = os.path.join(ROOT, "profiles", "k_render_1080p.md")


def render_traffic():
    """DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per rendered 1920 x 1080 frame of the current k_render,
    from the ncu capture that profiles/k_render_1080p.md summarises (its 'traffic per frame' line), with the capture's
    description; (None, reason) when the summary is missing."""
    import re
    try:
        with open(RENDER_PROFILE) as f:
            text = f.read()
    except OSError:
        return None, "no ncu summary"
    m = re.search(r"traffic per frame \(read \+ write\): ([0-9.]+) MB", text)
    c = re.search(r"capture: (.+)", text)
    if not m:
        return None, "no traffic line in the ncu summary"
    return float(m.group(1)) * 1e6, (c.group(1).strip() if c else "profiles/k_render_1080p.md")


def roofline_blocks(s, prof, nb):
    """The roofline of the HBM-bound render (the step's largest memory-bound kernel) and of the convs together, from
    the profiled run's per-kernel device times: nb frames per render launch, nb + 1 encoders and nb intervals of
    convs."""
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except Exception:
        pass
    p = s._m.plan_params(W, H)
    hbm = peaks.get("hbm_gbs")
    tensor = peaks.get("bf16_tflops")
    name, kms = ("render", prof["render"]) if "render" in prof else max(prof.items(), key=lambda kv: kv[1])
    if name == "render":
        alg = render_bytes(p) * nb
        achieved = alg / (kms / 1000.0) / 1e9
        traffic, tsrc = render_traffic()
        roof = {"bound": "hbm", "kernel": f"k_render (full-resolution render + keep_static + rgba8 out), {nb} frame(s) "
                                          "per launch",
                "achieved": achieved, "peak": hbm or 6650.0, "unit": "GB/s",
                "frac": achieved / (hbm or 6650.0), "traffic": traffic * nb if traffic else None,
                "traffic_source": tsrc, "algorithmic_bytes": alg, "design_bytes": render_design_bytes(p) * nb,
                "launch_ms": kms, "frames_per_launch": nb, "peak_source": "measured" if hbm else "fallback"}
    else:
        roof = {"bound": "unknown", "kernel": name, "launch_ms": kms, "achieved": None, "peak": None, "unit": None,
                "frac": None, "traffic": None}
    conv_ms = sum(v for k, v in prof.items() if k.startswith("conv "))
    flops = conv_flops(s, nb)
    ach = flops / (conv_ms / 1000.0) / 1e12
    roof_conv = {"bound": "tensor", "kernel": f"every conv launch of one profiled run ({nb + 1} frame encoders, {nb} "
                                              "interval(s) of pair + mid convs)", "achieved": ach,
                 "peak": tensor or 1590.0, "unit": "TFLOP/s", "frac": ach / (tensor or 1590.0), "flops": flops,
                 "ms": conv_ms, "peak_source": "measured" if tensor else "fallback"}
    return roof, roof_conv


if __name__ == "__main__":
    sys.exit(main())
