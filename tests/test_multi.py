"""Multi-GPU sharding of frame intervals (flyhigh_engine_b200.multi): no collective on the data path; the host-side
logic runs as two gloo ranks on the CPU, and on one GPU a rank's chunk with its static-state replay reproduces a
single session's run of the whole stream bit for bit."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flyhigh_engine_b200.multi import shard


def test_shard_covers_every_interval_once():
    for n in (0, 1, 7, 119, 120):
        for ws in (1, 2, 3, 8):
            parts = [shard(n, ws, r) for r in range(ws)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(parts[r][1] == parts[r + 1][0] for r in range(ws - 1))
            sizes = [e - s for s, e in parts]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard(10, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, ws, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    s, e = shard(119, ws, rank)
    owned = torch.zeros(119, dtype=torch.int32)
    owned[s:e] = 1
    dist.all_reduce(owned)  # every interval owned by exactly one rank
    t = torch.tensor([float(rank + 1) * 10.0])  # a rank's step time; the job time is the max over ranks
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    q.put((rank, owned.tolist(), float(t.item()), (s, e)))
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(v == 1 for v in res[0][1]) and res[0][1] == res[1][1]
    assert res[0][2] == res[1][2] == 20.0
    assert res[0][3] == (0, 60) and res[1][3] == (60, 119)


@pytest.mark.gpu
def test_chunk_with_static_replay_matches_one_session(synth_model_dir):
    import flyhigh_engine_b200 as fh
    from flyhigh_engine_b200 import synth_frames
    from flyhigh_engine_b200.multi import run_stream_chunk
    frames = synth_frames.sequence_c2(13, 640, 360, seed=9)
    eng = fh.Engine()
    model = fh.Model(synth_model_dir)
    whole = {}
    run_stream_chunk(fh.Session(eng, model, 640, 360), frames, 1, 0, 0.5, lambda i, f: whole.__setitem__(i, f))
    assert sorted(whole) == list(range(1, 13))
    for rank in (0, 1):
        part = {}
        got = run_stream_chunk(fh.Session(eng, model, 640, 360), frames, 2, rank, 0.5,
                               lambda i, f: part.__setitem__(i, f))
        assert got == list(range(1 + 6 * rank, 7 + 6 * rank))
        for i in got:
            assert part[i] == whole[i], f"interval {i} of rank {rank} differs"
