"""Multi-GPU execution of frame-interval work: one process per GPU, no collective on the data path.

The intervals of a sequence are independent for the network and the repair stage; only static protection carries
state from pair to pair (keep_static_age.wgsl, net/build.rs:576-603). A stream of n frames is split into contiguous
chunks of intervals, one per rank; a rank whose chunk starts at interval s first replays the static-age pass alone
(Session.advance_static) over the intervals before s, which reproduces the state a single GPU would have at s
exactly. Frames come from and go to host memory per rank. Independent streams (many users, config 4) need no replay:
they are sharded whole.
"""
from __future__ import annotations

from typing import Callable, List, Sequence, Tuple


def shard(n_items: int, world_size: int, rank: int) -> Tuple[int, int]:
    """The contiguous [start, end) of `n_items` owned by `rank` (sizes differ by at most one, earlier ranks larger)."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} of {world_size}")
    base, extra = divmod(n_items, world_size)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def run_stream_chunk(session, frames: Sequence, world_size: int, rank: int, t: float,
                     emit: Callable[[int, object], None], read: bool = True) -> List[int]:
    """This rank's intervals (i - 1, i), i in [start + 1, end + 1), of one stream: replays the static state over the
    prefix, then pair + mid per interval; emit(i, frame) receives each generated frame (bytes) when `read`.
    Returns the interval indices produced."""
    n_int = len(frames) - 1
    s, e = shard(n_int, world_size, rank)
    slots = [session.add_input(), session.add_input()]
    out = session.add_output()
    done = []
    if s == e:
        return done
    # the state at interval s: the age pass over intervals 1 .. s
    session.write(slots[0], frames[0])
    for i in range(1, s + 1):
        a, b = slots[(i - 1) % 2], slots[i % 2]
        session.write(b, frames[i])
        session.advance_static(a, b)
    for i in range(s + 1, e + 1):
        a, b = slots[(i - 1) % 2], slots[i % 2]
        session.write(b, frames[i])
        session.pair(a, b)
        session.mid(t, out)
        if read:
            emit(i, session.read(out))
        done.append(i)
    return done
