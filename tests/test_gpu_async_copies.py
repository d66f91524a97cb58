"""The asynchronous host copies of flyhigh_b200.h (fh_session_write_rgba_async / write_wait, read_rgba_async /
read_wait) give the bytes of the blocking calls, one interval at a time and on a batched session: readbacks of four
output slots issued right before the next batch rewrites them (the rewrite waits for the readbacks on the device), and
a pinned upload buffer refilled as soon as write_wait returns."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("batch", [1, 4])
def test_async_copies_match_blocking(synth_model_dir, batch):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import flyhigh_engine_b200 as fh
    from flyhigh_engine_b200 import synth_frames
    w, h, n = 640, 360, 11
    frames = synth_frames.sequence_c2(n, w, h, seed=31)
    model = fh.Model(synth_model_dir)
    eng = fh.Engine()

    ref = fh.Session(eng, model, w, h, batch=batch)
    ra, rb, ro = ref.add_input(), ref.add_input(), ref.add_output()
    want = []
    ref.write(ra, frames[0])
    for i in range(1, n):
        a, b = (ra, rb) if i % 2 else (rb, ra)
        ref.write(b, frames[i])
        ref.pair(a, b)
        ref.mid(0.5, ro)
        want.append(ref.read(ro))

    s = fh.Session(eng, model, w, h, batch=batch)
    sa, sb = s.add_input(), s.add_input()
    outs = [s.add_output() for _ in range(4)]
    up = torch.empty((h, w, 4), dtype=torch.uint8).pin_memory().numpy()
    back = [torch.empty((h, w, 4), dtype=torch.uint8).pin_memory().numpy() for _ in range(n)]
    up[...] = frames[0]
    s.write_async(sa, up)
    s.write_wait(sa)
    for i in range(1, n):
        a, b = (sa, sb) if i % 2 else (sb, sa)
        up[...] = frames[i]  # the previous upload has landed: write_wait returned
        s.write_async(b, up)
        s.write_wait(b)
        s.pair(a, b)
        s.mid(0.5, outs[(i - 1) % 4])
        if i % 4 == 0:
            # intervals i - 3 .. i have run (a full batch of 4, or one by one): their readbacks, which the next four
            # mids' writes of the same slots must wait for on the device
            for j in range(i - 3, i + 1):
                s.read_async(outs[(j - 1) % 4], back[j])
    for j in range(n - 1 - (n - 1) % 4 + 1, n):  # the last, shorter group: each read runs what is queued first
        s.read_async(outs[(j - 1) % 4], back[j])
    for o in outs:
        s.read_wait(o)
    for i in range(1, n):
        assert back[i].tobytes() == want[i - 1], i
    with pytest.raises(ValueError):
        s.read_async(outs[0], back[1][:, ::2])  # a strided view would need a temporary copy
