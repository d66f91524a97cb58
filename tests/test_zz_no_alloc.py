"""fhk_gmhs_noalloc: the repair stage for callers that must not allocate device memory once frames flow (hosts that
reserve their GPU memory up front, plugins whose memory belongs to the host application's allocator). Its scratch is
a device array inside the library, so it is checked here against the allocating entry point fhk_gmhs, which takes
the caller's scratch: the same inputs must give the same repaired flow, on two calls in a row with different inputs
(the shared array keeps the previous call's contents, which must not leak into the next result), and the second
call must leave the device's free memory as it found it.

This file sorts last so that a run stopping at the first failure has run every other test before it.
"""
import ctypes
from ctypes import Structure, c_int, c_longlong, c_void_p

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


class GmhsParams(Structure):  # include/flyhigh_kernels.h FhGmhsParams
    _fields_ = [("flow", c_void_p), ("flow_bs", c_longlong), ("h8", c_int), ("w8", c_int), ("a", c_void_p),
                ("b", c_void_p), ("ab_bs", c_longlong), ("h", c_int), ("w", c_int), ("full_w", c_int),
                ("level", c_int), ("scratch", c_void_p), ("n", c_int)]


def _device(torch, chw, cs):
    c, h, w = chw.shape
    t = torch.zeros((h, w, cs), dtype=torch.float16)
    t[:, :, :c] = torch.from_numpy(np.ascontiguousarray(chw.transpose(1, 2, 0))).to(torch.float16)
    return t.cuda()


def _repair(torch, lib, entry, a, b, flow, full_w, with_scratch):
    """Runs one repair entry point on fresh device copies of the inputs; returns the flow [4][h8][w8]."""
    _, h, w = a.shape
    _, h8, w8 = flow.shape
    A, B, F = _device(torch, a, 4), _device(torch, b, 4), _device(torch, flow, 8)
    scratch = None
    if with_scratch:
        scratch = torch.full((lib.fhk_gmhs_scratch_floats(h, w),), float("nan"), dtype=torch.float32, device="cuda")
    p = GmhsParams(F.data_ptr(), 0, h8, w8, A.data_ptr(), B.data_ptr(), 0, h, w, full_w, 1,
                   scratch.data_ptr() if scratch is not None else None, 1)
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    rc = entry(ctypes.byref(p), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, rc
    torch.cuda.synchronize()
    free_after = torch.cuda.mem_get_info()[0]
    return F[:, :, :4].permute(2, 0, 1).float().cpu().numpy(), free_before - free_after


def test_gmhs_without_allocation_matches_gmhs(synth_model_dir):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import flyhigh_engine_b200 as fh
    from flyhigh_engine_b200 import synth_frames
    from oracle.oracle import OracleModel, OracleSession
    lib = fh.lib()
    model = OracleModel(synth_model_dir)
    changed_total = 0
    for seed in (7, 11):  # two calls in a row, different inputs
        fa, fb, _ = synth_frames.pair_c0(1920, 1080, seed=seed)
        o = OracleSession(model, 1920, 1080)
        o.pair(fa, fb)
        a, b, pre, post = o.tensor("A"), o.tensor("B"), o.tensor("flow_pre"), o.tensor("flow")
        full_w = o.dims()["wp"]
        ref, _ = _repair(torch, lib, lib.fhk_gmhs, a, b, pre, full_w, with_scratch=True)
        got, taken = _repair(torch, lib, lib.fhk_gmhs_noalloc, a, b, pre, full_w, with_scratch=False)
        if seed == 11:  # past the first call (which may load the library's device code), a call takes no memory
            assert taken == 0, taken
        # the repair stage is bit-exact against the oracle, so the two entry points must agree exactly
        assert np.array_equal(got, ref), int((got != ref).any(axis=0).sum())
        assert np.array_equal(got, post)
        changed_total += int((pre != post).any(axis=0).sum())
    assert changed_total > 0, "the inputs should make the repair rewrite some cells"


def test_gmhs_without_allocation_rejects_too_large():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import flyhigh_engine_b200 as fh
    lib = fh.lib()
    cap = lib.fhk_gmhs_noalloc_max_floats()
    assert lib.fhk_gmhs_scratch_floats(480, 864) <= cap
    assert lib.fhk_gmhs_scratch_floats(1088, 1920) > cap
    dummy = torch.zeros(16, dtype=torch.float16, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = GmhsParams(dummy.data_ptr(), 0, 136, 240, dummy.data_ptr(), dummy.data_ptr(), 0, 1088, 1920, 1920, 1, None, 1)
    assert lib.fhk_gmhs_noalloc(ctypes.byref(p), stream) == 1  # cudaErrorInvalidValue: beyond the array
    p = GmhsParams(dummy.data_ptr(), 0, 60, 108, dummy.data_ptr(), dummy.data_ptr(), 0, 480, 864, 1920, 1,
                   dummy.data_ptr(), 1)
    assert lib.fhk_gmhs_noalloc(ctypes.byref(p), stream) == 1  # a caller scratch is refused: it allocates nothing


def test_gmhs_without_allocation_holds_device_memory_steady(synth_model_dir):
    """After a warm-up call, a further call changes neither the device's free memory (cudaMemGetInfo) nor torch's
    allocations: inputs and outputs are allocated before, nothing during the call."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import flyhigh_engine_b200 as fh
    from flyhigh_engine_b200 import synth_frames
    from oracle.oracle import OracleModel, OracleSession
    lib = fh.lib()
    fa, fb, _ = synth_frames.pair_c0(1920, 1080, seed=7)
    o = OracleSession(OracleModel(synth_model_dir), 1920, 1080)
    o.pair(fa, fb)
    a, b, pre = o.tensor("A"), o.tensor("B"), o.tensor("flow_pre")
    _, h, w = a.shape
    _, h8, w8 = pre.shape
    A, B, F = _device(torch, a, 4), _device(torch, b, 4), _device(torch, pre, 8)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = GmhsParams(F.data_ptr(), 0, h8, w8, A.data_ptr(), B.data_ptr(), 0, h, w, o.dims()["wp"], 1, None, 1)
    assert lib.fhk_gmhs_noalloc(ctypes.byref(p), stream) == 0  # the warm-up call
    torch.cuda.synchronize()
    free0, alloc0 = torch.cuda.mem_get_info()[0], torch.cuda.memory_allocated()
    assert lib.fhk_gmhs_noalloc(ctypes.byref(p), stream) == 0
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    assert torch.cuda.memory_allocated() == alloc0
