"""FlyHigh B200: the FlyHighFG Core (Session.pair / Session.mid) on an NVIDIA B200, through the drop-in C ABI.

The classes keep the names, arguments and errors of the reference's ctypes binding (Engine, Model, Session,
FlyHighError), so code written against that binding keeps working. A typical 2x interpolation loop over a list of
rgba8 frames (numpy arrays of shape (h, w, 4) or bytes) looks like this:

    import flyhigh_engine_b200 as fh
    sess = fh.Session(fh.Engine(), fh.Model(model_dir), width, height)
    slots, dst = (sess.add_input(), sess.add_input()), sess.add_output()
    sess.write(slots[0], frames[0])
    for i in range(1, len(frames)):
        sess.write(slots[i % 2], frames[i])
        sess.pair(slots[(i - 1) % 2], slots[i % 2])   # the motion between the two frames
        sess.mid(0.5, dst)                            # the frame halfway between them
        between = sess.read(dst)                      # width * height * 4 bytes

The library is libflyhigh.so next to this file (built by `flyhigh_engine_b200.build.build()`), or FLYHIGH_LIB.
There is no fallback: without the CUDA library every call raises.
"""
from __future__ import annotations

import ctypes
import json
import os
from ctypes import (POINTER, Structure, byref, c_char_p, c_double, c_float, c_int, c_long, c_size_t, c_uint8, c_uint32,
                    c_void_p, create_string_buffer)
from typing import Optional

__all__ = ["FlyHighError", "Engine", "Model", "Session", "Stream", "Classification", "Push", "library_path"]


class FlyHighError(RuntimeError):
    """Raised when a library call reports failure (NULL or a negative status); the text is fh_last_error()'s."""


class EngineOptions(Structure):  # flyhigh.h FhEngineOptions, field for field
    _fields_ = [("backend", c_uint32), ("tensor_cores", c_uint32), ("autotune", c_uint32), ("adapter", c_char_p),
                ("precision", c_uint32), ("tune_cache", c_char_p), ("compact_memory", c_uint32),
                ("dxc_path", c_char_p)]


class SessionOptions(Structure):  # flyhigh.h FhSessionOptions, field for field
    _fields_ = [("width", c_uint32), ("height", c_uint32), ("internal_w", c_uint32), ("internal_h", c_uint32),
                ("k", c_uint32), ("repair", c_uint32), ("render", c_uint32), ("keep_static", c_uint32),
                ("static_frames", c_uint32), ("static_tolerance", c_uint32), ("fast_render", c_uint32),
                ("linear_t", c_uint32), ("keep_maps", c_uint32), ("protection_mask", c_uint32), ("tune", c_char_p)]


class StreamOptions(Structure):  # flyhigh.h FhStreamOptions, field for field
    _fields_ = [("mode", c_uint32), ("cadence", c_uint32), ("scene_cut", c_double), ("held_frames", c_uint32),
                ("held_mean", c_double), ("held_max", c_double), ("inputs", c_uint32), ("outputs", c_uint32)]


class _Classification(Structure):  # flyhigh.h FhClassification
    _fields_ = [("kind", c_uint32), ("mean", c_float), ("max", c_float), ("black", c_uint32), ("motion", c_double)]


class _Push(Structure):  # flyhigh.h FhPush
    _fields_ = [("ready", c_uint32), ("base_slot", ctypes.c_int32), ("stats_pending", c_uint32),
                ("start_pts", c_double), ("end_pts", c_double)]


class GeneratorOptions(Structure):  # flyhigh.h FhOptions, field for field
    _fields_ = [(n, c_uint32) for n in ("width", "height", "k", "internal_w", "internal_h", "mode", "repair", "cadence",
                                        "render_sampling", "keep_static", "static_frames", "static_tolerance",
                                        "fast_render", "linear_t")]


class PacerOptions(Structure):  # flyhigh.h FhPacerOptions (the Pacer is declared, not built)
    _fields_ = [("mode", c_uint32), ("factor", c_uint32), ("target_fps", c_double), ("max_factor", c_uint32),
                ("fps_limit", c_double), ("lookahead", c_uint32), ("limit_to_display", c_uint32),
                ("fill_display", c_uint32), ("display_headroom", c_double), ("compute_budget", c_double),
                ("delay_floor_ms", c_double), ("delay_max_ms", c_double), ("lateness_intervals", c_double),
                ("queue_capacity", c_uint32), ("pressure_tau_ms", c_double), ("penalty_up", c_double),
                ("penalty_burst", c_double), ("penalty_min_gap_ms", c_double), ("penalty_max", c_uint32),
                ("recovery_after_ms", c_double), ("stall_window_ms", c_double), ("stall_rate_limit", c_double),
                ("settle_ms", c_double), ("motion_adaptive", c_uint32), ("min_present_interval_ms", c_double),
                ("playback_rate", c_double), ("mid_cost_seed_ms", c_double), ("pair_cost_seed_ms", c_double),
                ("gpu_timestamps", c_uint32), ("low_latency", c_uint32)]


def library_path() -> str:
    env = os.environ.get("FLYHIGH_LIB")
    if env:
        return env
    return os.path.join(os.path.dirname(os.path.abspath(__file__)), "libflyhigh.so")


_lib = None

# every export of include/flyhigh.h, include/flyhigh_b200.h and include/flyhigh_kernels.h: (name, restype, argtypes)
EXPORTS = [
    ("fh_last_error", c_char_p, []),
    ("fh_engine_options_default", EngineOptions, []),
    ("fh_engine_create", c_void_p, [POINTER(EngineOptions)]),
    ("fh_engine_destroy", None, [c_void_p]),
    ("fh_engine_info", c_int, [c_void_p, c_char_p, c_size_t]),
    ("fh_engine_report_json", c_int, [c_void_p, c_char_p, c_size_t]),
    ("fh_model_load", c_void_p, [c_char_p]),
    ("fh_model_from_bytes", c_void_p, [POINTER(c_uint8), c_size_t, POINTER(c_uint8), c_size_t, POINTER(c_uint8),
                                       c_size_t]),
    ("fh_model_destroy", None, [c_void_p]),
    ("fh_model_info", c_int, [c_void_p, c_char_p, c_size_t]),
    ("fh_session_options_default", SessionOptions, [c_uint32, c_uint32]),
    ("fh_session_create", c_void_p, [c_void_p, c_void_p, POINTER(SessionOptions)]),
    ("fh_session_create_batched", c_void_p, [c_void_p, c_void_p, POINTER(SessionOptions), c_uint32]),
    ("fh_session_destroy", None, [c_void_p]),
    ("fh_session_add_input", c_int, [c_void_p]),
    ("fh_session_add_output", c_int, [c_void_p]),
    ("fh_session_write_rgba", c_int, [c_void_p, c_uint32, c_void_p, c_size_t]),
    ("fh_session_write_mask", c_int, [c_void_p, c_void_p, c_size_t]),
    ("fh_session_read_rgba", c_int, [c_void_p, c_uint32, c_void_p, c_size_t]),
    ("fh_session_pair", c_int, [c_void_p, c_uint32, c_uint32]),
    ("fh_session_mid", c_int, [c_void_p, c_float, c_uint32]),
    ("fh_session_generate", c_int, [c_void_p, c_uint32, c_uint32, c_float, c_uint32]),
    ("fh_session_pair_timed", c_int, [c_void_p, c_uint32, c_uint32, POINTER(c_double)]),
    ("fh_session_mid_timed", c_int, [c_void_p, c_float, c_uint32, POINTER(c_double)]),
    ("fh_session_warm_up", c_int, [c_void_p]),
    ("fh_session_import_d3d11", c_int, [c_void_p, c_void_p, ctypes.c_ssize_t, c_uint32, c_uint32]),
    ("fh_session_report_json", c_int, [c_void_p, c_char_p, c_size_t]),
    ("fh_session_cuda_stream", c_int, [c_void_p, POINTER(c_void_p)]),
    ("fh_session_join", c_int, [c_void_p]),
    ("fh_session_kernel_launches", ctypes.c_longlong, [c_void_p]),
    ("fh_session_slot_device_ptr", c_int, [c_void_p, c_uint32, c_int, POINTER(c_void_p)]),
    ("fh_session_write_rgba_device", c_int, [c_void_p, c_uint32, c_void_p, c_size_t]),
    ("fh_session_debug_tensor", c_long, [c_void_p, c_char_p, POINTER(c_float), c_size_t, POINTER(c_int)]),
    ("fh_session_debug_tensor_at", c_long, [c_void_p, c_char_p, c_int, POINTER(c_float), c_size_t, POINTER(c_int)]),
    ("fh_model_fingerprint", c_long, [c_void_p]),
    ("fh_session_plan_params", c_int, [c_void_p, POINTER(SessionOptions), POINTER(c_int), POINTER(c_float)]),
    ("fh_session_advance_static", c_int, [c_void_p, c_uint32, c_uint32]),
    ("fh_session_profile_json", c_int, [c_void_p, c_uint32, c_uint32, c_float, c_uint32, c_char_p, c_size_t]),
    ("fh_session_launch_counts", c_int, [c_void_p, POINTER(c_int), POINTER(c_int), POINTER(c_int)]),
    ("fh_session_profile_batch_json", c_int, [c_void_p, c_char_p, c_size_t]),
    ("fh_stream_options_default", StreamOptions, []),
    ("fh_stream_create", c_void_p, [c_void_p, c_void_p, POINTER(SessionOptions), POINTER(StreamOptions)]),
    ("fh_stream_destroy", None, [c_void_p]),
    ("fh_stream_add_input", c_int, [c_void_p, c_void_p]),
    ("fh_stream_add_output", c_int, [c_void_p, c_void_p]),
    ("fh_stream_next_input", c_int, [c_void_p, POINTER(c_uint32), c_size_t]),
    ("fh_stream_write_rgba", c_int, [c_void_p, c_void_p, c_uint32, c_void_p, c_size_t]),
    ("fh_stream_write_rgba_device", c_int, [c_void_p, c_uint32, c_void_p, c_size_t]),
    ("fh_stream_write_mask", c_int, [c_void_p, c_void_p, c_void_p, c_size_t]),
    ("fh_stream_classify", c_int, [c_void_p, c_void_p, c_uint32, c_uint32, POINTER(_Classification)]),
    ("fh_stream_push", c_int, [c_void_p, c_void_p, c_uint32, c_double, POINTER(_Push)]),
    ("fh_stream_resolve_stats", c_int, [c_void_p, c_void_p]),
    ("fh_stream_real_replaced", c_int, [c_void_p]),
    ("fh_stream_generate", c_int, [c_void_p, c_void_p, c_float, c_uint32]),
    ("fh_stream_read_rgba", c_int, [c_void_p, c_void_p, c_uint32, c_void_p, c_size_t]),
    ("fh_stream_warm_up", c_int, [c_void_p, c_void_p]),
    ("fh_stream_import_d3d11", c_int, [c_void_p, c_void_p, ctypes.c_ssize_t, c_uint32, c_uint32]),
    ("fh_stream_reset", c_int, [c_void_p]),
    ("fh_stream_mouse", c_int, [c_void_p, c_void_p, c_double, c_double, c_double]),
    ("fh_stream_set_mouse_captured", c_int, [c_void_p, c_uint32]),
    ("fh_stream_warp", c_int, [c_void_p, c_void_p, c_uint32, c_uint32, c_uint32, c_double]),
    ("fh_stream_report_json", c_int, [c_void_p, c_char_p, c_size_t]),
    ("fh_stream_camera_warp", c_void_p, [c_void_p]),
    ("fh_session_write_rgba_async", c_int, [c_void_p, c_uint32, c_void_p, c_size_t]),
    ("fh_session_write_wait", c_int, [c_void_p, c_uint32]),
    ("fh_session_read_rgba_async", c_int, [c_void_p, c_uint32, c_void_p, c_size_t]),
    ("fh_session_read_wait", c_int, [c_void_p, c_uint32]),
    ("fh_options_default", GeneratorOptions, [c_uint32, c_uint32]),
    ("fh_generator_create", c_void_p, [c_void_p, c_void_p, POINTER(GeneratorOptions)]),
    ("fh_generator_destroy", None, [c_void_p]),
    ("fh_generator_warmup", c_int, [c_void_p]),
    ("fh_generator_push", c_int, [c_void_p, c_void_p, c_size_t, c_uint32]),
    ("fh_generator_pop", c_int, [c_void_p, c_void_p, c_size_t, POINTER(c_float), POINTER(c_int)]),
    ("fh_pacer_options_default", PacerOptions, []),
    ("fh_pacer_create", c_void_p, [POINTER(PacerOptions)]),
    ("fh_pacer_destroy", None, [c_void_p]),
    ("fh_pacer_set_options", c_int, [c_void_p, c_double, POINTER(PacerOptions)]),
    ("fh_pacer_tick", c_int, [c_void_p, c_double, c_void_p]),
    ("fh_pacer_source_frame", c_int, [c_void_p, c_double, c_void_p]),
    ("fh_pacer_requests", c_int, [c_void_p, c_void_p, c_size_t]),
    ("fh_pacer_generated", c_int, [c_void_p, c_double, ctypes.c_uint64, c_uint32]),
    ("fh_pacer_skipped", c_int, [c_void_p, ctypes.c_uint64]),
    ("fh_pacer_cost_sample", c_int, [c_void_p, c_double, c_uint32, c_double]),
    ("fh_pacer_host_stall", c_int, [c_void_p, c_double, c_double]),
    ("fh_pacer_mode_change", c_int, [c_void_p, c_double]),
    ("fh_pacer_reset", c_int, [c_void_p, c_double]),
    ("fh_pacer_report_json", c_int, [c_void_p, c_char_p, c_size_t]),
    ("fh_pacer_record", c_int, [c_void_p, c_char_p]),
    ("fh_pacer_trace_json", c_int, [c_void_p, c_char_p, c_size_t]),
    ("fh_engine_vulkan_interop", c_int, [c_void_p, c_void_p]),
    ("fh_vk_row_pitch", c_uint32, [c_uint32]),
    ("fh_vk_buffer_import", c_void_p, [c_void_p, c_void_p, ctypes.c_uint64]),
    ("fh_vk_buffer_destroy", None, [c_void_p]),
    ("fh_vk_semaphore_import", c_void_p, [c_void_p, ctypes.c_ssize_t, c_uint32]),
    ("fh_vk_semaphore_destroy", None, [c_void_p]),
    ("fh_vk_signal", c_int, [c_void_p, c_void_p, ctypes.c_uint64]),
    ("fh_stream_copy_in", c_int, [c_void_p, c_void_p, c_uint32, c_void_p, c_uint32, c_void_p, ctypes.c_uint64]),
    ("fh_stream_copy_out", c_int, [c_void_p, c_void_p, c_uint32, c_void_p, c_uint32, c_void_p, ctypes.c_uint64]),
    ("fh_session_copy_in", c_int, [c_void_p, c_void_p, c_uint32, c_void_p, c_uint32, c_void_p, ctypes.c_uint64]),
    ("fh_session_copy_out", c_int, [c_void_p, c_void_p, c_uint32, c_void_p, c_uint32, c_void_p, ctypes.c_uint64]),
    ("fh_warp_create", c_void_p, [c_void_p, c_uint32, c_uint32, c_double]),
    ("fh_warp_destroy", None, [c_void_p]),
    ("fh_warp_mouse", c_int, [c_void_p, c_double, c_double, c_double]),
    ("fh_warp_set_captured", c_int, [c_void_p, c_uint32]),
    ("fh_warp_break_pair", c_int, [c_void_p]),
    ("fh_warp_frame", c_int, [c_void_p, c_void_p, c_double]),
    ("fh_warp_collect", c_int, [c_void_p, c_int]),
    ("fh_warp_last_shift", c_int, [c_void_p, POINTER(c_double), POINTER(c_double)]),
    ("fh_warp_shift", c_int, [c_void_p, c_double, c_double, POINTER(c_double), POINTER(c_double)]),
    ("fh_warp_decide", c_int, [c_void_p, c_double, c_double, POINTER(c_double), POINTER(c_double)]),
    ("fh_warp_render_shift", c_void_p, [c_void_p, c_void_p, c_double, c_double]),
    ("fh_warp_render_into", c_int, [c_void_p, c_void_p, c_void_p, c_double, c_double]),
    ("fh_warp_cuda_stream", c_int, [c_void_p, POINTER(c_void_p)]),
    ("fh_warp_read_mask", ctypes.c_long, [c_void_p, POINTER(c_float), c_size_t]),
    ("fh_warp_debug_tensor", ctypes.c_long, [c_void_p, c_char_p, POINTER(c_float), c_size_t]),
    ("fh_warp_report_json", c_int, [c_void_p, c_char_p, c_size_t]),
    ("fhk_conv3x3", c_int, [c_void_p, c_int, c_void_p]),
    ("fhk_conv_pack_weights", c_int, [c_void_p, c_int, c_int, c_void_p, c_int, c_void_p]),
    ("fhk_conv_packed_elems", c_size_t, [c_int, c_int]),
    ("fhk_conv_wait_timeouts", ctypes.c_longlong, [c_int]),
    ("fhk_conv3x3_umma", c_int, [c_void_p, c_void_p]),
    ("fhk_conv_umma_fits", c_int, [c_int, c_int, c_int]),
    ("fhk_conv_umma_persistent_fits", c_int, [c_int, c_int]),
    ("fhk_conv_pack_weights_umma", c_int, [c_void_p, c_int, c_int, c_void_p, c_int, c_void_p]),
    ("fhk_conv_packed_elems_umma", c_size_t, [c_int, c_int]),
    ("fhk_gmhs", c_int, [c_void_p, c_void_p]),
    ("fhk_gmhs_scratch_floats", c_size_t, [c_int, c_int]),
    ("fhk_gmhs_noalloc", c_int, [c_void_p, c_void_p]),
    ("fhk_gmhs_noalloc_max_floats", c_size_t, []),
]


def lib():
    """The loaded libflyhigh.so (raises FlyHighError when it is missing: there is no CPU fallback)."""
    global _lib
    if _lib is None:
        path = library_path()
        if not os.path.exists(path):
            raise FlyHighError(f"{path} is missing: build it with flyhigh_engine_b200.build.build()")
        L = ctypes.CDLL(path)
        for name, res, args in EXPORTS:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _error() -> FlyHighError:
    msg = lib().fh_last_error()
    return FlyHighError(msg.decode("utf-8", "replace") if msg else "unknown error")


def _check(rc: int) -> int:
    if rc < 0:
        raise _error()
    return rc


def _json(fn, handle) -> dict:
    cap = 1 << 12
    while True:
        buf = create_string_buffer(cap)
        n = fn(handle, buf, cap)
        if n >= 0:
            return json.loads(buf.raw[:n].decode("utf-8"))
        if b"buffer too small" in (lib().fh_last_error() or b"") and cap < (1 << 24):
            cap *= 4
            continue
        raise _error()


def _buffer(data):
    """(pointer, length, keep-alive) of a bytes-like object or numpy array, without a copy where possible."""
    try:
        import numpy as np
        if isinstance(data, np.ndarray):
            a = np.ascontiguousarray(data)
            return a.ctypes.data_as(c_void_p), a.nbytes, a
    except ImportError:
        pass
    mv = memoryview(data).cast("B")
    if mv.readonly:
        b = ctypes.create_string_buffer(bytes(mv), len(mv))
        return ctypes.cast(b, c_void_p), len(mv), b
    arr = (c_uint8 * len(mv)).from_buffer(mv)
    return ctypes.cast(arr, c_void_p), len(mv), arr


def _async_buffer(data, n):
    """(pointer, length) of memory an asynchronous copy may use after the call returns: a pointer (int), or a
    C-contiguous numpy array (the caller keeps it alive); anything that would need a temporary copy is refused."""
    if isinstance(data, int):
        return c_void_p(data), n
    import numpy as np
    if isinstance(data, np.ndarray) and data.flags["C_CONTIGUOUS"]:
        return data.ctypes.data_as(c_void_p), data.nbytes
    raise ValueError("asynchronous copies take a pointer or a C-contiguous numpy array (pinned host memory)")


_PRECISION = {"auto": 0, "f16": 1, "f32": 2}
_RENDER = {"model": 0, "bilinear": 1, "bicubic": 2}


class Engine:
    """The device: Engine(adapter=None | "#N" (CUDA device N), precision="auto"|"f16"). The graphics-API options of
    the reference (backend, dxc_path, ...) are accepted and ignored."""

    def __init__(self, backend: str = "auto", precision: str = "auto", tensor_cores: bool = True, autotune: bool = True,
                 adapter: Optional[str] = None, tune_cache: Optional[str] = None, compact_memory: bool = True,
                 dxc_path: Optional[str] = None):
        L = lib()
        o = L.fh_engine_options_default()
        o.precision = _PRECISION[precision]
        o.tensor_cores = int(tensor_cores)
        o.autotune = int(autotune)
        o.compact_memory = int(compact_memory)
        self._keep = [s.encode() if s else None for s in (adapter, tune_cache, dxc_path)]
        o.adapter, o.tune_cache, o.dxc_path = self._keep
        self._h = L.fh_engine_create(byref(o))
        if not self._h:
            raise _error()

    def info(self) -> dict:
        return _json(lib().fh_engine_info, self._h)

    def report(self) -> dict:
        return _json(lib().fh_engine_report_json, self._h)

    def close(self):
        if getattr(self, "_h", None):
            lib().fh_engine_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except TypeError:  # interpreter shutdown: the module's globals are already gone, the process frees everything
            pass


class Model:
    """Model(directory) with graph.json, flyhighfg.json and flyhighfg.bin; or Model.from_bytes(...)."""

    def __init__(self, directory: Optional[str] = None, _handle=None):
        if _handle is not None:
            self._h = _handle
        else:
            self._h = lib().fh_model_load(str(directory).encode())
        if not self._h:
            raise _error()

    @classmethod
    def from_bytes(cls, graph_json: bytes, manifest_json: bytes, weights: bytes) -> "Model":
        bufs = [(c_uint8 * len(b)).from_buffer_copy(b) for b in (graph_json, manifest_json, weights)]
        h = lib().fh_model_from_bytes(bufs[0], len(graph_json), bufs[1], len(manifest_json), bufs[2], len(weights))
        if not h:
            raise _error()
        return cls(_handle=h)

    def info(self) -> dict:
        return _json(lib().fh_model_info, self._h)

    def fingerprint(self) -> int:
        return int(lib().fh_model_fingerprint(self._h))

    def plan_params(self, width: int, height: int, **options) -> dict:
        """The sizes and parameter words a session of these options derives (no device needed)."""
        o = session_options(width, height, **options)
        iv = (c_int * 22)()
        fv = (c_float * 6)()
        _check(lib().fh_session_plan_params(self._h, byref(o), iv, fv))
        names = ["hp", "wp", "ihp", "iwp", "internal", "NH", "NW", "qh", "qw", "h8", "w8", "h16", "w16", "hc", "wc",
                 "r_blk", "r_dwin", "k", "repair", "cubic", "protects", "render_flags"]
        d = dict(zip(names, list(iv)))
        d.update(zip(["fsx", "fsy", "dmin", "delta", "min_age", "static_thr"], list(fv)))
        return d

    def close(self):
        if getattr(self, "_h", None):
            lib().fh_model_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except TypeError:  # interpreter shutdown: the module's globals are already gone, the process frees everything
            pass


def session_options(width: int, height: int, internal=None, k: int = 1, repair: int = 1, render: str = "model",
                    static_protection=None, fast_render: bool = False, linear_t: bool = False,
                    keep_maps: bool = False, protection_mask: bool = False, tune: Optional[str] = None) -> SessionOptions:
    o = lib().fh_session_options_default(width, height)
    if internal == "frame":
        o.internal_w, o.internal_h = width, height
    elif internal not in (None, "auto"):
        o.internal_w, o.internal_h = int(internal[0]), int(internal[1])
    o.k = k
    o.repair = repair
    o.render = _RENDER[render]
    if static_protection is False:
        o.keep_static = 0
    elif static_protection:
        o.keep_static = 1
        if isinstance(static_protection, dict):
            o.static_frames = int(static_protection.get("frames", o.static_frames))
            o.static_tolerance = int(static_protection.get("tolerance", o.static_tolerance))
    o.fast_render = int(fast_render)
    o.linear_t = int(linear_t)
    o.keep_maps = int(keep_maps)
    o.protection_mask = int(protection_mask)
    o.tune = tune.encode() if tune else None
    return o


class Session:
    """A model planned for one frame size, with its input and output slots.

    Keyword options map onto FhSessionOptions: internal ("auto", "frame" or a (w, h) network size), k (fine-loop
    passes), repair (0-2), render ("model", "bilinear", "bicubic"), static_protection (None for the default, a bool,
    or a dict with "frames" / "tolerance"), fast_render, linear_t, keep_maps, protection_mask and tune. batch = n > 1
    builds a batched session (fh_session_create_batched): pair / mid calls queue up and n chained intervals run per
    launch; None leaves the choice to the FH_BATCH environment variable."""

    def __init__(self, engine: Engine, model: Model, width: int, height: int, batch=None, **options):
        self._o = session_options(width, height, **options)
        self.width, self.height = width, height
        self._e, self._m = engine, model
        if batch is None:
            self._h = lib().fh_session_create(engine._h, model._h, byref(self._o))
        else:
            self._h = lib().fh_session_create_batched(engine._h, model._h, byref(self._o), int(batch))
        if not self._h:
            raise _error()

    def add_input(self) -> int:
        return _check(lib().fh_session_add_input(self._h))

    def add_output(self) -> int:
        return _check(lib().fh_session_add_output(self._h))

    def write(self, slot: int, rgba) -> None:
        p, n, _keep = _buffer(rgba)
        _check(lib().fh_session_write_rgba(self._h, slot, p, n))

    def write_device(self, slot: int, device_ptr: int, nbytes: int) -> None:
        """A frame already in device memory (a CUDA pointer) into an input slot."""
        _check(lib().fh_session_write_rgba_device(self._h, slot, c_void_p(device_ptr), nbytes))

    def write_mask(self, mask) -> None:
        p, n, _keep = _buffer(mask)
        _check(lib().fh_session_write_mask(self._h, p, n))

    def read(self, slot: int) -> bytes:
        n = self.width * self.height * 4
        buf = (c_uint8 * n)()
        _check(lib().fh_session_read_rgba(self._h, slot, ctypes.cast(buf, c_void_p), n))
        return bytes(buf)

    def read_into(self, slot: int, out) -> None:
        """Into a caller buffer (e.g. pinned host memory: a numpy array over it, or a torch tensor's data_ptr())."""
        if isinstance(out, int):
            p, n = c_void_p(out), self.width * self.height * 4
        else:
            p, n, _keep = _buffer(out)
        _check(lib().fh_session_read_rgba(self._h, slot, p, n))

    def write_async(self, slot: int, rgba) -> None:
        """fh_session_write_rgba_async: the upload is issued and the call returns; `rgba` (pinned host memory, a numpy
        array over it or a pointer) must stay unchanged until write_wait(slot)."""
        p, n = _async_buffer(rgba, self.width * self.height * 4)
        _check(lib().fh_session_write_rgba_async(self._h, slot, p, n))

    def write_wait(self, slot: int) -> None:
        _check(lib().fh_session_write_wait(self._h, slot))

    def read_async(self, slot: int, out) -> None:
        """fh_session_read_rgba_async into a caller buffer (pinned host memory); its bytes are there after
        read_wait(slot)."""
        p, n = _async_buffer(out, self.width * self.height * 4)
        _check(lib().fh_session_read_rgba_async(self._h, slot, p, n))

    def read_wait(self, slot: int) -> None:
        _check(lib().fh_session_read_wait(self._h, slot))

    def pair(self, a: int, b: int) -> None:
        _check(lib().fh_session_pair(self._h, a, b))

    def mid(self, t: float, out: int) -> None:
        _check(lib().fh_session_mid(self._h, t, out))

    def generate(self, a: int, b: int, t: float, out: int) -> None:
        _check(lib().fh_session_generate(self._h, a, b, t, out))

    def pair_timed(self, a: int, b: int) -> Optional[float]:
        ms = c_double()
        return ms.value if _check(lib().fh_session_pair_timed(self._h, a, b, byref(ms))) == 1 else None

    def mid_timed(self, t: float, out: int) -> Optional[float]:
        ms = c_double()
        return ms.value if _check(lib().fh_session_mid_timed(self._h, t, out, byref(ms))) == 1 else None

    def warm_up(self) -> None:
        _check(lib().fh_session_warm_up(self._h))

    def report(self) -> dict:
        return _json(lib().fh_session_report_json, self._h)

    # ---- additions (include/flyhigh_b200.h) ----
    def cuda_stream(self) -> int:
        p = c_void_p()
        _check(lib().fh_session_cuda_stream(self._h, byref(p)))
        return p.value or 0

    def kernel_launches(self) -> int:
        """Kernels this session has launched so far (graph kernel nodes and eager launches; profiling excepted)."""
        return _check(lib().fh_session_kernel_launches(self._h))

    def join(self) -> None:
        """Orders every batch render issued so far before the work later issued on cuda_stream()."""
        _check(lib().fh_session_join(self._h))

    def slot_ptr(self, slot: int, output: bool = False) -> int:
        p = c_void_p()
        _check(lib().fh_session_slot_device_ptr(self._h, slot, int(output), byref(p)))
        return p.value

    def advance_static(self, a: int, b: int) -> None:
        """The static-protection state of the pair (a, b) without the network (see multi.py)."""
        _check(lib().fh_session_advance_static(self._h, a, b))

    def profile(self, a: int, b: int, t: float, out: int) -> list:
        """Device ms of every kernel of one pair + mid, run eagerly ([{"kernel", "ms"}])."""
        cap = 1 << 16
        buf = create_string_buffer(cap)
        n = _check(lib().fh_session_profile_json(self._h, a, b, t, out, buf, cap))
        return json.loads(buf.raw[:n].decode())

    def profile_batch(self) -> list:
        """Device ms of every kernel of one batch of a batched session, run eagerly on its batch arena."""
        cap = 1 << 16
        buf = create_string_buffer(cap)
        n = _check(lib().fh_session_profile_batch_json(self._h, buf, cap))
        return json.loads(buf.raw[:n].decode())

    def launch_counts(self) -> dict:
        a, b, c = c_int(), c_int(), c_int()
        _check(lib().fh_session_launch_counts(self._h, byref(a), byref(b), byref(c)))
        return {"pair": a.value, "mid": b.value, "frame": c.value}

    def tensor(self, name: str, interval: int = -1):
        """A tensor of the last pair / mid as a float32 numpy array [c][h][w] (the reference's planar order); with
        interval >= 0, that interval of the last batch (0 = its oldest) of a batched session."""
        import numpy as np
        dims = (c_int * 3)()
        n = lib().fh_session_debug_tensor_at(self._h, name.encode(), interval, None, 0, dims)
        if n < 0:
            raise _error()
        out = np.zeros(n, np.float32)
        _check(lib().fh_session_debug_tensor_at(self._h, name.encode(), interval,
                                                out.ctypes.data_as(POINTER(c_float)), n, dims))
        return out.reshape(dims[0], dims[1], dims[2])

    def close(self):
        if getattr(self, "_h", None):
            lib().fh_session_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except TypeError:  # interpreter shutdown: the module's globals are already gone, the process frees everything
            pass


_KIND = {0: "motion", 1: "cut", 2: "hold"}
_MODE = {"realtime": 0, "video": 1}


class Classification:
    """A pair's kind as Stream.classify found it: kind ("motion", "cut" or "hold"), mean and max cell difference (0..1),
    black (the frames are identical) and motion (the mean in the Pacer's 0..765 units)."""

    def __init__(self, c: _Classification):
        self.kind = _KIND.get(c.kind, "motion")
        self.mean, self.max, self.black, self.motion = c.mean, c.max, bool(c.black), c.motion

    def __repr__(self):
        return f"Classification({self.kind}, mean={self.mean:.4f}, max={self.max:.4f})"


class Push:
    """The interval a Stream.push made ready: ready, base_slot (its real first frame), stats_pending, start_pts,
    end_pts."""

    def __init__(self, p: _Push):
        self.ready, self.base_slot, self.stats_pending = bool(p.ready), p.base_slot, bool(p.stats_pending)
        self.start_pts, self.end_pts = p.start_pts, p.end_pts

    def __repr__(self):
        return f"Push(ready={self.ready}, base_slot={self.base_slot}, {self.start_pts}..{self.end_pts})"


class Stream:
    """Source frames with timestamps in, generatable intervals out (fh_stream_*).

    Stream(engine, model, width, height, mode="realtime" | "video", cadence=False, scene_cut=0.08 (0: never),
    held_frames=False | True | {"mean", "max"}, inputs=4, outputs=4, **session options). Realtime runs the pair of the
    previous and the newest frame at each push; video keeps one frame of lookahead. Re-timing of elements animated on
    twos (cadence) is not part of this build and is refused."""

    def __init__(self, engine: Engine, model: Model, width: int, height: int, mode: str = "realtime",
                 cadence: bool = False, scene_cut: float = 0.08, held_frames=False, inputs: int = 4, outputs: int = 4,
                 **session_opts):
        L = lib()
        self._so = session_options(width, height, **session_opts)
        o = L.fh_stream_options_default()
        o.mode = _MODE[mode]
        o.cadence = int(cadence)
        o.scene_cut = float(scene_cut)
        o.held_frames = int(bool(held_frames))
        if isinstance(held_frames, dict):
            o.held_mean = float(held_frames.get("mean", 0.0))
            o.held_max = float(held_frames.get("max", 0.0))
        o.inputs, o.outputs = inputs, outputs
        self.width, self.height = width, height
        self._e, self._m = engine, model
        self._h = L.fh_stream_create(engine._h, model._h, byref(self._so), byref(o))
        if not self._h:
            raise _error()

    def add_input(self) -> int:
        return _check(lib().fh_stream_add_input(self._h, self._e._h))

    def add_output(self) -> int:
        return _check(lib().fh_stream_add_output(self._h, self._e._h))

    def next_input(self, in_use=()) -> Optional[int]:
        """The slot to write the next frame into (never one the stream or the host still needs), or None."""
        arr = (c_uint32 * max(1, len(in_use)))(*in_use)
        slot = lib().fh_stream_next_input(self._h, arr, len(in_use))  # -1: the ring is exhausted (not an error)
        return None if slot < 0 else slot

    def write(self, slot: int, rgba) -> None:
        p, n, _keep = _buffer(rgba)
        _check(lib().fh_stream_write_rgba(self._h, self._e._h, slot, p, n))

    def write_device(self, slot: int, device_ptr: int, nbytes: int) -> None:
        """A frame already in device memory (a CUDA pointer) into an input slot."""
        _check(lib().fh_stream_write_rgba_device(self._h, slot, c_void_p(device_ptr), nbytes))

    def write_mask(self, mask) -> None:
        p, n, _keep = _buffer(mask)
        _check(lib().fh_stream_write_mask(self._h, self._e._h, p, n))

    def classify(self, previous: int, slot: int) -> Optional[Classification]:
        """The kind of the pair (previous, slot) before pushing it; None without a classifier (take it as motion)."""
        c = _Classification()
        return Classification(c) if _check(lib().fh_stream_classify(self._h, self._e._h, previous, slot,
                                                                    byref(c))) == 1 else None

    def push(self, slot: int, pts: float) -> Push:
        p = _Push()
        _check(lib().fh_stream_push(self._h, self._e._h, slot, pts, byref(p)))
        return Push(p)

    def resolve_stats(self) -> None:
        _check(lib().fh_stream_resolve_stats(self._h, self._e._h))

    def real_replaced(self) -> bool:
        return bool(_check(lib().fh_stream_real_replaced(self._h)))

    def generate(self, t: float, out: int) -> bool:
        """True when out holds phase t of the current interval; False when the source frame is enough (t <= 0)."""
        return _check(lib().fh_stream_generate(self._h, self._e._h, t, out)) == 1

    def read(self, out: int) -> bytes:
        n = self.width * self.height * 4
        buf = (c_uint8 * n)()
        _check(lib().fh_stream_read_rgba(self._h, self._e._h, out, ctypes.cast(buf, c_void_p), n))
        return bytes(buf)

    def warm_up(self) -> None:
        _check(lib().fh_stream_warm_up(self._h, self._e._h))

    def reset(self) -> None:
        _check(lib().fh_stream_reset(self._h))

    def mouse(self, t: float, dx: float, dy: float) -> None:
        _check(lib().fh_stream_mouse(self._h, self._e._h, t, dx, dy))

    def set_mouse_captured(self, captured: bool) -> None:
        _check(lib().fh_stream_set_mouse_captured(self._h, int(bool(captured))))

    def warp(self, slot: int, out: int, now: float, output: bool = False) -> bool:
        """The frame about to be presented at `now` (input slot, or output slot with output=True) turned by the mouse
        motion since the moment it shows, into output slot `out`: True = present `out`; False = the warp is off
        (present the frame as it is)."""
        return _check(lib().fh_stream_warp(self._h, self._e._h, int(output), slot, out, now)) == 1

    def camera_warp(self) -> Optional["Warp"]:
        """The stream's camera warp (started by the first mouse call), or None; it lives as long as the stream."""
        h = lib().fh_stream_camera_warp(self._h)
        return Warp._borrowed(h, self) if h else None

    def report(self) -> dict:
        return _json(lib().fh_stream_report_json, self._h)

    def close(self):
        if getattr(self, "_h", None):
            lib().fh_stream_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except TypeError:  # interpreter shutdown: the module's globals are already gone, the process frees everything
            pass


class Warp:
    """The camera warp (fh_warp_*, CameraWarp of warp/gpu.rs) over frames in device memory (rgba8, CUDA pointers).

    Warp(engine, width, height, hfov_deg=106). frame(ptr, t) measures the frame's shift against the previous one on the
    GPU; collect() hands finished measurements to the calibrator; render_shift / render_into turn a frame. Frames given
    to frame() must be complete on the device (synchronise the stream that wrote them, or write them on
    cuda_stream()), and stay unchanged until the next frame() call."""

    def __init__(self, engine: Engine, width: int, height: int, hfov_deg: float = 0.0):
        self.width, self.height = width, height
        self._owner = engine
        self._own = True
        self._h = lib().fh_warp_create(engine._h, width, height, hfov_deg)
        if not self._h:
            raise _error()

    @classmethod
    def _borrowed(cls, h, owner):
        w = cls.__new__(cls)
        w._h, w._owner, w._own = h, owner, False
        w.width, w.height = owner.width, owner.height
        return w

    def mouse(self, t: float, dx: float, dy: float) -> None:
        _check(lib().fh_warp_mouse(self._h, t, dx, dy))

    def set_captured(self, captured: bool) -> None:
        _check(lib().fh_warp_set_captured(self._h, int(bool(captured))))

    def break_pair(self) -> None:
        _check(lib().fh_warp_break_pair(self._h))

    def frame(self, device_ptr: int, t: float) -> None:
        _check(lib().fh_warp_frame(self._h, c_void_p(device_ptr), t))

    def collect(self, wait: bool = False) -> None:
        _check(lib().fh_warp_collect(self._h, int(wait)))

    def last_shift(self):
        """The last collected shift (pixels at the centre), or None when it could not be measured."""
        x, y = c_double(), c_double()
        return (x.value, y.value) if _check(lib().fh_warp_last_shift(self._h, byref(x), byref(y))) == 1 else None

    def shift(self, t_frame: float, now: float):
        x, y = c_double(), c_double()
        return (x.value, y.value) if _check(lib().fh_warp_shift(self._h, t_frame, now, byref(x), byref(y))) else None

    def decide(self, t_frame: float, now: float):
        x, y = c_double(), c_double()
        return (x.value, y.value) if _check(lib().fh_warp_decide(self._h, t_frame, now, byref(x), byref(y))) else None

    def render_shift(self, src_ptr: int, sx: float, sy: float) -> int:
        """src turned by (sx, sy) into the warp's own buffer; its device pointer (valid until the render after next)."""
        p = lib().fh_warp_render_shift(self._h, c_void_p(src_ptr), sx, sy)
        if not p:
            raise _error()
        return p

    def render_into(self, src_ptr: int, dst_ptr: int, sx: float, sy: float) -> None:
        _check(lib().fh_warp_render_into(self._h, c_void_p(src_ptr), c_void_p(dst_ptr), sx, sy))

    def cuda_stream(self) -> int:
        s = c_void_p()
        _check(lib().fh_warp_cuda_stream(self._h, byref(s)))
        return s.value or 0

    def read_mask(self):
        """The screen-locked mask as the lock wrote it, [ceil(h/8)][ceil(w/8)] float32."""
        import numpy as np
        gw, gh = (self.width + 7) // 8, (self.height + 7) // 8
        out = np.zeros((gh, gw), np.float32)
        _check(lib().fh_warp_read_mask(self._h, out.ctypes.data_as(POINTER(c_float)), out.size))
        return out

    def tensor(self, name: str):
        """A warp buffer as float32 (cells0..2, prev_cells0..2, best, sad, mask, grown)."""
        import numpy as np
        n = lib().fh_warp_debug_tensor(self._h, name.encode(), None, 0)
        if n < 0:
            raise _error()
        out = np.zeros(n, np.float32)
        _check(lib().fh_warp_debug_tensor(self._h, name.encode(), out.ctypes.data_as(POINTER(c_float)), n))
        return out

    def report(self) -> dict:
        return _json(lib().fh_warp_report_json, self._h)

    def close(self):
        if getattr(self, "_own", False) and getattr(self, "_h", None):
            lib().fh_warp_destroy(self._h)
        self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except TypeError:  # interpreter shutdown
            pass


class Generator:
    """Source frames in, the frames to display out, in order (fh_generator_*, api.rs Generator).

    Generator(engine, model, width, height, mode="realtime" | "video", k=1, internal=None, repair=1, render="model",
    keep_static=True, static_frames=8, static_tolerance=4, fast_render=False, linear_t=False). push(rgba, factor)
    queues the frames to display; pop() takes the next as (rgba bytes, phase, real), or None."""

    def __init__(self, engine: Engine, model: Model, width: int, height: int, mode: str = "realtime", k: int = 1,
                 internal=None, repair: int = 1, render: str = "model", keep_static: bool = True,
                 static_frames: int = 8, static_tolerance: int = 4, fast_render: bool = False,
                 linear_t: bool = False, cadence: bool = False):
        L = lib()
        o = L.fh_options_default(width, height)
        o.k, o.mode, o.repair, o.cadence = k, _MODE[mode], repair, int(cadence)
        if internal is not None:
            o.internal_w, o.internal_h = internal
        o.render_sampling = _RENDER[render]
        o.keep_static, o.static_frames, o.static_tolerance = int(keep_static), static_frames, static_tolerance
        o.fast_render, o.linear_t = int(fast_render), int(linear_t)
        self.width, self.height = width, height
        self._e, self._m = engine, model
        self._h = L.fh_generator_create(engine._h, model._h, byref(o))
        if not self._h:
            raise _error()

    def warmup(self) -> int:
        return _check(lib().fh_generator_warmup(self._h))

    def push(self, rgba, factor: int = 2) -> int:
        p, n, _keep = _buffer(rgba)
        return _check(lib().fh_generator_push(self._h, p, n, factor))

    def pop(self):
        n = self.width * self.height * 4
        buf = (c_uint8 * n)()
        phase, real = c_float(), c_int()
        if _check(lib().fh_generator_pop(self._h, ctypes.cast(buf, c_void_p), n, byref(phase), byref(real))) == 0:
            return None
        return bytes(buf), phase.value, bool(real.value)

    def frames(self, rgba, factor: int = 2) -> list:
        """push, then every queued frame as (rgba bytes, phase, real)."""
        self.push(rgba, factor)
        out = []
        while True:
            f = self.pop()
            if f is None:
                return out
            out.append(f)

    def close(self):
        if getattr(self, "_h", None):
            lib().fh_generator_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except TypeError:  # interpreter shutdown
            pass
