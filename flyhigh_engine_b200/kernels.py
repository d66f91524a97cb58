"""The kernel-level C ABI (include/flyhigh_kernels.h) from Python: ctypes mirrors of its parameter structs and a 3x3
conv on NHWC f16 device tensors, for hosts that drive the conv kernels without the session layer (and for bench.py's
per-conv sweep). Device memory is torch's; the kernels run on the caller's CUDA stream."""
from __future__ import annotations

import ctypes
from ctypes import Structure, c_float, c_int, c_longlong, c_void_p

import numpy as np

from . import FlyHighError, lib

MAX_SRC = 6


class ConvSrc(Structure):  # FhConvSrc
    _fields_ = [("p", c_void_p), ("bs", c_longlong), ("cs", c_int), ("nc", c_int), ("scale", c_float), ("slot", c_int)]


class ConvParams(Structure):  # FhConvParams
    _fields_ = [("src", ConvSrc * MAX_SRC), ("nsrc", c_int), ("h", c_int), ("w", c_int), ("ho", c_int), ("wo", c_int),
                ("cp", c_int), ("cout", c_int), ("wpack", c_void_p), ("bias", c_void_p), ("slope", c_void_p),
                ("epi", c_int), ("out", c_void_p), ("out_cs", c_int), ("out_bs", c_longlong), ("res", c_void_p),
                ("res_cs", c_int), ("res_bs", c_longlong), ("n", c_int), ("wm", c_int), ("ngroups", c_int),
                ("wsmem", c_int), ("wait_cycles", c_longlong), ("test_extra_tx", c_int)]


def _up8(c: int) -> int:
    return (c + 7) // 8 * 8


class Conv3x3:
    """One 3x3 conv layer (pad 1, bias, optional PReLU slopes, optional residual) on NHWC f16 torch tensors.

    kernel "mma" (fhk_conv3x3: mma.sync, stride 1 or 2; wm = rows per CTA pair, 0 = by size) or "umma"
    (fhk_conv3x3_umma: tcgen05, stride 1 where fhk_conv_umma_fits; wm 1 = its persistent variant). weight: [cout][cin][3][3] (float values, rounded
    to f16); the input tensor is [n][h][w][cs] with cs = 4 for cin <= 4 else cin rounded up to 8."""

    def __init__(self, weight, bias, slope=None, stride: int = 1, kernel: str = "mma", wm: int = 0, device="cuda"):
        import torch
        L = lib()
        w = np.asarray(weight, np.float32)
        self.cout, self.cin = int(w.shape[0]), int(w.shape[1])
        self.stride, self.kernel, self.wm = int(stride), kernel, int(wm)
        self.cs = 4 if self.cin <= 4 else _up8(self.cin)
        self.cp = (_up8(self.cin) + 15) // 16 * 16
        umma = kernel == "umma"
        if umma and not (stride == 1 and L.fhk_conv_umma_fits(self.cp, self.cout, 1)):
            raise FlyHighError(f"conv {self.cin}->{self.cout} stride {stride}: the tcgen05 kernel does not take it")
        if umma and wm == 1 and not L.fhk_conv_umma_persistent_fits(self.cp, self.cout):
            raise FlyHighError(f"conv {self.cin}->{self.cout}: the persistent tcgen05 variant does not take it")
        cmap = np.full(self.cp, -1, np.int32)
        cmap[:self.cin] = np.arange(self.cin)
        n_pack = (L.fhk_conv_packed_elems_umma if umma else L.fhk_conv_packed_elems)(self.cout, self.cp)
        packed = np.zeros(n_pack, np.uint16)
        bits = np.ascontiguousarray(w.astype(np.float16)).view(np.uint16)
        pack = L.fhk_conv_pack_weights_umma if umma else L.fhk_conv_pack_weights
        if pack(bits.ctypes.data, self.cin, self.cout, cmap.ctypes.data, self.cp, packed.ctypes.data) != 0:
            raise FlyHighError("weight packing failed")
        self.wpack = torch.from_numpy(packed.view(np.int16)).to(device)
        self.bias = torch.from_numpy(np.asarray(bias, np.float32)).to(device)
        self.slope = None if slope is None else torch.from_numpy(np.asarray(slope, np.float32)).to(device)
        self.ocs = _up8(self.cout)

    def out_shape(self, n: int, h: int, w: int):
        return (n, (h - 1) // self.stride + 1, (w - 1) // self.stride + 1, self.ocs)

    def params(self, x, out, res=None) -> ConvParams:
        n, h, w, cs = x.shape
        assert cs == self.cs and tuple(out.shape) == self.out_shape(n, h, w)
        p = ConvParams()
        p.src[0] = ConvSrc(x.data_ptr(), h * w * cs, cs, self.cin, 1.0, 0)
        p.nsrc, p.h, p.w = 1, h, w
        p.ho, p.wo = out.shape[1], out.shape[2]
        p.cp, p.cout = self.cp, self.cout
        p.wpack, p.bias = self.wpack.data_ptr(), self.bias.data_ptr()
        p.slope = self.slope.data_ptr() if self.slope is not None else None
        p.out, p.out_cs, p.out_bs = out.data_ptr(), self.ocs, out.shape[1] * out.shape[2] * self.ocs
        if res is not None:
            assert tuple(res.shape) == tuple(out.shape)
            p.res, p.res_cs, p.res_bs = res.data_ptr(), self.ocs, p.out_bs
        p.n, p.wm = n, self.wm
        return p

    def launch(self, p: ConvParams, stream: int) -> None:
        L = lib()
        st = c_void_p(stream)
        rc = L.fhk_conv3x3_umma(ctypes.byref(p), st) if self.kernel == "umma" else \
            L.fhk_conv3x3(ctypes.byref(p), self.stride, st)
        if rc != 0:
            raise FlyHighError(f"conv launch failed: CUDA error {rc}")

    def __call__(self, x, res=None, out=None):
        import torch
        n, h, w, _ = x.shape
        if out is None:
            out = torch.zeros(self.out_shape(n, h, w), dtype=torch.float16, device=x.device)
        self.launch(self.params(x, out, res), torch.cuda.current_stream().cuda_stream)
        return out
