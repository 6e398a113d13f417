"""Convolution host interface: the reference's conv descriptors on the mm4 C ABI.

Mirrors Sources/ConvolutionShared/ConvolutionShared.swift: `Conv2DDimensions`
(:5-70), `Conv3DDimensions` (:72-153, plus depth padding as an extension),
the tensor-op sessions (:844-1575) as `ConvPlan`, and the weight permutation
session (:1577-1675) as `permute_weights`. Activations are NHWC / NDHWC,
outputs NHWO / NDHWO, fp16; the math runs in libmm4.so.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

from . import _lib
from ._lib import (WEIGHTS_DHWIO, WEIGHTS_HWIO, WEIGHTS_ODHWI, WEIGHTS_OHWI, WEIGHTS_OIDHW,  # noqa: F401
                   WEIGHTS_OIHW)


def _out(inp, plo, phi, k, s, d):
    return (inp + plo + phi - ((k - 1) * d + 1)) // s + 1


@dataclass
class Conv2DDimensions:
    batchSize: int
    inputHeight: int
    inputWidth: int
    inputChannels: int
    outputChannels: int
    kernelHeight: int
    kernelWidth: int
    strideY: int = 1
    strideX: int = 1
    dilationY: int = 1
    dilationX: int = 1
    paddingTop: int = 0
    paddingBottom: int = 0
    paddingLeft: int = 0
    paddingRight: int = 0

    @property
    def outputHeight(self):
        return _out(self.inputHeight, self.paddingTop, self.paddingBottom, self.kernelHeight, self.strideY,
                    self.dilationY)

    @property
    def outputWidth(self):
        return _out(self.inputWidth, self.paddingLeft, self.paddingRight, self.kernelWidth, self.strideX,
                    self.dilationX)

    def flops(self) -> float:
        """operationsCount (ConvolutionShared.swift:5324-5330): 2*N*OH*OW*O*KH*KW*C."""
        return 2.0 * self.batchSize * self.outputHeight * self.outputWidth * self.outputChannels * \
            self.kernelHeight * self.kernelWidth * self.inputChannels


@dataclass
class Conv3DDimensions:
    batchSize: int
    inputDepth: int
    inputHeight: int
    inputWidth: int
    inputChannels: int
    outputChannels: int
    kernelDepth: int
    kernelHeight: int
    kernelWidth: int
    strideZ: int = 1
    strideY: int = 1
    strideX: int = 1
    dilationZ: int = 1
    dilationY: int = 1
    dilationX: int = 1
    paddingTop: int = 0
    paddingBottom: int = 0
    paddingLeft: int = 0
    paddingRight: int = 0
    paddingFront: int = 0   # extension: the reference has no depth padding
    paddingBack: int = 0

    @property
    def outputDepth(self):
        return _out(self.inputDepth, self.paddingFront, self.paddingBack, self.kernelDepth, self.strideZ,
                    self.dilationZ)

    @property
    def outputHeight(self):
        return _out(self.inputHeight, self.paddingTop, self.paddingBottom, self.kernelHeight, self.strideY,
                    self.dilationY)

    @property
    def outputWidth(self):
        return _out(self.inputWidth, self.paddingLeft, self.paddingRight, self.kernelWidth, self.strideX,
                    self.dilationX)

    def flops(self) -> float:
        """operationsCount 3-D (ConvolutionShared.swift:5343-5352): 2*N*OD*OH*OW*O*KD*KH*KW*C."""
        return 2.0 * self.batchSize * self.outputDepth * self.outputHeight * self.outputWidth * \
            self.outputChannels * self.kernelDepth * self.kernelHeight * self.kernelWidth * self.inputChannels


@dataclass
class BuildOptions:
    """The reference's conv BuildOptions (ConvolutionShared.swift:155-185). mm4 chooses its own tiles
    (128- or 256-pixel implicit-GEMM tiles, see `ConvPlan.tile_grid`); these fields are accepted as
    tuning hints and recorded in harness reports."""
    executionSIMDGroups: int = 1
    outputTileWidth: int | None = None
    outputTileHeight: int | None = None
    outputBaseX: int | None = None
    outputBaseY: int | None = None
    dispatchGridWidth: int | None = None
    dispatchGridHeight: int | None = None

    @property
    def usesOutputTiling(self) -> bool:
        return self.outputTileWidth is not None and self.outputTileHeight is not None


class ConvPlan:
    """A conv2d/conv3d shape + weight layout dispatched to the implicit-GEMM kernel."""

    def __init__(self, dims, weight_layout: int | None = None, bias: bool = False):
        self._L = _lib.lib()
        self.dims = dims
        self.bias = bool(bias)
        handle = ctypes.c_void_p()
        if isinstance(dims, Conv2DDimensions):
            self.weight_layout = WEIGHTS_HWIO if weight_layout is None else weight_layout
            d = _lib.Conv2dDesc(dims.batchSize, dims.inputHeight, dims.inputWidth, dims.inputChannels,
                                dims.outputChannels, dims.kernelHeight, dims.kernelWidth, dims.strideY, dims.strideX,
                                dims.dilationY, dims.dilationX, dims.paddingTop, dims.paddingBottom,
                                dims.paddingLeft, dims.paddingRight, self.weight_layout, int(bias))
            _lib.check(self._L.mm4_conv2d_plan_create(ctypes.byref(handle), ctypes.byref(d)))
            self.out_shape = (dims.batchSize, dims.outputHeight, dims.outputWidth, dims.outputChannels)
            self.in_shape = (dims.batchSize, dims.inputHeight, dims.inputWidth, dims.inputChannels)
            kd = 1
        else:
            self.weight_layout = WEIGHTS_DHWIO if weight_layout is None else weight_layout
            d = _lib.Conv3dDesc(dims.batchSize, dims.inputDepth, dims.inputHeight, dims.inputWidth,
                                dims.inputChannels, dims.outputChannels, dims.kernelDepth, dims.kernelHeight,
                                dims.kernelWidth, dims.strideZ, dims.strideY, dims.strideX, dims.dilationZ,
                                dims.dilationY, dims.dilationX, dims.paddingTop, dims.paddingBottom,
                                dims.paddingLeft, dims.paddingRight, dims.paddingFront, dims.paddingBack,
                                self.weight_layout, int(bias))
            _lib.check(self._L.mm4_conv3d_plan_create(ctypes.byref(handle), ctypes.byref(d)))
            self.out_shape = (dims.batchSize, dims.outputDepth, dims.outputHeight, dims.outputWidth,
                              dims.outputChannels)
            self.in_shape = (dims.batchSize, dims.inputDepth, dims.inputHeight, dims.inputWidth, dims.inputChannels)
            kd = dims.kernelDepth
        self._h = handle
        self.kernel_name = self._L.mm4_conv_plan_kernel_name(handle).decode()
        self.weight_elements = dims.outputChannels * dims.inputChannels * kd * dims.kernelHeight * dims.kernelWidth

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            self._L.mm4_conv_plan_destroy(h)
            self._h = None

    @property
    def handle(self):
        return self._h

    def tile_grid(self) -> tuple[int, int, int]:
        """Output tiles of the launch (pixel tiles, channel tiles, 1): the analogue of the reference's
        threadgroup dispatch grid."""
        g = (ctypes.c_int32 * 3)()
        _lib.check(self._L.mm4_conv_plan_tile_grid(self._h, g))
        return (g[0], g[1], g[2])

    def run(self, x, w, bias=None, y=None, stream=None, duplicatedCount: int = 1):
        import torch
        if tuple(x.shape) != self.in_shape or x.dtype != torch.float16 or not x.is_cuda or not x.is_contiguous():
            raise ValueError(f"x must be a contiguous CUDA fp16 tensor of shape {self.in_shape}")
        if w.numel() != self.weight_elements or w.dtype != torch.float16 or not w.is_cuda or not w.is_contiguous():
            raise ValueError("w must be a contiguous CUDA fp16 tensor in the plan's weight layout")
        if self.bias and (bias is None or bias.numel() != self.dims.outputChannels):
            raise ValueError("bias of Cout elements is required")
        if y is None:
            y = torch.empty(self.out_shape, dtype=torch.float16, device=x.device)
        _lib.check(self._L.mm4_conv_run(self._h, x.data_ptr(), w.data_ptr(),
                                        bias.data_ptr() if self.bias else None, y.data_ptr(),
                                        _lib.stream_handle(stream), int(duplicatedCount)))
        return y

    def run_host(self, x, w, bias, y, staging, chunks: int = 16, stream=None):
        """y = conv(x, w) (+bias) for CPU tensors (pinned for the copies to overlap) through the CUDA tensors
        staging = (dx, dw, dbias, dy) of the full shapes (dbias may be None without bias): the weights and
        bias are copied in first, then groups of batch elements are copied in, convolved and copied out as a
        pipeline over `chunks` pieces (mm4_conv_run_host). Ordered on `stream`."""
        import torch
        dx, dw, db, dy = staging
        for name, t, shape, cuda in (("x", x, self.in_shape, False), ("y", y, self.out_shape, False),
                                     ("dx", dx, self.in_shape, True), ("dy", dy, self.out_shape, True)):
            if t.is_cuda != cuda or t.dtype != torch.float16 or not t.is_contiguous() or tuple(t.shape) != shape:
                where = "CUDA" if cuda else "CPU"
                raise ValueError(f"{name} must be a contiguous {where} fp16 tensor of shape {shape}")
        for name, t, cuda in (("w", w, False), ("dw", dw, True)):
            if t.numel() != self.weight_elements or t.dtype != torch.float16 or t.is_cuda != cuda \
                    or not t.is_contiguous():
                raise ValueError(f"{name} must hold the plan's weights as contiguous fp16")
        if self.bias:
            for name, t, cuda in (("bias", bias, False), ("dbias", db, True)):
                if t is None or t.numel() != self.dims.outputChannels or t.is_cuda != cuda:
                    raise ValueError(f"{name} of Cout elements is required")
        _lib.check(self._L.mm4_conv_run_host(
            self._h, x.data_ptr(), w.data_ptr(), bias.data_ptr() if self.bias else None, y.data_ptr(),
            dx.data_ptr(), dw.data_ptr(), db.data_ptr() if self.bias else None, dy.data_ptr(), int(chunks),
            _lib.stream_handle(stream)))
        return y


def permute_weights(src, from_layout: int, to_layout: int, dims5, stream=None, dst=None):
    """Weight layout transform on the GPU; dims5 = (Cout, Cin, KD, KH, KW). Writes `dst` (same size as
    src) when given, else a new tensor."""
    import torch
    L = _lib.lib()
    if dst is None:
        dst = torch.empty_like(src)
    elif dst.numel() != src.numel() or dst.dtype != src.dtype:
        raise ValueError("dst must match src in size and dtype")
    arr = (ctypes.c_int32 * 5)(*dims5)
    _lib.check(L.mm4_permute_weights(from_layout, to_layout, arr, src.data_ptr(), dst.data_ptr(),
                                     _lib.stream_handle(stream)))
    return dst
