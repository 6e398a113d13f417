"""GEMM host interface: the reference's GEMM descriptor API on the mm4 C ABI.

Mirrors Sources/matmul/matmul.swift: `GEMMDimensions` (:5-9), `BuildOptions`
(:11-16) and createSource(matrixDimensions:blockDimensions:transpose:bias:
buildOptions:) + run(...) (:18-329, :345-511). A `GemmPlan` plays the role of
the generated, compiled kernel; `GemmPlan.run` the role of the dispatch.
Tensors are torch CUDA tensors (fp16); the math runs in libmm4.so.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

from . import _lib


@dataclass
class GEMMDimensions:
    M: int
    N: int
    K: int


@dataclass
class BuildOptions:
    cooperativeExecutionSIMDGroups: int = 4
    preemptiveExecutionSIMDGroups: int = 1
    swapMN: bool = False
    splitK: int = 1


class GemmPlan:
    """One GEMM shape + options, dispatched to an sm_100a kernel instance.

    transpose = (left, right) keeps the reference's meaning
    (matmul.swift:80-117): left=False -> A is [M][K]; right=True -> B is
    [N][K] (the reference default); right=False -> B is [K][N] (row-major NN).
    """

    def __init__(self, matrixDimensions: GEMMDimensions, blockDimensions: GEMMDimensions | None = None,
                 transpose: tuple[bool, bool] = (False, True), bias: bool = True,
                 buildOptions: BuildOptions | None = None):
        bo = buildOptions or BuildOptions()
        bd = blockDimensions or GEMMDimensions(0, 0, 0)
        self.dims = matrixDimensions
        self.transpose = (bool(transpose[0]), bool(transpose[1]))
        self.bias = bool(bias)
        self.options = bo
        desc = _lib.GemmDesc(matrixDimensions.M, matrixDimensions.N, matrixDimensions.K, int(transpose[0]),
                             int(transpose[1]), int(bias), int(bo.splitK), bd.M, bd.N, bd.K,
                             int(bo.cooperativeExecutionSIMDGroups), int(bo.preemptiveExecutionSIMDGroups),
                             int(bo.swapMN))
        self._L = _lib.lib()
        handle = ctypes.c_void_p()
        _lib.check(self._L.mm4_gemm_plan_create(ctypes.byref(handle), ctypes.byref(desc)))
        self._h = handle
        self.workspace_bytes = int(self._L.mm4_gemm_workspace_size(handle))
        self.kernel_name = self._L.mm4_gemm_plan_kernel_name(handle).decode()
        self._ws = {}

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            self._L.mm4_gemm_plan_destroy(h)
            self._h = None

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._h

    def workspace(self, device):
        """A zero-filled workspace for this plan on `device` (kernels leave it zeroed)."""
        import torch
        if self.workspace_bytes == 0:
            return None
        key = str(device)
        if key not in self._ws:
            self._ws[key] = torch.zeros(self.workspace_bytes, dtype=torch.uint8, device=device)
        return self._ws[key]

    def a_shape(self):
        d = self.dims
        return (d.K, d.M) if self.transpose[0] else (d.M, d.K)

    def b_shape(self):
        d = self.dims
        return (d.N, d.K) if self.transpose[1] else (d.K, d.N)

    def run(self, A, B, bias=None, C=None, workspace=None, stream=None, duplicatedCount: int = 1):
        """C = A*B (+bias) on the GPU; returns C ([M][N] fp16)."""
        import torch
        d = self.dims
        _check_tensor(A, self.a_shape(), "A")
        _check_tensor(B, self.b_shape(), "B")
        if self.bias:
            _check_tensor(bias, (d.N,), "bias")
        if C is None:
            C = torch.empty((d.M, d.N), dtype=torch.float16, device=A.device)
        ws = workspace if workspace is not None else self.workspace(A.device)
        _lib.check(self._L.mm4_gemm_run(self._h, A.data_ptr(), B.data_ptr(), bias.data_ptr() if self.bias else None,
                                        C.data_ptr(), ws.data_ptr() if ws is not None else None,
                                        ws.numel() if ws is not None else 0, _lib.stream_handle(stream),
                                        int(duplicatedCount)))
        return C

    def partial(self, A, B, C32=None, workspace=None, stream=None):
        """fp32 partial A*B over this plan's K (no bias), for cross-rank split-K."""
        import torch
        d = self.dims
        _check_tensor(A, self.a_shape(), "A")
        _check_tensor(B, self.b_shape(), "B")
        if C32 is None:
            C32 = torch.empty((d.M, d.N), dtype=torch.float32, device=A.device)
        ws = workspace if workspace is not None else self.workspace(A.device)
        _lib.check(self._L.mm4_gemm_partial_run(self._h, A.data_ptr(), B.data_ptr(), C32.data_ptr(),
                                                ws.data_ptr() if ws is not None else None,
                                                ws.numel() if ws is not None else 0, _lib.stream_handle(stream)))
        return C32


def splitk_finalize(C32, bias, C=None, stream=None):
    """C = fp16(C32 + bias): the bias/cast step after summing fp32 partials."""
    import torch
    M, N = C32.shape
    if C is None:
        C = torch.empty((M, N), dtype=torch.float16, device=C32.device)
    L = _lib.lib()
    _lib.check(L.mm4_splitk_finalize(M, N, C32.data_ptr(), bias.data_ptr() if bias is not None else None,
                                     C.data_ptr(), _lib.stream_handle(stream)))
    return C


def _check_tensor(t, shape, name):
    import torch
    if t is None:
        raise ValueError(f"{name} is required")
    if not t.is_cuda or t.dtype != torch.float16:
        raise ValueError(f"{name} must be a CUDA float16 tensor")
    if tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name} has shape {tuple(t.shape)}, expected {tuple(shape)}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
