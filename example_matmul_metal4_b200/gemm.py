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

    def run_host(self, A, B, bias, C, staging, workspace=None, chunks: int = 16, stream=None):
        """C = A*B (+bias) for CPU tensors (pinned for the copies to overlap) through the CUDA tensors
        staging = (dA, dB, dbias, dC) of the full shapes (dbias may be None without bias): B and bias are
        copied in first, then A's row blocks, their GEMMs and C's row blocks run as a pipeline over
        `chunks` pieces (mm4_gemm_run_host). Ordered on `stream`."""
        import torch
        d = self.dims
        dA, dB, db, dC = staging
        _check_tensor(dA, self.a_shape(), "dA")
        _check_tensor(dB, self.b_shape(), "dB")
        _check_tensor(dC, (d.M, d.N), "dC")
        if self.bias:
            _check_tensor(db, (d.N,), "dbias")
        for name, h, shape in (("A", A, self.a_shape()), ("B", B, self.b_shape()), ("C", C, (d.M, d.N))):
            if h.is_cuda or h.dtype != torch.float16 or not h.is_contiguous() or tuple(h.shape) != tuple(shape):
                raise ValueError(f"{name} must be a contiguous CPU fp16 tensor of shape {tuple(shape)}")
        ws = workspace if workspace is not None else self.workspace(dA.device)
        _lib.check(self._L.mm4_gemm_run_host(
            self._h, A.data_ptr(), B.data_ptr(), bias.data_ptr() if self.bias else None, C.data_ptr(),
            dA.data_ptr(), dB.data_ptr(), db.data_ptr() if self.bias else None, dC.data_ptr(),
            ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0, int(chunks),
            _lib.stream_handle(stream)))
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


@dataclass
class RunResult:
    """What the reference's run(...) prints, as a record: GFLOP/s over the GPU time of the launches, and
    the elements farther than 5e-3 from the fp32 expectation."""
    gflops: float
    latencyMS: float
    maxAbsoluteError: float
    mismatches: int
    kernel: str


def _gpu_time(launch, duplicatedCount: int) -> float:
    """Seconds of GPU time of `duplicatedCount` launches (CUDA events around them)."""
    import torch

    from ._lib import sync_check
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record()
    for _ in range(duplicatedCount):
        launch()
    end.record()
    sync_check()
    return start.elapsed_time(end) / 1e3


def _check(expected, got, name: str, tolerance: float, log) -> tuple[float, int]:
    import numpy as np
    err = np.abs(expected - got)
    bad = np.argwhere(err > tolerance)
    for idx in bad[:8]:
        i = tuple(int(v) for v in idx)
        log(f"CPU calculated {name}{list(i)}: {expected[i]}")
        log(f"GPU calculated {name}{list(i)}: {got[i]}")
    return float(err.max()) if err.size else 0.0, int(len(bad))


def run(M: int, N: int, K: int, blockDimensions: GEMMDimensions | None = None,
        buildOptions: BuildOptions | None = None, duplicatedCount: int = 1, seed: int = 1,
        log=print) -> RunResult:
    """The reference's matmul run(M:N:K:blockDimensions:buildOptions:duplicatedCount:) (matmul.swift:345-511):
    A [M][K], B [N][K] (transpose right), bias [N], each U[0,1] * (1/sqrt K) in fp16 (:406-415; drawn here on
    the device from a seeded generator); `duplicatedCount` launches; "GFlops" over their GPU time (:481-489);
    every element of C checked against bias + A B^T in fp32 with tolerance 5e-3 (:499-510), the expectation
    formed on the device in fp32 with TF32 off."""
    import numpy as np
    import torch
    bo = buildOptions or BuildOptions()
    bo = BuildOptions(bo.cooperativeExecutionSIMDGroups, bo.preemptiveExecutionSIMDGroups, M > N, bo.splitK)
    dev = torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    nf = float(np.float16(1 / np.sqrt(K)))

    def scaled(shape):  # fp16(U) * fp16(1/sqrt K), one fp16 rounding of the product, as in Swift's Float16 math
        return (torch.rand(shape, generator=gen, device=dev).half().float() * nf).half()

    tA, tB, tb = scaled((M, K)), scaled((N, K)), scaled((N,))
    plan = GemmPlan(GEMMDimensions(M, N, K), blockDimensions, transpose=(False, True), bias=True, buildOptions=bo)
    C = torch.empty((M, N), dtype=torch.float16, device=dev)
    ws = plan.workspace(dev)
    seconds = _gpu_time(lambda: plan.run(tA, tB, tb, C=C, workspace=ws), duplicatedCount)
    gflops = 2.0 * M * N * K * duplicatedCount / seconds / 1e9 if seconds > 0 else 0.0
    log(f"GFlops: {int(gflops)}")
    tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        expected = torch.addmm(tb.float(), tA.float(), tB.float().T).cpu().numpy()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = tf32
    max_err, bad = _check(expected, C.float().cpu().numpy(), "C", 5e-3, log)
    return RunResult(gflops, seconds * 1e3, max_err, bad, plan.kernel_name)


def profileCorrectness(sizes=range(1, 16385), log=print) -> list[RunResult]:
    """The reference's square sweep (matmul.swift:337-342): run(i, i, i) with 32x64x64 block hints,
    1 cooperative / 4 preemptive SIMD groups. The full 1..16384 range checks each size on the host and
    takes hours; pass a smaller `sizes`."""
    out = []
    for i in sizes:
        log(f"Problem size: {i}")
        out.append(run(i, i, i, GEMMDimensions(32, 64, 64), BuildOptions(1, 4, True, 1), 1, log=log))
    return out
