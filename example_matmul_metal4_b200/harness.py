"""ConvolutionHarness: the reference's conv validation and profiling entry points and their reports,
on the mm4 path.

Mirrors Sources/ConvolutionShared/ConvolutionShared.swift:
- the report structs (ValidationResult ... ConvolutionProfileResult, :187-622) as dataclasses with the
  same field names; `to_dict()` / `to_json()` give the keys Swift's synthesized Codable writes (stored
  properties, nil optionals left out), so reports read like the reference app's (RunModel.swift:6-28);
- `ConvolutionHarness` (:2134-3411) with the same entry points, defaults and case lists.

What stands where on B200:
- the tensor-op session is the mm4 implicit-GEMM conv (`ConvPlan`: libmm4.so on the GPU);
- the expected values (referenceConvolution / referenceConvolutionWithBias, :4994-5096) are the fp32
  convolution of the reference's formula data (createActivationData / createWeightData / createBiasData,
  :4874-4990), computed by torch on the host;
- the MPSGraph slots (`mpsGraphValidation`, `backendAgreement`, `mpsGraph`, `mpsGraphWallLatencyMS`)
  hold torch's cuDNN convolution on the same GPU (fp16, channels-last): this platform's library path, as
  MPSGraph is Apple's;
- wall latency is host time around the launches, their completion and (for `run`) the read-back; GPU
  latency is CUDA events around the launches.
Validation is the reference's: an absolute error above 2e-2 is a mismatch (validateOutput /
compareOutputs, :5174-5322), and permuted weights must match exactly (validateFlatOutput, :5381-5405).
The Apple-only entry points (GPU trace capture, MPSGraph weight-layout sweeps, the tensor-op variant
debug sweep) have no counterpart.
"""
from __future__ import annotations

import json
import time
from dataclasses import dataclass, fields, is_dataclass
from typing import Callable

import numpy as np

from . import data
from .conv import (WEIGHTS_DHWIO, WEIGHTS_HWIO, WEIGHTS_OIDHW, BuildOptions, Conv2DDimensions, Conv3DDimensions,
                   ConvPlan, permute_weights)

TOLERANCE = 2e-2  # validateOutput / compareOutputs (ConvolutionShared.swift:5183)

Log = Callable[[str], None]


def _quiet(_: str) -> None:
    pass


# ---------------------------------------------------------------------------
# reports (ConvolutionShared.swift:187-622)
# ---------------------------------------------------------------------------

def _encode(obj):
    if is_dataclass(obj):
        return {f.name: _encode(getattr(obj, f.name)) for f in fields(obj) if getattr(obj, f.name) is not None}
    if isinstance(obj, (list, tuple)):
        return [_encode(v) for v in obj]
    if isinstance(obj, (np.floating, np.integer)):
        return obj.item()
    return obj


class _Codable:
    def to_dict(self) -> dict:
        return _encode(self)

    def to_json(self, **kw) -> str:
        return json.dumps(self.to_dict(), **kw)


@dataclass
class ValidationResult(_Codable):
    maxAbsoluteError: float
    mismatches: int


@dataclass
class ConvolutionCaseResult(_Codable):
    dimensions: Conv2DDimensions
    tensorOpValidation: ValidationResult
    mpsGraphValidation: ValidationResult
    backendAgreement: ValidationResult
    tensorOpWallLatencyMS: float | None
    tensorOpGPULatencyMS: float | None
    mpsGraphWallLatencyMS: float | None


@dataclass
class ConvolutionValidationSuiteResult(_Codable):
    deviceName: str
    allPassed: bool
    cases: list


@dataclass
class ProfileOptions(_Codable):
    warmupIterations: int
    timedIterations: int
    duplicatedCount: int = 1


@dataclass
class BackendProfileResult(_Codable):
    averageWallLatencyMS: float
    averageGPULatencyMS: float | None
    throughputGFLOPS: float


@dataclass
class DispatchGridSize(_Codable):
    width: int
    height: int
    depth: int


@dataclass
class TensorOpTileRegionProfileResult(_Codable):
    label: str
    buildOptions: BuildOptions
    dispatchGrid: DispatchGridSize
    averageWallLatencyMS: float
    averageGPULatencyMS: float | None


@dataclass
class TensorOpTileProfileResult(_Codable):
    dimensions: Conv2DDimensions
    tileWidth: int
    tileHeight: int
    options: ProfileOptions
    regions: list
    averageWallLatencyMS: float
    averageGPULatencyMS: float | None
    wallThroughputGFLOPS: float
    gpuThroughputGFLOPS: float | None


@dataclass
class Convolution3DCaseResult(_Codable):
    dimensions: Conv3DDimensions
    tensorOpValidation: ValidationResult
    tensorOpWallLatencyMS: float | None
    tensorOpGPULatencyMS: float | None


@dataclass
class Convolution3DValidationSuiteResult(_Codable):
    deviceName: str
    allPassed: bool
    cases: list


@dataclass
class TensorOpConv3DProfileResult(_Codable):
    dimensions: Conv3DDimensions
    buildOptions: BuildOptions
    options: ProfileOptions
    dispatchGrid: DispatchGridSize
    averageWallLatencyMS: float
    averageGPULatencyMS: float | None
    wallThroughputGFLOPS: float
    gpuThroughputGFLOPS: float | None


@dataclass
class TensorOpConv3DPermutationProfileResult(_Codable):
    validationDimensions: Conv3DDimensions
    profileDimensions: Conv3DDimensions
    buildOptions: BuildOptions
    options: ProfileOptions
    permutationValidation: ValidationResult
    combinedValidation: ValidationResult
    permutationAverageWallLatencyMS: float
    permutationAverageGPULatencyMS: float | None
    permutationWallBandwidthGBPS: float
    permutationGPUBandwidthGBPS: float | None
    combinedAverageWallLatencyMS: float
    combinedAverageGPULatencyMS: float | None
    combinedWallThroughputGFLOPS: float
    combinedGPUThroughputGFLOPS: float | None


@dataclass
class ConvolutionProfileResult(_Codable):
    dimensions: Conv2DDimensions
    options: ProfileOptions
    tensorOpValidation: ValidationResult
    mpsGraphValidation: ValidationResult
    backendAgreement: ValidationResult
    tensorOp: BackendProfileResult
    mpsGraph: BackendProfileResult


# ---------------------------------------------------------------------------
# validators and work accounting (ConvolutionShared.swift:5174-5405)
# ---------------------------------------------------------------------------

def _mismatch_report(err: np.ndarray, lhs: np.ndarray, rhs: np.ndarray, tolerance: float, message, log: Log):
    bad = err > tolerance
    for idx in np.argwhere(bad)[:8]:
        log(message(tuple(int(i) for i in idx), float(lhs[tuple(idx)]), float(rhs[tuple(idx)])))
    return ValidationResult(maxAbsoluteError=float(err.max()) if err.size else 0.0, mismatches=int(bad.sum()))


def _coords(idx) -> str:
    names = ("n", "h", "w", "o") if len(idx) == 4 else ("n", "z", "h", "w", "o")
    return ", ".join(f"{k}={v}" for k, v in zip(names, idx))


def validateOutput(actual, expected, label: str = "", log: Log = _quiet) -> ValidationResult:
    """Absolute error above 2e-2 counts as a mismatch; the first 8 are logged (:5174-5240).
    Outputs are [N][(D)][H][W][O] arrays."""
    actual = np.asarray(actual, dtype=np.float32)
    expected = np.asarray(expected, dtype=np.float32)
    if actual.shape != expected.shape:
        raise ValueError(f"{label}: shape {actual.shape} != expected {expected.shape}")
    err = np.abs(expected - actual)
    return _mismatch_report(err, expected, actual, TOLERANCE,
                            lambda i, e, a: f"{label} mismatch at {_coords(i)}: expected {e}, got {a}", log)


def compareOutputs(lhs, rhs, lhsLabel: str = "", rhsLabel: str = "", log: Log = _quiet) -> ValidationResult:
    """Backend agreement with the same rule (:5242-5322)."""
    lhs = np.asarray(lhs, dtype=np.float32)
    rhs = np.asarray(rhs, dtype=np.float32)
    if lhs.shape != rhs.shape:
        raise ValueError(f"{lhsLabel} vs {rhsLabel}: shape {lhs.shape} != {rhs.shape}")
    err = np.abs(lhs - rhs)
    return _mismatch_report(err, lhs, rhs, TOLERANCE,
                            lambda i, a, b: f"{lhsLabel} vs {rhsLabel} mismatch at {_coords(i)}: {a} vs {b}", log)


def validateFlatOutput(actual, expected, label: str = "", log: Log = _quiet) -> ValidationResult:
    """Element-wise exact comparison of flat arrays (tolerance 0, :5381-5405)."""
    actual = np.asarray(actual, dtype=np.float32).reshape(-1)
    expected = np.asarray(expected, dtype=np.float32).reshape(-1)
    if actual.shape != expected.shape:
        raise ValueError(f"{label}: {actual.size} elements != expected {expected.size}")
    err = np.abs(actual - expected)
    bad = err > 0
    for i in np.flatnonzero(bad)[:8]:
        log(f"{label} mismatch at linear index {int(i)}: expected {float(expected[i])}, got {float(actual[i])}")
    return ValidationResult(maxAbsoluteError=float(err.max()) if err.size else 0.0, mismatches=int(bad.sum()))


def operationsCount(dimensions, duplicatedCount: int = 1) -> int:
    """2*N*(OD)*OH*OW*O*(KD)*KH*KW*C per launch (:5324-5352)."""
    d = dimensions
    if isinstance(d, Conv3DDimensions):
        return (2 * d.batchSize * d.outputDepth * d.outputHeight * d.outputWidth * d.outputChannels * d.kernelDepth
                * d.kernelHeight * d.kernelWidth * d.inputChannels * duplicatedCount)
    return (2 * d.batchSize * d.outputHeight * d.outputWidth * d.outputChannels * d.kernelHeight * d.kernelWidth
            * d.inputChannels * duplicatedCount)


def throughputGFLOPS(dimensions, latency: float, duplicatedCount: int = 1) -> float:
    return operationsCount(dimensions, duplicatedCount) / latency / 1e9 if latency > 0 else 0.0


def permutationBytesCount(dimensions: Conv3DDimensions, duplicatedCount: int = 1) -> int:
    """Bytes a weight permutation reads and writes (:5362-5368)."""
    d = dimensions
    return 2 * d.kernelDepth * d.kernelHeight * d.kernelWidth * d.inputChannels * d.outputChannels * 2 * \
        duplicatedCount


def bandwidthGBPS(dimensions: Conv3DDimensions, latency: float, duplicatedCount: int = 1) -> float:
    return permutationBytesCount(dimensions, duplicatedCount) / latency / 1e9 if latency > 0 else 0.0


# ---------------------------------------------------------------------------
# formula data and the fp32 expectation
# ---------------------------------------------------------------------------

def createActivationData(dimensions) -> np.ndarray:
    d = dimensions
    if isinstance(d, Conv3DDimensions):
        return data.conv3d_activation(d.batchSize, d.inputDepth, d.inputHeight, d.inputWidth, d.inputChannels)
    return data.conv2d_activation(d.batchSize, d.inputHeight, d.inputWidth, d.inputChannels, d.outputChannels,
                                  d.kernelHeight, d.kernelWidth)


def createWeightData(dimensions, layout: int | None = None) -> np.ndarray:
    """HWIO (2-D) / DHWIO (3-D) by default; WEIGHTS_OIDHW stores the same values transposed, as the
    reference does (values from the DHWIO index, :4957-4983)."""
    d = dimensions
    if isinstance(d, Conv3DDimensions):
        w = data.conv3d_weights_dhwio(d.inputChannels, d.outputChannels, d.kernelDepth, d.kernelHeight,
                                      d.kernelWidth)
        if layout == WEIGHTS_OIDHW:
            return np.ascontiguousarray(w.transpose(4, 3, 0, 1, 2))
        return w
    return data.conv2d_weights_hwio(d.inputChannels, d.outputChannels, d.kernelHeight, d.kernelWidth)


def createBiasData(dimensions) -> np.ndarray:
    return data.conv3d_bias(dimensions.outputChannels)


def _torch_conv(dims, x, w_hwio, bias, device, dtype):
    """conv of NHWC / NDHWC x with HWIO / DHWIO weights through torch, returned NHWO / NDHWO."""
    import torch
    import torch.nn.functional as F
    d = dims
    three = isinstance(d, Conv3DDimensions)
    xt = torch.as_tensor(np.ascontiguousarray(x)).to(device=device, dtype=dtype)
    wt = torch.as_tensor(np.ascontiguousarray(w_hwio)).to(device=device, dtype=dtype)
    if three:
        xt = xt.permute(0, 4, 1, 2, 3)
        wt = wt.permute(4, 3, 0, 1, 2)
        xt = F.pad(xt, (d.paddingLeft, d.paddingRight, d.paddingTop, d.paddingBottom, d.paddingFront,
                        d.paddingBack))
        conv, stride, dil = F.conv3d, (d.strideZ, d.strideY, d.strideX), (d.dilationZ, d.dilationY, d.dilationX)
        mf = torch.channels_last_3d
    else:
        xt = xt.permute(0, 3, 1, 2)
        wt = wt.permute(3, 2, 0, 1)
        xt = F.pad(xt, (d.paddingLeft, d.paddingRight, d.paddingTop, d.paddingBottom))
        conv, stride, dil = F.conv2d, (d.strideY, d.strideX), (d.dilationY, d.dilationX)
        mf = torch.channels_last
    xt = xt.contiguous(memory_format=mf)
    wt = wt.contiguous(memory_format=mf)
    bt = None if bias is None else torch.as_tensor(np.ascontiguousarray(bias)).to(device=device, dtype=dtype)
    return lambda: conv(xt, wt, bt, stride=stride, dilation=dil), three


def referenceConvolution(dimensions, activation, weights, bias=None) -> np.ndarray:
    """fp32 expectation of the conv of the fp16 inputs (referenceConvolution / WithBias, :4994-5096),
    weights HWIO / DHWIO, output NHWO / NDHWO."""
    import torch
    with torch.no_grad():
        fn, three = _torch_conv(dimensions, activation, weights, bias, "cpu", torch.float32)
        y = fn()
        y = y.permute(0, 2, 3, 4, 1) if three else y.permute(0, 2, 3, 1)
        return y.contiguous().numpy()


# ---------------------------------------------------------------------------
# sessions (the reference's run(duplicatedCount:) -> ExecutionResult)
# ---------------------------------------------------------------------------

@dataclass
class ExecutionResult:
    output: np.ndarray | None
    wallLatency: float | None  # seconds
    gpuLatency: float | None   # seconds


def _device_name() -> str:
    import torch
    return torch.cuda.get_device_name(torch.cuda.current_device())


def _timed(launch: Callable[[int], None], duplicatedCount: int, readback) -> ExecutionResult:
    import torch

    from ._lib import sync_check
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    start.record()
    launch(duplicatedCount)
    end.record()
    out = readback() if readback is not None else None
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    sync_check()
    return ExecutionResult(out, wall, start.elapsed_time(end) / 1e3)


class _TensorOpSession:
    """The mm4 conv on the GPU, standing where the reference's TensorOpSession / TensorOpSession3D /
    TensorOpBiasSession3D / TensorOpHorizontalPaddingSession3D stand (:844-1575)."""

    def __init__(self, dimensions, activation, weights, bias=None, weight_layout=None,
                 buildOptions: BuildOptions | None = None):
        import torch
        dev = torch.device("cuda", torch.cuda.current_device())
        self.buildOptions = buildOptions
        self.plan = ConvPlan(dimensions, weight_layout=weight_layout, bias=bias is not None)
        self.x = torch.from_numpy(np.ascontiguousarray(activation)).to(dev)
        self.w = torch.from_numpy(np.ascontiguousarray(weights)).to(dev)
        self.b = None if bias is None else torch.from_numpy(np.ascontiguousarray(bias)).to(dev)
        self.y = torch.empty(self.plan.out_shape, dtype=torch.float16, device=dev)

    def dispatch_grid(self) -> DispatchGridSize:
        w, h, d = self.plan.tile_grid()
        return DispatchGridSize(w, h, d)

    def _launch(self, duplicatedCount: int) -> None:
        self.plan.run(self.x, self.w, self.b, y=self.y, duplicatedCount=duplicatedCount)

    def run(self, duplicatedCount: int = 1) -> ExecutionResult:
        return _timed(self._launch, duplicatedCount, lambda: self.y.float().cpu().numpy())

    def runWithoutOutputReadback(self, duplicatedCount: int = 1) -> ExecutionResult:
        return _timed(self._launch, duplicatedCount, None)


class _LibrarySession:
    """torch's cuDNN convolution (fp16, channels-last) on the same GPU, standing where the reference's
    MPSGraphSession stands."""

    def __init__(self, dimensions, activation, weights_hwio, bias=None):
        import torch
        self.fn, self.three = _torch_conv(dimensions, activation, weights_hwio, bias,
                                          torch.device("cuda", torch.cuda.current_device()), torch.float16)
        self.y = None

    def _launch(self, duplicatedCount: int) -> None:
        import torch
        with torch.no_grad():
            for _ in range(duplicatedCount):
                self.y = self.fn()

    def _readback(self):
        y = self.y.permute(0, 2, 3, 4, 1) if self.three else self.y.permute(0, 2, 3, 1)
        return y.float().contiguous().cpu().numpy()

    def run(self, duplicatedCount: int = 1) -> ExecutionResult:
        r = _timed(self._launch, duplicatedCount, self._readback)
        return ExecutionResult(r.output, r.wallLatency, None)  # like MPSGraph: wall latency only


class _PermutationSession:
    """OIDHW -> DHWIO weight permutation on the GPU (WeightPermutationSession3D, :1577-1675)."""

    def __init__(self, dimensions: Conv3DDimensions, sourceWeightsOIDHW):
        import torch
        d = dimensions
        self.dims5 = (d.outputChannels, d.inputChannels, d.kernelDepth, d.kernelHeight, d.kernelWidth)
        self.src = torch.from_numpy(np.ascontiguousarray(sourceWeightsOIDHW)).to(
            torch.device("cuda", torch.cuda.current_device()))
        self.dst = torch.empty_like(self.src)

    def _launch(self, duplicatedCount: int) -> None:
        for _ in range(duplicatedCount):
            permute_weights(self.src, WEIGHTS_OIDHW, WEIGHTS_DHWIO, self.dims5, dst=self.dst)

    def run(self, duplicatedCount: int = 1) -> ExecutionResult:
        return _timed(self._launch, duplicatedCount, lambda: self.dst.float().cpu().numpy())

    def runWithoutOutputReadback(self, duplicatedCount: int = 1) -> ExecutionResult:
        return _timed(self._launch, duplicatedCount, None)


class _PermuteThenTensorOpSession:
    """Permutation then conv, one stream (PermuteThenTensorOpSession3D)."""

    def __init__(self, dimensions: Conv3DDimensions, activation, sourceWeightsOIDHW,
                 buildOptions: BuildOptions | None = None):
        self.perm = _PermutationSession(dimensions, sourceWeightsOIDHW)
        # the conv reads the permutation's output buffer in place
        self.conv = _TensorOpSession(dimensions, activation, np.zeros(sourceWeightsOIDHW.shape, np.float16),
                                     weight_layout=WEIGHTS_DHWIO, buildOptions=buildOptions)
        self.conv.w = self.perm.dst

    def _launch(self, duplicatedCount: int) -> None:
        for _ in range(duplicatedCount):
            self.perm._launch(1)
            self.conv._launch(1)

    def run(self, duplicatedCount: int = 1) -> ExecutionResult:
        return _timed(self._launch, duplicatedCount, lambda: self.conv.y.float().cpu().numpy())

    def runWithoutOutputReadback(self, duplicatedCount: int = 1) -> ExecutionResult:
        return _timed(self._launch, duplicatedCount, None)


def _ms(seconds):
    return None if seconds is None else seconds * 1e3


def _check_options(options: ProfileOptions) -> None:
    if options.warmupIterations < 0 or options.timedIterations <= 0 or options.duplicatedCount <= 0:
        raise ValueError("ProfileOptions need warmupIterations >= 0, timedIterations > 0, duplicatedCount > 0")


def _average(session, options: ProfileOptions, readback: bool = False):
    """Warm-up, then the mean wall / GPU latency (seconds) over the timed iterations."""
    run = session.run if readback else session.runWithoutOutputReadback
    for _ in range(options.warmupIterations):
        run(options.duplicatedCount)
    wall = gpu = 0.0
    for _ in range(options.timedIterations):
        r = run(options.duplicatedCount)
        wall += r.wallLatency or 0.0
        gpu += r.gpuLatency or 0.0
    return wall / options.timedIterations, gpu / options.timedIterations


# ---------------------------------------------------------------------------
# ConvolutionHarness (ConvolutionShared.swift:2134-3411)
# ---------------------------------------------------------------------------

class ConvolutionHarness:
    """The reference's harness entry points, same names and defaults."""

    # -- case lists and defaults ------------------------------------------------

    @staticmethod
    def defaultValidationCases() -> list[Conv2DDimensions]:
        """:2143-2211."""
        return [
            Conv2DDimensions(1, 5, 5, 1, 1, 3, 3, 1, 1, 1, 1),
            Conv2DDimensions(1, 5, 5, 4, 8, 3, 3, 1, 1, 1, 1),
            Conv2DDimensions(1, 6, 7, 3, 5, 3, 3, 1, 1, 1, 1),
            Conv2DDimensions(1, 7, 8, 3, 4, 3, 3, 2, 2, 1, 1),
            Conv2DDimensions(1, 9, 10, 2, 3, 3, 3, 1, 1, 2, 2),
        ]

    @staticmethod
    def defaultProfileDimensions() -> Conv2DDimensions:
        """:2213-2227."""
        return Conv2DDimensions(1, 128, 128, 32, 32, 3, 3, 1, 1, 1, 1)

    @staticmethod
    def largeMPSGraphProfileDimensions() -> Conv2DDimensions:
        """:2229-2243."""
        return Conv2DDimensions(1, 256, 256, 512, 512, 3, 3, 1, 1, 1, 1)

    @staticmethod
    def largeMPSGraphValidationDimensions() -> Conv2DDimensions:
        return ConvolutionHarness.defaultProfileDimensions()

    @staticmethod
    def largeMPSGraphProfileOptions() -> ProfileOptions:
        return ProfileOptions(warmupIterations=1, timedIterations=3, duplicatedCount=1)

    @staticmethod
    def defaultTensorOpConv3DValidationCases() -> list[Conv3DDimensions]:
        """:2693-2764."""
        return [
            Conv3DDimensions(1, 5, 5, 5, 1, 1, 3, 3, 3, 1, 1, 1, 1, 1, 1),
            Conv3DDimensions(1, 4, 5, 5, 4, 8, 3, 3, 3, 1, 1, 1, 1, 1, 1),
            Conv3DDimensions(2, 7, 6, 7, 3, 5, 3, 3, 3, 2, 1, 1, 1, 1, 1),
            Conv3DDimensions(1, 7, 7, 7, 2, 3, 3, 3, 3, 1, 1, 1, 2, 2, 2),
        ]

    @staticmethod
    def defaultTensorOpConv3DBuildOptions() -> BuildOptions:
        """:2766-2768."""
        return BuildOptions(executionSIMDGroups=4, outputTileWidth=8, outputTileHeight=8)

    @staticmethod
    def defaultTensorOpConv3DLeftRightPaddingValidationCases() -> list[Conv3DDimensions]:
        """:2770-2878 (padding 1 on all four H/W sides)."""
        return [
            Conv3DDimensions(1, 5, 5, 5, 1, 1, 3, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1),
            Conv3DDimensions(1, 4, 5, 5, 4, 8, 3, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1),
            Conv3DDimensions(2, 7, 6, 7, 3, 5, 3, 3, 3, 2, 1, 1, 1, 1, 1, 1, 1, 1, 1),
            Conv3DDimensions(1, 5, 17, 19, 8, 12, 3, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1),
            Conv3DDimensions(1, 4, 33, 35, 4, 8, 3, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1),
        ]

    @staticmethod
    def largeTensorOpConv3DProfileDimensions() -> Conv3DDimensions:
        """:2880-2898."""
        return Conv3DDimensions(1, 3, 256, 256, 512, 512, 3, 3, 3, 1, 1, 1, 1, 1, 1)

    @staticmethod
    def largeTensorOpConv3DProfileOptions() -> ProfileOptions:
        return ProfileOptions(warmupIterations=2, timedIterations=5, duplicatedCount=1)

    @staticmethod
    def defaultTensorOpConv3DPermutationValidationDimensions() -> Conv3DDimensions:
        return ConvolutionHarness.defaultTensorOpConv3DValidationCases()[1]

    # -- conv2d -------------------------------------------------------------------

    @staticmethod
    def validateCorrectness(buildOptions: BuildOptions | None = None,
                            log: Log = _quiet) -> ConvolutionValidationSuiteResult:
        """Every default case through the tensor-op path and the library path, each against the fp32
        expectation and against each other (:2383-2465)."""
        buildOptions = buildOptions or BuildOptions(executionSIMDGroups=1)
        cases, all_passed = [], True
        for dims in ConvolutionHarness.defaultValidationCases():
            x, w = createActivationData(dims), createWeightData(dims)
            expected = referenceConvolution(dims, x, w)
            tensor_op = _TensorOpSession(dims, x, w, weight_layout=WEIGHTS_HWIO, buildOptions=buildOptions).run(1)
            library = _LibrarySession(dims, x, w).run(1)
            t_val = validateOutput(tensor_op.output, expected, "Tensor op", log)
            l_val = validateOutput(library.output, expected, "cuDNN", log)
            agree = compareOutputs(tensor_op.output, library.output, "Tensor op", "cuDNN", log)
            cases.append(ConvolutionCaseResult(dims, t_val, l_val, agree, _ms(tensor_op.wallLatency),
                                               _ms(tensor_op.gpuLatency), _ms(library.wallLatency)))
            log(f"Validated {dims}")
            log(f"Tensor op max absolute error: {t_val.maxAbsoluteError}")
            log(f"Tensor op mismatches above tolerance: {t_val.mismatches}")
            log(f"Tensor op vs cuDNN max absolute diff: {agree.maxAbsoluteError}")
            if t_val.mismatches or l_val.mismatches or agree.mismatches:
                all_passed = False
        log("Convolution validation passed." if all_passed else "Convolution validation failed.")
        return ConvolutionValidationSuiteResult(_device_name(), all_passed, cases)

    @staticmethod
    def profile(dimensions: Conv2DDimensions | None = None, buildOptions: BuildOptions | None = None,
                options: ProfileOptions | None = None, log: Log = _quiet) -> ConvolutionProfileResult:
        """Validation at the profile shape, then timed runs of both backends (:2467-2570)."""
        dims = dimensions or ConvolutionHarness.defaultProfileDimensions()
        buildOptions = buildOptions or BuildOptions(executionSIMDGroups=1)
        options = options or ProfileOptions(warmupIterations=3, timedIterations=10)
        _check_options(options)
        x, w = createActivationData(dims), createWeightData(dims)
        expected = referenceConvolution(dims, x, w)
        tensor_op = _TensorOpSession(dims, x, w, weight_layout=WEIGHTS_HWIO, buildOptions=buildOptions)
        library = _LibrarySession(dims, x, w)
        t_ref, l_ref = tensor_op.run(1), library.run(1)
        t_val = validateOutput(t_ref.output, expected, "Tensor op", log)
        l_val = validateOutput(l_ref.output, expected, "cuDNN", log)
        agree = compareOutputs(t_ref.output, l_ref.output, "Tensor op", "cuDNN", log)
        t_wall, t_gpu = _average(tensor_op, options, readback=True)
        l_wall, _ = _average(library, options, readback=True)
        dup = options.duplicatedCount
        t_prof = BackendProfileResult(t_wall * 1e3, t_gpu * 1e3, throughputGFLOPS(dims, t_wall, dup))
        l_prof = BackendProfileResult(l_wall * 1e3, None, throughputGFLOPS(dims, l_wall, dup))
        log(f"Profiled {dims}")
        log(f"Tensor op average wall latency: {t_prof.averageWallLatencyMS:.6f} ms, average GPU latency: "
            f"{t_gpu * 1e3:.6f} ms, throughput: {t_prof.throughputGFLOPS:.3f} GFLOP/s")
        log(f"cuDNN average wall latency: {l_prof.averageWallLatencyMS:.6f} ms, throughput: "
            f"{l_prof.throughputGFLOPS:.3f} GFLOP/s")
        return ConvolutionProfileResult(dims, options, t_val, l_val, agree, t_prof, l_prof)

    @staticmethod
    def profileTensorOpOnly(dimensions: Conv2DDimensions | None = None, buildOptions: BuildOptions | None = None,
                            options: ProfileOptions | None = None, log: Log = _quiet) -> BackendProfileResult:
        """Timed tensor-op runs without output read-back (:2572-2638)."""
        dims = dimensions or ConvolutionHarness.defaultProfileDimensions()
        buildOptions = buildOptions or BuildOptions(executionSIMDGroups=1)
        options = options or ProfileOptions(warmupIterations=3, timedIterations=10)
        _check_options(options)
        session = _TensorOpSession(dims, createActivationData(dims), createWeightData(dims),
                                   weight_layout=WEIGHTS_HWIO, buildOptions=buildOptions)
        wall, gpu = _average(session, options)
        grid = session.dispatch_grid()
        log(f"Tensor-op only profile on {dims}")
        log(f"Dispatch tiles: {grid.width}x{grid.height}x{grid.depth}, kernel {session.plan.kernel_name}")
        log(f"Tensor op average wall latency: {wall * 1e3:.6f} ms, throughput: "
            f"{throughputGFLOPS(dims, wall, options.duplicatedCount):.3f} GFLOP/s")
        return BackendProfileResult(wall * 1e3, gpu * 1e3, throughputGFLOPS(dims, wall, options.duplicatedCount))

    @staticmethod
    def profileTensorOpTileCoverage(tileWidth: int, tileHeight: int, dimensions: Conv2DDimensions | None = None,
                                    buildOptions: BuildOptions | None = None, options: ProfileOptions | None = None,
                                    log: Log = _quiet) -> TensorOpTileProfileResult:
        """The tensor-op profile with output-tile hints, as one full-grid region (:2640-2691). mm4 keeps
        its own tiles; the region's dispatch grid is the plan's output-tile grid."""
        if tileWidth <= 0 or tileHeight <= 0:
            raise ValueError("tileWidth and tileHeight must be positive")
        dims = dimensions or ConvolutionHarness.largeMPSGraphProfileDimensions()
        base = buildOptions or BuildOptions(executionSIMDGroups=1)
        options = options or ProfileOptions(warmupIterations=1, timedIterations=1)
        tiled = BuildOptions(executionSIMDGroups=base.executionSIMDGroups, outputTileWidth=tileWidth,
                             outputTileHeight=tileHeight)
        grid = ConvPlan(dims, weight_layout=WEIGHTS_HWIO).tile_grid()
        log(f"Tensor-op tiled coverage profile on {dims}")
        prof = ConvolutionHarness.profileTensorOpOnly(dims, tiled, options, log)
        gpu_tp = None if prof.averageGPULatencyMS is None else throughputGFLOPS(
            dims, prof.averageGPULatencyMS / 1e3, options.duplicatedCount)
        region = TensorOpTileRegionProfileResult("full-grid", tiled, DispatchGridSize(*grid),
                                                 prof.averageWallLatencyMS, prof.averageGPULatencyMS)
        return TensorOpTileProfileResult(dims, tileWidth, tileHeight, options, [region], prof.averageWallLatencyMS,
                                         prof.averageGPULatencyMS, prof.throughputGFLOPS, gpu_tp)

    # -- conv3d -------------------------------------------------------------------

    @staticmethod
    def _validate3d(dimensionsList, buildOptions, log, label, with_bias) -> Convolution3DValidationSuiteResult:
        cases, all_passed = [], True
        for dims in dimensionsList:
            x, w = createActivationData(dims), createWeightData(dims)
            b = createBiasData(dims) if with_bias else None
            expected = referenceConvolution(dims, x, w, b)
            r = _TensorOpSession(dims, x, w, b, weight_layout=WEIGHTS_DHWIO, buildOptions=buildOptions).run(1)
            val = validateOutput(r.output, expected, label, log)
            all_passed = all_passed and val.mismatches == 0
            cases.append(Convolution3DCaseResult(dims, val, _ms(r.wallLatency), _ms(r.gpuLatency)))
        return Convolution3DValidationSuiteResult(_device_name(), all_passed, cases)

    @staticmethod
    def validateTensorOpConv3D(dimensionsList=None, buildOptions: BuildOptions | None = None,
                               log: Log = _quiet) -> Convolution3DValidationSuiteResult:
        """:2904-2959."""
        return ConvolutionHarness._validate3d(
            dimensionsList or ConvolutionHarness.defaultTensorOpConv3DValidationCases(),
            buildOptions or ConvolutionHarness.defaultTensorOpConv3DBuildOptions(), log, "Tensor-op Conv3D", False)

    @staticmethod
    def validateTensorOpConv3DLeftRightPadding(dimensionsList=None, buildOptions: BuildOptions | None = None,
                                               log: Log = _quiet) -> Convolution3DValidationSuiteResult:
        """:2960-3015."""
        return ConvolutionHarness._validate3d(
            dimensionsList or ConvolutionHarness.defaultTensorOpConv3DLeftRightPaddingValidationCases(),
            buildOptions or ConvolutionHarness.defaultTensorOpConv3DBuildOptions(), log,
            "Tensor-op Conv3D left/right padding", False)

    @staticmethod
    def validateTensorOpConv3DBias(dimensionsList=None, buildOptions: BuildOptions | None = None,
                                   log: Log = _quiet) -> Convolution3DValidationSuiteResult:
        """:3016-3077."""
        return ConvolutionHarness._validate3d(
            dimensionsList or ConvolutionHarness.defaultTensorOpConv3DValidationCases(),
            buildOptions or ConvolutionHarness.defaultTensorOpConv3DBuildOptions(), log, "Tensor-op Conv3D Bias",
            True)

    @staticmethod
    def _profile3d(dims, buildOptions, options, log, with_bias) -> TensorOpConv3DProfileResult:
        dims = dims or ConvolutionHarness.largeTensorOpConv3DProfileDimensions()
        buildOptions = buildOptions or ConvolutionHarness.defaultTensorOpConv3DBuildOptions()
        options = options or ConvolutionHarness.largeTensorOpConv3DProfileOptions()
        _check_options(options)
        session = _TensorOpSession(dims, createActivationData(dims), createWeightData(dims),
                                   createBiasData(dims) if with_bias else None, weight_layout=WEIGHTS_DHWIO,
                                   buildOptions=buildOptions)
        wall, gpu = _average(session, options)
        dup = options.duplicatedCount
        log(f"Conv3D tensor op ({session.plan.kernel_name}) average wall latency: {wall * 1e3:.6f} ms, "
            f"GPU latency: {gpu * 1e3:.6f} ms, throughput: {throughputGFLOPS(dims, gpu, dup):.3f} GFLOP/s")
        return TensorOpConv3DProfileResult(dims, buildOptions, options, session.dispatch_grid(), wall * 1e3,
                                           gpu * 1e3, throughputGFLOPS(dims, wall, dup),
                                           throughputGFLOPS(dims, gpu, dup))

    @staticmethod
    def profileTensorOpConv3D(dimensions: Conv3DDimensions | None = None, buildOptions: BuildOptions | None = None,
                              options: ProfileOptions | None = None, log: Log = _quiet) -> TensorOpConv3DProfileResult:
        """:3079-3161."""
        return ConvolutionHarness._profile3d(dimensions, buildOptions, options, log, False)

    @staticmethod
    def profileTensorOpConv3DBias(dimensions: Conv3DDimensions | None = None, buildOptions: BuildOptions | None = None,
                                  options: ProfileOptions | None = None,
                                  log: Log = _quiet) -> TensorOpConv3DProfileResult:
        """:3163-3247."""
        return ConvolutionHarness._profile3d(dimensions, buildOptions, options, log, True)

    @staticmethod
    def profileTensorOpConv3DWithPermutation(validationDimensions: Conv3DDimensions | None = None,
                                             profileDimensions: Conv3DDimensions | None = None,
                                             buildOptions: BuildOptions | None = None,
                                             options: ProfileOptions | None = None,
                                             log: Log = _quiet) -> TensorOpConv3DPermutationProfileResult:
        """OIDHW -> DHWIO permutation alone and followed by the conv: validated on a small shape,
        timed on the profile shape (:3253-3408)."""
        vdims = validationDimensions or ConvolutionHarness.defaultTensorOpConv3DPermutationValidationDimensions()
        pdims = profileDimensions or ConvolutionHarness.largeTensorOpConv3DProfileDimensions()
        buildOptions = buildOptions or ConvolutionHarness.defaultTensorOpConv3DBuildOptions()
        options = options or ConvolutionHarness.largeTensorOpConv3DProfileOptions()
        _check_options(options)
        w_oidhw = createWeightData(vdims, WEIGHTS_OIDHW)
        w_dhwio = createWeightData(vdims)
        x = createActivationData(vdims)
        expected = referenceConvolution(vdims, x, w_dhwio)
        perm = _PermutationSession(vdims, w_oidhw).run(1)
        perm_val = validateFlatOutput(perm.output, w_dhwio, "OIDHW->DHWIO permutation", log)
        combined = _PermuteThenTensorOpSession(vdims, x, w_oidhw, buildOptions).run(1)
        comb_val = validateOutput(combined.output, expected, "Permute+Tensor-op Conv3D", log)

        perm_s = _PermutationSession(pdims, createWeightData(pdims, WEIGHTS_OIDHW))
        comb_s = _PermuteThenTensorOpSession(pdims, createActivationData(pdims),
                                             createWeightData(pdims, WEIGHTS_OIDHW), buildOptions)
        p_wall, p_gpu = _average(perm_s, options)
        c_wall, c_gpu = _average(comb_s, options)
        dup = options.duplicatedCount
        log(f"Permutation average GPU latency: {p_gpu * 1e3:.6f} ms, bandwidth: "
            f"{bandwidthGBPS(pdims, p_gpu, dup):.3f} GB/s")
        log(f"Permute+Conv3D average GPU latency: {c_gpu * 1e3:.6f} ms, throughput: "
            f"{throughputGFLOPS(pdims, c_gpu, dup):.3f} GFLOP/s")
        return TensorOpConv3DPermutationProfileResult(
            vdims, pdims, buildOptions, options, perm_val, comb_val, p_wall * 1e3, p_gpu * 1e3,
            bandwidthGBPS(pdims, p_wall, dup), bandwidthGBPS(pdims, p_gpu, dup), c_wall * 1e3, c_gpu * 1e3,
            throughputGFLOPS(pdims, c_wall, dup), throughputGFLOPS(pdims, c_gpu, dup))
