"""ConvolutionHarness on the CPU: report keys as the reference's Codable structs
write them (ConvolutionShared.swift:187-622), the validators' rules
(:5174-5405), the fp32 expectation against the C oracle on every harness case
list, and every entry point's flow with host stand-ins for the GPU sessions."""
import json
import types

import numpy as np
import pytest

import oracle
from cases import oracle_kwargs2d, oracle_kwargs3d
from example_matmul_metal4_b200 import harness
from example_matmul_metal4_b200.conv import WEIGHTS_OIDHW, BuildOptions, Conv2DDimensions, Conv3DDimensions
from example_matmul_metal4_b200.harness import ConvolutionHarness as H

# Stored properties of the reference structs, in declaration order.
REFERENCE_KEYS = {
    harness.ValidationResult: ["maxAbsoluteError", "mismatches"],
    harness.ConvolutionCaseResult: ["dimensions", "tensorOpValidation", "mpsGraphValidation", "backendAgreement",
                                    "tensorOpWallLatencyMS", "tensorOpGPULatencyMS", "mpsGraphWallLatencyMS"],
    harness.ConvolutionValidationSuiteResult: ["deviceName", "allPassed", "cases"],
    harness.ProfileOptions: ["warmupIterations", "timedIterations", "duplicatedCount"],
    harness.BackendProfileResult: ["averageWallLatencyMS", "averageGPULatencyMS", "throughputGFLOPS"],
    harness.DispatchGridSize: ["width", "height", "depth"],
    harness.TensorOpTileRegionProfileResult: ["label", "buildOptions", "dispatchGrid", "averageWallLatencyMS",
                                              "averageGPULatencyMS"],
    harness.TensorOpTileProfileResult: ["dimensions", "tileWidth", "tileHeight", "options", "regions",
                                        "averageWallLatencyMS", "averageGPULatencyMS", "wallThroughputGFLOPS",
                                        "gpuThroughputGFLOPS"],
    harness.Convolution3DCaseResult: ["dimensions", "tensorOpValidation", "tensorOpWallLatencyMS",
                                      "tensorOpGPULatencyMS"],
    harness.Convolution3DValidationSuiteResult: ["deviceName", "allPassed", "cases"],
    harness.TensorOpConv3DProfileResult: ["dimensions", "buildOptions", "options", "dispatchGrid",
                                          "averageWallLatencyMS", "averageGPULatencyMS", "wallThroughputGFLOPS",
                                          "gpuThroughputGFLOPS"],
    harness.TensorOpConv3DPermutationProfileResult: [
        "validationDimensions", "profileDimensions", "buildOptions", "options", "permutationValidation",
        "combinedValidation", "permutationAverageWallLatencyMS", "permutationAverageGPULatencyMS",
        "permutationWallBandwidthGBPS", "permutationGPUBandwidthGBPS", "combinedAverageWallLatencyMS",
        "combinedAverageGPULatencyMS", "combinedWallThroughputGFLOPS", "combinedGPUThroughputGFLOPS"],
    harness.ConvolutionProfileResult: ["dimensions", "options", "tensorOpValidation", "mpsGraphValidation",
                                       "backendAgreement", "tensorOp", "mpsGraph"],
    BuildOptions: ["executionSIMDGroups", "outputTileWidth", "outputTileHeight", "outputBaseX", "outputBaseY",
                   "dispatchGridWidth", "dispatchGridHeight"],
}
CONV2D_KEYS = ["batchSize", "inputHeight", "inputWidth", "inputChannels", "outputChannels", "kernelHeight",
               "kernelWidth", "strideY", "strideX", "dilationY", "dilationX", "paddingTop", "paddingBottom",
               "paddingLeft", "paddingRight"]


def test_report_fields_are_the_reference_fields():
    from dataclasses import fields
    for cls, keys in REFERENCE_KEYS.items():
        assert [f.name for f in fields(cls)] == keys, cls.__name__
    assert [f.name for f in fields(Conv2DDimensions)] == CONV2D_KEYS


def test_json_leaves_out_nil_optionals_and_nests_dimensions():
    v = harness.ValidationResult(0.5, 2)
    r = harness.Convolution3DCaseResult(H.defaultTensorOpConv3DValidationCases()[0], v, None, 1.25)
    d = json.loads(r.to_json())
    assert set(d) == {"dimensions", "tensorOpValidation", "tensorOpGPULatencyMS"}
    assert d["tensorOpValidation"] == {"maxAbsoluteError": 0.5, "mismatches": 2}
    assert d["dimensions"]["inputDepth"] == 5 and d["dimensions"]["kernelDepth"] == 3
    assert harness._encode(BuildOptions(executionSIMDGroups=4)) == {"executionSIMDGroups": 4}


def test_validators_follow_the_reference_rules():
    exp = np.zeros((1, 2, 2, 3), np.float32)
    act = exp.copy()
    act[0, 1, 0, 2] = 0.021   # above the absolute 2e-2
    act[0, 0, 1, 1] = -0.019  # within
    logs = []
    v = harness.validateOutput(act, exp, "x", logs.append)
    assert v.mismatches == 1 and abs(v.maxAbsoluteError - 0.021) < 1e-7
    assert logs == ["x mismatch at n=0, h=1, w=0, o=2: expected 0.0, got 0.020999999716877937"]
    big = np.full((1, 1, 1, 1), 1000.0, np.float32)
    assert harness.validateOutput(big + 0.03, big).mismatches == 1  # absolute, not relative
    assert harness.compareOutputs(act, exp).mismatches == 1
    w = np.arange(12, dtype=np.float16)
    assert harness.validateFlatOutput(w.astype(np.float32), w).mismatches == 0
    w2 = w.astype(np.float32)
    w2[5] += 2 ** -10
    assert harness.validateFlatOutput(w2, w).mismatches == 1  # exact match required


def test_work_accounting():
    d2 = Conv2DDimensions(2, 9, 10, 3, 4, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1)
    assert harness.operationsCount(d2, 3) == 2 * 2 * 9 * 10 * 4 * 3 * 3 * 3 * 3
    assert harness.throughputGFLOPS(d2, 0.0) == 0.0
    d3 = H.largeTensorOpConv3DProfileDimensions()
    assert harness.operationsCount(d3) == 2 * 1 * 1 * 254 * 254 * 512 * 27 * 512
    assert harness.permutationBytesCount(d3, 2) == 2 * 27 * 512 * 512 * 2 * 2
    assert harness.bandwidthGBPS(d3, 1e-3) == harness.permutationBytesCount(d3) / 1e-3 / 1e9


def test_case_lists_and_defaults():
    assert len(H.defaultValidationCases()) == 5 and H.defaultValidationCases()[3].strideX == 2
    assert H.defaultValidationCases()[4].dilationX == 2
    assert H.defaultTensorOpConv3DBuildOptions() == BuildOptions(4, 8, 8)
    assert [c.paddingLeft for c in H.defaultTensorOpConv3DLeftRightPaddingValidationCases()] == [1] * 5
    assert H.defaultTensorOpConv3DPermutationValidationDimensions() == H.defaultTensorOpConv3DValidationCases()[1]
    assert H.largeMPSGraphProfileOptions() == harness.ProfileOptions(1, 3, 1)
    assert H.largeTensorOpConv3DProfileOptions() == harness.ProfileOptions(2, 5, 1)


def test_oidhw_weights_are_the_dhwio_values_transposed():
    d = H.defaultTensorOpConv3DValidationCases()[1]
    w = harness.createWeightData(d)
    wo = harness.createWeightData(d, WEIGHTS_OIDHW)
    assert wo.shape == (8, 4, 3, 3, 3)
    assert np.array_equal(wo, w.transpose(4, 3, 0, 1, 2))


@pytest.mark.parametrize("which", ["2d", "3d", "3d_padded", "3d_bias"])
def test_expectation_matches_the_oracle(which):
    if which == "2d":
        for d in H.defaultValidationCases() + [Conv2DDimensions(1, 17, 19, 8, 12, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1)]:
            x, w = harness.createActivationData(d), harness.createWeightData(d)
            ref = oracle.conv2d(x, w, None, layout=0, **oracle_kwargs2d(d))
            np.testing.assert_allclose(harness.referenceConvolution(d, x, w), ref.reshape(
                d.batchSize, d.outputHeight, d.outputWidth, d.outputChannels), rtol=1e-5, atol=1e-5)
        return
    cases = (H.defaultTensorOpConv3DLeftRightPaddingValidationCases() if which == "3d_padded"
             else H.defaultTensorOpConv3DValidationCases())
    for d in cases:
        x, w = harness.createActivationData(d), harness.createWeightData(d)
        b = harness.createBiasData(d) if which == "3d_bias" else None
        ref = oracle.conv3d(x, w, b, layout=3, **oracle_kwargs3d(d))
        got = harness.referenceConvolution(d, x, w, b)
        np.testing.assert_allclose(got.reshape(-1), ref.reshape(-1), rtol=1e-5, atol=1e-5)


# ---------------------------------------------------------------------------
# entry-point flow with host stand-ins for the GPU sessions
# ---------------------------------------------------------------------------

def _fp16(a):
    return a.astype(np.float16).astype(np.float32)


class _HostTensorOp:
    def __init__(self, dims, x, w, bias=None, weight_layout=None, buildOptions=None):
        self.dims, self.x, self.w, self.b = dims, x, w, bias
        self.plan = types.SimpleNamespace(kernel_name="host stand-in", tile_grid=lambda: (3, 1, 1))

    def dispatch_grid(self):
        return harness.DispatchGridSize(3, 1, 1)

    def run(self, duplicatedCount=1):
        return harness.ExecutionResult(_fp16(harness.referenceConvolution(self.dims, self.x, self.w, self.b)),
                                       2e-3, 1e-3)

    def runWithoutOutputReadback(self, duplicatedCount=1):
        return harness.ExecutionResult(None, 2e-3, 1e-3)


class _HostLibrary(_HostTensorOp):
    def __init__(self, dims, x, w, bias=None):
        super().__init__(dims, x, w, bias)

    def run(self, duplicatedCount=1):
        r = super().run(duplicatedCount)
        return harness.ExecutionResult(r.output, 4e-3, None)


class _HostPermutation:
    def __init__(self, dims, w_oidhw):
        self.w = w_oidhw

    def run(self, duplicatedCount=1):
        return harness.ExecutionResult(self.w.transpose(2, 3, 4, 1, 0).astype(np.float32), 1e-4, 5e-5)

    def runWithoutOutputReadback(self, duplicatedCount=1):
        return harness.ExecutionResult(None, 1e-4, 5e-5)


class _HostPermuteThenConv(_HostTensorOp):
    def __init__(self, dims, x, w_oidhw, buildOptions=None):
        super().__init__(dims, x, np.ascontiguousarray(w_oidhw.transpose(2, 3, 4, 1, 0)))


@pytest.fixture
def host_sessions(monkeypatch):
    monkeypatch.setattr(harness, "_TensorOpSession", _HostTensorOp)
    monkeypatch.setattr(harness, "_LibrarySession", _HostLibrary)
    monkeypatch.setattr(harness, "_PermutationSession", _HostPermutation)
    monkeypatch.setattr(harness, "_PermuteThenTensorOpSession", _HostPermuteThenConv)
    monkeypatch.setattr(harness, "_device_name", lambda: "host")
    monkeypatch.setattr(harness, "ConvPlan", lambda dims, weight_layout=None: types.SimpleNamespace(
        tile_grid=lambda: (7, 2, 1)))


def test_conv2d_entry_points(host_sessions):
    logs = []
    suite = H.validateCorrectness(log=logs.append)
    assert suite.allPassed and suite.deviceName == "host" and len(suite.cases) == 5
    case = suite.cases[0].to_dict()
    assert case["tensorOpWallLatencyMS"] == pytest.approx(2.0) and case["tensorOpGPULatencyMS"] == pytest.approx(1.0)
    assert case["mpsGraphWallLatencyMS"] == pytest.approx(4.0) and case["backendAgreement"]["mismatches"] == 0
    assert logs[-1] == "Convolution validation passed."
    small = Conv2DDimensions(1, 16, 16, 8, 8, 3, 3, 1, 1, 1, 1)
    opts = harness.ProfileOptions(1, 2)
    prof = H.profile(small, options=opts)
    assert prof.tensorOpValidation.mismatches == 0 and prof.mpsGraph.averageGPULatencyMS is None
    assert prof.tensorOp.throughputGFLOPS == pytest.approx(harness.throughputGFLOPS(small, 2e-3))
    assert "averageGPULatencyMS" not in prof.to_dict()["mpsGraph"]
    only = H.profileTensorOpOnly(small, options=opts)
    assert only.averageGPULatencyMS == pytest.approx(1.0)
    tiles = H.profileTensorOpTileCoverage(tileWidth=8, tileHeight=4, dimensions=small, options=opts)
    d = tiles.to_dict()
    assert d["regions"][0]["label"] == "full-grid" and d["regions"][0]["dispatchGrid"] == {
        "width": 7, "height": 2, "depth": 1}
    assert d["regions"][0]["buildOptions"] == {"executionSIMDGroups": 1, "outputTileWidth": 8, "outputTileHeight": 4}
    with pytest.raises(ValueError):
        H.profile(small, options=harness.ProfileOptions(0, 0))


def test_conv3d_entry_points(host_sessions):
    for fn in (H.validateTensorOpConv3D, H.validateTensorOpConv3DLeftRightPadding, H.validateTensorOpConv3DBias):
        suite = fn()
        assert suite.allPassed and all(c.tensorOpValidation.mismatches == 0 for c in suite.cases)
    small = Conv3DDimensions(1, 3, 8, 8, 16, 16, 3, 3, 3, 1, 1, 1, 1, 1, 1)
    opts = harness.ProfileOptions(1, 2)
    p = H.profileTensorOpConv3DBias(small, options=opts)
    assert p.dispatchGrid == harness.DispatchGridSize(3, 1, 1)
    assert p.gpuThroughputGFLOPS == pytest.approx(harness.throughputGFLOPS(small, 1e-3))
    perm = H.profileTensorOpConv3DWithPermutation(profileDimensions=small, options=opts)
    assert perm.permutationValidation.mismatches == 0 and perm.combinedValidation.mismatches == 0
    assert perm.permutationGPUBandwidthGBPS == pytest.approx(harness.bandwidthGBPS(small, 5e-5))
    assert json.loads(perm.to_json())["buildOptions"] == {"executionSIMDGroups": 4, "outputTileWidth": 8,
                                                          "outputTileHeight": 8}


def test_tile_grid_matches_kernel_units():
    """The plan's output-tile grid is the unit count the CTA-pair kernels walk on the BASELINE conv
    shapes (256 virtual pixels per unit, rows OW + 2 wide) -- host-only, no launch."""
    from example_matmul_metal4_b200.conv import ConvPlan
    assert ConvPlan(Conv2DDimensions(32, 56, 56, 256, 256, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1)).tile_grid() == (406, 1, 1)
    assert ConvPlan(Conv3DDimensions(8, 16, 64, 64, 128, 128, 3, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1)
                    ).tile_grid() == (2112, 1, 1)
    # one-CTA gather path (stride 2): 128-pixel tiles over the real output rows
    d = Conv2DDimensions(1, 7, 8, 3, 4, 3, 3, 2, 2, 1, 1)
    assert ConvPlan(d).tile_grid() == (1, 1, 1)


def test_driver_check_reports_like_the_reference():
    from example_matmul_metal4_b200.gemm import _check
    exp = np.zeros((2, 3), np.float32)
    got = exp.copy()
    got[1, 2] = 0.006
    got[0, 0] = 0.004
    logs = []
    worst, bad = _check(exp, got, "C", 5e-3, logs.append)
    assert bad == 1 and abs(worst - 0.006) < 1e-7
    assert logs == ["CPU calculated C[1, 2]: 0.0", "GPU calculated C[1, 2]: 0.006000000052154064"]
