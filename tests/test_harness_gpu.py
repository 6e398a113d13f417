"""ConvolutionHarness on the GPU: the reference's validation suites pass on
the mm4 path and on the cuDNN comparator, and the profile entry points return
well-formed reports (small profile shapes and iteration counts)."""
import pytest

from example_matmul_metal4_b200 import harness
from example_matmul_metal4_b200.conv import Conv3DDimensions
from example_matmul_metal4_b200.harness import ConvolutionHarness as H

pytestmark = pytest.mark.gpu

OPTS = harness.ProfileOptions(warmupIterations=1, timedIterations=2)


def test_validate_correctness(cuda):
    suite = H.validateCorrectness()
    assert suite.allPassed, suite.to_json()
    assert len(suite.cases) == 5 and suite.deviceName


@pytest.mark.parametrize("entry", ["validateTensorOpConv3D", "validateTensorOpConv3DLeftRightPadding",
                                   "validateTensorOpConv3DBias"])
def test_conv3d_validation_suites(cuda, entry):
    suite = getattr(H, entry)()
    assert suite.allPassed, suite.to_json()


def test_profile_reports(cuda):
    p = H.profile(options=OPTS)
    assert p.tensorOpValidation.mismatches == 0 and p.backendAgreement.mismatches == 0, p.to_json()
    assert p.tensorOp.throughputGFLOPS > 0 and p.tensorOp.averageGPULatencyMS > 0
    t = H.profileTensorOpTileCoverage(tileWidth=8, tileHeight=8, dimensions=H.defaultProfileDimensions(),
                                      options=OPTS)
    assert t.regions[0].dispatchGrid.width >= 1 and t.wallThroughputGFLOPS > 0


def test_conv3d_profiles(cuda):
    small = Conv3DDimensions(1, 3, 32, 32, 64, 64, 3, 3, 3, 1, 1, 1, 1, 1, 1)
    p = H.profileTensorOpConv3DBias(small, options=OPTS)
    assert p.gpuThroughputGFLOPS > 0 and p.dispatchGrid.width >= 1
    perm = H.profileTensorOpConv3DWithPermutation(profileDimensions=small, options=OPTS)
    assert perm.permutationValidation.mismatches == 0 and perm.combinedValidation.mismatches == 0, perm.to_json()
    assert perm.permutationGPUBandwidthGBPS > 0 and perm.combinedGPUThroughputGFLOPS > 0

