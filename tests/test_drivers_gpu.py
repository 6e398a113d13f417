"""The reference executables' run(...) drivers on the GPU: its matmul main
shape (matmul.swift:334: 32x3072x80000, B stored [N][K], splitK 30) and points
of its attention sweep (attention.swift:390-395), each element within the
drivers' 5e-3 of the fp32 expectation."""
import pytest

from example_matmul_metal4_b200 import attention, gemm

pytestmark = pytest.mark.gpu


def test_matmul_main_shape(cuda):
    r = gemm.run(32, 3072, 80000, gemm.GEMMDimensions(128, 64, 64), gemm.BuildOptions(4, 1, True, 30), 1,
                 log=lambda s: None)
    assert r.mismatches == 0, r
    assert r.gflops > 0 and "splitk" in r.kernel


@pytest.mark.parametrize("S", [1, 64, 300])
def test_attention_sweep_points(cuda, S):
    r = attention.run(S, 128, 8, 8, attention.BuildOptions(16, True), 1, log=lambda s: None)
    assert r.mismatches == 0, r


def test_matmul_profile_correctness_sample(cuda):
    """Points of the reference's M = N = K sweep (matmul.swift:337-342), its block hints and options:
    both sides of every power of two up to 512, through the reduced-alignment and tensor-core kernels."""
    sizes = sorted({1, 2, 3} | {v for p in range(3, 10) for v in (2 ** p - 1, 2 ** p, 2 ** p + 1)})
    results = gemm.profileCorrectness(sizes=sizes, log=lambda s: None)
    bad = {n: r for n, r in zip(sizes, results) if r.mismatches}
    assert not bad, bad
