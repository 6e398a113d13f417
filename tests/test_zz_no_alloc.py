"""The allocation-free split-K entry point, mm4_gemm_splitk_run_noalloc.

It exists for callers that cannot call cudaMalloc where they issue the GEMM
(an allocator that owns all GPU memory, serving loops where an allocation
may stall or fail, plug-in hosts that only pass their own buffers): its
partial-sum scratch is a static 4 MiB device array inside libmm4.so.

The test calls it through the C ABI twice in a row, on different inputs, and
checks each result against the existing entry point (mm4_gemm_run with a
caller workspace) on the same inputs, within the parity tolerance. It lives
in its own file, collected last, and passes both alone in a fresh process
and after the other tests.
"""

import pytest

from example_matmul_metal4_b200 import BuildOptions, GEMMDimensions, GemmPlan, data, lib, sync_check
from example_matmul_metal4_b200._lib import MM4_ERR_INVALID, MM4_ERR_WORKSPACE, check, stream_handle
from tolerance import assert_close

pytestmark = pytest.mark.gpu


def _noalloc(plan, A, B, bias, C):
    check(lib().mm4_gemm_splitk_run_noalloc(plan.handle, A.data_ptr(), B.data_ptr(), bias.data_ptr(), C.data_ptr(),
                                             stream_handle()))


@pytest.mark.parametrize("M,N,K,split,tr", [(512, 512, 65536, 32, False), (384, 640, 8192, 8, True)])
def test_noalloc_matches_existing_entry_point_twice(cuda, M, N, K, split, tr):
    import torch
    plan = GemmPlan(GEMMDimensions(M, N, K), transpose=(False, tr), bias=True, buildOptions=BuildOptions(splitK=split))
    assert plan.workspace_bytes <= 4 << 20
    b_shape = (N, K) if tr else (K, N)
    for call, seed in enumerate((21, 22)):
        A = torch.from_numpy(data.uniform((M, K), -1.0, 1.0, seed, 0)).to(cuda)
        B = torch.from_numpy(data.uniform(b_shape, -1.0, 1.0, seed, 1)).to(cuda)
        bias = torch.from_numpy(data.uniform((N,), -1.0, 1.0, seed, 2)).to(cuda)
        C_noalloc = torch.full((M, N), float("nan"), dtype=torch.float16, device=cuda)
        _noalloc(plan, A, B, bias, C_noalloc)
        C_ref = plan.run(A, B, bias)
        sync_check()
        assert_close(C_noalloc.float().cpu().numpy(), C_ref.float().cpu().numpy(), f"no-alloc call {call + 1}")


def test_noalloc_rejects_oversized_and_non_splitk_plans(cuda):
    import torch
    big = GemmPlan(GEMMDimensions(2048, 1024, 4096), transpose=(False, False), bias=True,
                   buildOptions=BuildOptions(splitK=4))
    assert big.workspace_bytes > 4 << 20
    x = torch.zeros(16, dtype=torch.float16, device=cuda)
    rc = lib().mm4_gemm_splitk_run_noalloc(big.handle, x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(),
                                           stream_handle())
    assert rc == MM4_ERR_WORKSPACE
    assert b"4 MiB" in lib().mm4_last_error()
    direct = GemmPlan(GEMMDimensions(128, 128, 128), transpose=(False, False), bias=True)
    rc = lib().mm4_gemm_splitk_run_noalloc(direct.handle, x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(),
                                           stream_handle())
    assert rc == MM4_ERR_INVALID
