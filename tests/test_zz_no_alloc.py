"""The allocation-free split-K entry point, mm4_gemm_splitk_run_noalloc.

It exists for callers that cannot call cudaMalloc where they issue the GEMM
(an allocator that owns all GPU memory, serving loops where an allocation
may stall or fail, plug-in hosts that only pass their own buffers): its
partial-sum scratch is a static 4 MiB device array inside libmm4.so.

The tests call it through the C ABI twice in a row, on different inputs, and
check each result against the existing entry point (mm4_gemm_run with a
caller workspace) and against the oracle (the reference's CPU loop,
matmul.swift:499-510), within the parity tolerance. They also check that a
device-side wait that ran out is reported once by mm4_check and leaves the
next call correct. The file is collected last and passes both alone in a
fresh process and after the other tests.
"""

import pytest

import oracle
from example_matmul_metal4_b200 import BuildOptions, GEMMDimensions, GemmPlan, data, lib, sync_check
from example_matmul_metal4_b200._lib import (MM4_ERR_INVALID, MM4_ERR_TIMEOUT, MM4_ERR_WORKSPACE, check,
                                             stream_handle)
from tolerance import assert_close

pytestmark = pytest.mark.gpu


def _noalloc(plan, A, B, bias, C):
    check(lib().mm4_gemm_splitk_run_noalloc(plan.handle, A.data_ptr(), B.data_ptr(), bias.data_ptr(), C.data_ptr(),
                                             stream_handle()))


def _inputs(cuda, M, N, K, tr, seed):
    import torch
    hA = data.uniform((M, K), -1.0, 1.0, seed, 0)
    hB = data.uniform((N, K) if tr else (K, N), -1.0, 1.0, seed, 1)
    hb = data.uniform((N,), -1.0, 1.0, seed, 2)
    return (hA, hB, hb), tuple(torch.from_numpy(x).to(cuda) for x in (hA, hB, hb))


def _oracle_rows(host, M, N, K, tr, rows):
    hA, hB, hb = host
    return oracle.gemm(hA, hB, hb, M, N, K, False, tr, rows=rows, threads=oracle.default_threads())


@pytest.mark.parametrize("M,N,K,split,tr", [(512, 512, 65536, 32, False), (384, 640, 8192, 8, True)])
def test_noalloc_matches_existing_entry_point_twice(cuda, M, N, K, split, tr):
    import torch
    plan = GemmPlan(GEMMDimensions(M, N, K), transpose=(False, tr), bias=True, buildOptions=BuildOptions(splitK=split))
    assert plan.workspace_bytes <= 4 << 20
    for call, seed in enumerate((21, 22)):
        host, (A, B, bias) = _inputs(cuda, M, N, K, tr, seed)
        C_noalloc = torch.full((M, N), float("nan"), dtype=torch.float16, device=cuda)
        _noalloc(plan, A, B, bias, C_noalloc)
        C_ref = plan.run(A, B, bias)
        sync_check()
        got = C_noalloc.float().cpu().numpy()
        assert_close(got, C_ref.float().cpu().numpy(), f"no-alloc call {call + 1} vs mm4_gemm_run")
        # the oracle on a band of rows at each end (all rows for the smaller shape)
        bands = [(0, M)] if M * N * K <= 384 * 640 * 8192 else [(0, 16), (M - 16, M)]
        for r0, r1 in bands:
            assert_close(got[r0:r1], _oracle_rows(host, M, N, K, tr, (r0, r1)),
                         f"no-alloc call {call + 1} vs oracle rows {r0}-{r1}")


def test_noalloc_timeout_is_reported_once_and_later_calls_are_correct(cuda):
    """A run-out wait recorded in the no-alloc status word (the debug hook's one-warp wait on an mbarrier
    nothing arrives at) must not make later no-alloc calls abort: the next call's result is correct, and
    mm4_check reports the timeout exactly once."""
    import torch
    M, N, K, split = 256, 512, 16384, 16
    plan = GemmPlan(GEMMDimensions(M, N, K), transpose=(False, False), bias=True,
                    buildOptions=BuildOptions(splitK=split))
    L = lib()
    assert L.mm4_check(stream_handle()) == 0  # start clean
    # make sure the no-alloc words exist on this device, then record a timeout in them
    host, (A, B, bias) = _inputs(cuda, M, N, K, False, 31)
    C = torch.empty((M, N), dtype=torch.float16, device=cuda)
    _noalloc(plan, A, B, bias, C)
    assert L.mm4_debug_noalloc_wait_timeout(2_000_000, stream_handle()) == 0  # 2 ms
    for call in range(2):
        C.fill_(float("nan"))
        _noalloc(plan, A, B, bias, C)
        torch.cuda.synchronize()
        assert_close(C.float().cpu().numpy(), _oracle_rows(host, M, N, K, False, (0, M)),
                     f"no-alloc call {call + 1} after a recorded timeout")
        rc = L.mm4_check(stream_handle())
        if call == 0:
            assert rc == MM4_ERR_TIMEOUT, rc
            assert b"site 99" in L.mm4_last_error()
        else:
            assert rc == 0, L.mm4_last_error()
    # a timeout recorded by the last call before a check is reported too
    assert L.mm4_debug_noalloc_wait_timeout(2_000_000, stream_handle()) == 0
    assert L.mm4_check(stream_handle()) == MM4_ERR_TIMEOUT
    assert L.mm4_check(stream_handle()) == 0


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
