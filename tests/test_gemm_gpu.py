"""GEMM parity on the GPU: mm4 (through the C ABI) vs the C oracle
(matmul.swift:499-510 restated), on seeded inputs."""
import pytest

import oracle
from example_matmul_metal4_b200 import BuildOptions, GEMMDimensions, GemmPlan, MM4Error, lib, sync_check
from example_matmul_metal4_b200 import data
from example_matmul_metal4_b200.gemm import splitk_finalize
from tolerance import assert_close

pytestmark = pytest.mark.gpu


def _inputs(M, N, K, tl, tr, seed, lo=-1.0, hi=1.0):
    a_shape = (K, M) if tl else (M, K)
    b_shape = (N, K) if tr else (K, N)
    A = data.uniform(a_shape, lo, hi, seed, 0)
    B = data.uniform(b_shape, lo, hi, seed, 1)
    bias = data.uniform((N,), lo, hi, seed, 2)
    return A, B, bias


def _run(cuda, M, N, K, tl, tr, split=1, bias=True, seed=7, rows=None, dup=1):
    import torch
    A, B, b = _inputs(M, N, K, tl, tr, seed)
    plan = GemmPlan(GEMMDimensions(M, N, K), transpose=(tl, tr), bias=bias, buildOptions=BuildOptions(splitK=split))
    tA = torch.from_numpy(A).to(cuda)
    tB = torch.from_numpy(B).to(cuda)
    tb = torch.from_numpy(b).to(cuda)
    C = plan.run(tA, tB, tb if bias else None, duplicatedCount=dup)
    sync_check()
    got = C.float().cpu().numpy()
    ref = oracle.gemm(A, B, b if bias else None, M, N, K, tl, tr, rows=rows, threads=oracle.default_threads())
    if rows:
        got = got[rows[0]:rows[1]]
    return plan, got, ref


@pytest.mark.parametrize("tl,tr", [(False, False), (False, True), (True, False), (True, True)])
def test_layouts(cuda, tl, tr):
    plan, got, ref = _run(cuda, 256, 384, 320, tl, tr)
    assert "sm100" in plan.kernel_name
    assert_close(got, ref, f"layout tl={tl} tr={tr}")


def test_baseline_config1_1024_nn_bias(cuda):
    """M=N=K=1024, row-major NN, bias, U[-1,1], seed 1."""
    plan, got, ref = _run(cuda, 1024, 1024, 1024, False, False, seed=1)
    assert_close(got, ref, "1024^3")


def test_reference_nt_shape_split30(cuda):
    """The reference's own NT split-K run (matmul.swift:335): M=32, N=3072, K=80000, B stored [N][K],
    splitK 30 -- more (split, tile) units than CTAs, so the last-arriving split finalizes each tile."""
    plan, got, ref = _run(cuda, 32, 3072, 80000, False, True, split=30, seed=5)
    assert "splitk" in plan.kernel_name
    assert_close(got, ref, "32x3072x80000 NT split 30")


def test_8192_cube_vs_fp32_reference(cuda):
    """The north-star 8192^3 GEMM+bias at full size (CTA-pair kernel): every output against a plain
    PyTorch fp32 GEMM (TF32 off) of the same fp16 inputs, plus the C oracle on a row sample."""
    import torch
    torch.backends.cuda.matmul.allow_tf32 = False
    M = N = K = 8192
    g = torch.Generator(device=cuda)
    g.manual_seed(11)
    A = (torch.rand((M, K), generator=g, device=cuda) * 2 - 1).half()
    B = (torch.rand((K, N), generator=g, device=cuda) * 2 - 1).half()
    b = (torch.rand((N,), generator=g, device=cuda) * 2 - 1).half()
    plan = GemmPlan(GEMMDimensions(M, N, K), transpose=(False, False), bias=True)
    assert "pair" in plan.kernel_name
    C = plan.run(A, B, b)
    sync_check()
    ref = torch.addmm(b.float(), A.float(), B.float())
    err = (C.float() - ref).abs()
    bad = int((err > 2e-2 + 1e-2 * ref.abs()).sum().item())
    assert bad == 0, f"{bad} mismatches, max abs err {err.max().item():.4g}"
    rows = (4096, 4100)
    ref_rows = oracle.gemm(A.cpu().numpy(), B.cpu().numpy(), b.cpu().numpy(), M, N, K, rows=rows,
                           threads=oracle.default_threads())
    assert_close(C[rows[0]:rows[1]].float().cpu().numpy(), ref_rows, "8192^3 oracle rows")


@pytest.mark.parametrize("M,N,K", [(200, 136, 200), (129, 264, 72), (1, 8, 8), (130, 520, 1000), (64, 64, 64)])
def test_edges_and_k_tails(cuda, M, N, K):
    plan, got, ref = _run(cuda, M, N, K, False, False)
    assert "sm100" in plan.kernel_name
    assert_close(got, ref, f"{M}x{N}x{K}")


@pytest.mark.parametrize("M,N,K", [(33, 40, 31), (17, 9, 1), (64, 33, 33)])
def test_unaligned_uses_reduced_alignment_kernel(cuda, M, N, K):
    plan, got, ref = _run(cuda, M, N, K, False, True)
    assert "simt" in plan.kernel_name
    assert_close(got, ref, f"{M}x{N}x{K}")


@pytest.mark.parametrize("K,split", [(8192, 32), (8192, 5), (4160, 7)])
def test_split_k(cuda, K, split):
    plan, got, ref = _run(cuda, 512, 512, K, False, False, split=split)
    assert "splitk" in plan.kernel_name
    assert_close(got, ref, f"split {split} K={K}")


@pytest.mark.parametrize("M,N,K,split,tr", [(1024, 1024, 8192, 16, False), (640, 768, 4096, 12, True),
                                            (512, 300, 2048, 4, False), (384, 136, 4096, 8, False)])
def test_split_k_tiles_and_finalize_modes(cuda, M, N, K, split, tr):
    """128x512 tiles with more units than SMs (last-arriving-unit finalize),
    with as many units as SMs or fewer (cooperative sliced finalize), N tails,
    and both B layouts."""
    plan, got, ref = _run(cuda, M, N, K, False, tr, split=split, rows=(0, min(M, 256)))
    assert_close(got, ref, f"{M}x{N}x{K} split {split} {plan.kernel_name}")
    plan, got2, ref2 = _run(cuda, M, N, K, False, tr, split=split, rows=(max(0, M - 64), M))
    assert_close(got2, ref2, "last rows")


def test_split_k_repeat_leaves_workspace_clean(cuda):
    """duplicatedCount re-runs the same launch; each run must re-zero its
    workspace so every repetition produces the same result."""
    plan, got, ref = _run(cuda, 256, 512, 4096, False, False, split=16, dup=3)
    assert_close(got, ref, "split-K x3")


@pytest.mark.slow
@pytest.mark.parametrize("K", [65536, 65520])
def test_baseline_config2_split_k_full(cuda, K):
    """M=N=512, K=65536 / 65520, split-K 32, seed 2."""
    plan, got, ref = _run(cuda, 512, 512, K, False, False, split=32, seed=2)
    assert_close(got, ref, f"512x512x{K}")


def test_partial_and_finalize(cuda):
    import torch
    M, N, K = 256, 256, 1024
    A, B, b = _inputs(M, N, K, False, False, 3)
    tA, tB, tb = (torch.from_numpy(x).to(cuda) for x in (A, B, b))
    # two K shards summed on the host side, then bias + cast
    half = K // 2
    p0 = GemmPlan(GEMMDimensions(M, N, half), transpose=(False, False), bias=False)
    c0 = p0.partial(tA[:, :half].contiguous(), tB[:half].contiguous())
    c1 = p0.partial(tA[:, half:].contiguous(), tB[half:].contiguous())
    C = splitk_finalize(c0 + c1, tb)
    sync_check()
    ref = oracle.gemm(A, B, b, M, N, K, False, False, threads=oracle.default_threads())
    assert_close(C.float().cpu().numpy(), ref, "partial+finalize")


def test_bounded_wait_reports_timeout_and_context_survives(cuda):
    L = lib()
    assert L.mm4_debug_wait_timeout(2_000_000, None) == 0  # 2 ms
    with pytest.raises(MM4Error) as e:
        sync_check()
    assert "TIMEOUT" in str(e.value)
    # the context is still usable
    plan, got, ref = _run(cuda, 128, 128, 128, False, False)
    assert_close(got, ref, "after timeout")


def test_invalid_descriptor_rejected():
    with pytest.raises(MM4Error):
        GemmPlan(GEMMDimensions(0, 16, 16))


@pytest.mark.parametrize("M,N,K,split,tr", [(512, 512, 65536, 32, False), (32, 3072, 80000, 30, True),
                                            (640, 768, 4160, 7, False)])
def test_deterministic_split_k(cuda, monkeypatch, M, N, K, split, tr):
    """MM4_SPLITK_DETERMINISTIC=1 (read when the plan is created): each split stores its partial and the
    finalize sums the splits in order, so repeated runs give identical bits; within tolerance of the oracle
    (rows at both ends; all rows for the smaller shapes). Covers the cooperative finalize (512x512, the
    BASELINE shape), the last-arriver finalize (the reference's 32x3072x80000 NT run) and a K tail."""
    import torch
    monkeypatch.setenv("MM4_SPLITK_DETERMINISTIC", "1")
    A, B, b = _inputs(M, N, K, False, tr, 9)
    plan = GemmPlan(GEMMDimensions(M, N, K), transpose=(False, tr), bias=True, buildOptions=BuildOptions(splitK=split))
    assert "splitk-deterministic" in plan.kernel_name
    tA, tB, tb = (torch.from_numpy(x).to(cuda) for x in (A, B, b))
    ws = plan.workspace(cuda)
    first = plan.run(tA, tB, tb, workspace=ws).clone()
    for _ in range(3):
        again = plan.run(tA, tB, tb, workspace=ws)
        sync_check()
        assert torch.equal(again, first)
    rows = (0, M) if M * N <= 640 * 768 else (0, 8)
    ref = oracle.gemm(A, B, b, M, N, K, False, tr, rows=rows, threads=oracle.default_threads())
    assert_close(first.float().cpu().numpy()[rows[0]:rows[1]], ref, f"deterministic split {split}")
    if M * N > 640 * 768:
        ref2 = oracle.gemm(A, B, b, M, N, K, False, tr, rows=(M - 8, M), threads=oracle.default_threads())
        assert_close(first.float().cpu().numpy()[M - 8:M], ref2, f"deterministic split {split} last rows")


@pytest.mark.parametrize("M,N,K,tl,tr,split", [(1000, 768, 1024, False, False, 1), (1024, 1024, 1024, False, True, 1),
                                               (512, 640, 4096, True, False, 1), (768, 512, 8192, False, False, 8)])
def test_host_buffer_gemm(cuda, M, N, K, tl, tr, split):
    """mm4_gemm_run_host (pinned host A, B, bias in, C out, pipelined over 256-row blocks): the bits of
    mm4_gemm_run for direct plans (row blocks, a ragged last block, B stored [N][K], A stored [K][M] as one
    block), and within tolerance of the oracle for a split-K plan, whose blocks are GEMMs of their own."""
    import torch
    A, B, b = _inputs(M, N, K, tl, tr, 11)
    plan = GemmPlan(GEMMDimensions(M, N, K), transpose=(tl, tr), bias=True, buildOptions=BuildOptions(splitK=split))
    tA, tB, tb = (torch.from_numpy(x).to(cuda) for x in (A, B, b))
    ref = plan.run(tA, tB, tb).cpu()
    sync_check()
    hA, hB, hb = (x.cpu().pin_memory() for x in (tA, tB, tb))
    hC = torch.empty((M, N), dtype=torch.float16).pin_memory()
    staging = (torch.empty_like(tA), torch.empty_like(tB), torch.empty_like(tb),
               torch.empty((M, N), dtype=torch.float16, device=cuda))
    for chunks in (1, 3, 64):
        hC.fill_(float("nan"))
        plan.run_host(hA, hB, hb, hC, staging, chunks=chunks)
        sync_check()
        if split == 1:
            assert torch.equal(hC, ref), chunks
        else:
            got = hC.float().numpy()
            assert_close(got[:8], oracle.gemm(A, B, b, M, N, K, tl, tr, rows=(0, 8), threads=oracle.default_threads()),
                         f"host-buffer split-K chunks={chunks}")
            assert_close(got, ref.float().numpy(), f"host-buffer split-K vs device run, chunks={chunks}")


@pytest.mark.parametrize("deterministic", [False, True])
def test_host_buffer_and_device_runs_share_one_workspace(cuda, monkeypatch, deterministic):
    """A split-K plan's workspace serves mm4_gemm_run and mm4_gemm_run_host in any order: the host-buffer
    path's block plans use the plan's own arrival counters, so neither path leaves the other a counter that
    is not a multiple of the split count or a partial area that is not clean. Deterministic mode gives the
    same bits on every repeat of each path."""
    import torch
    if deterministic:
        monkeypatch.setenv("MM4_SPLITK_DETERMINISTIC", "1")
    else:
        monkeypatch.delenv("MM4_SPLITK_DETERMINISTIC", raising=False)
    M, N, K, split = 768, 768, 8192, 8
    A, B, b = _inputs(M, N, K, False, False, 13)
    plan = GemmPlan(GEMMDimensions(M, N, K), transpose=(False, False), bias=True,
                    buildOptions=BuildOptions(splitK=split))
    assert ("splitk-deterministic" in plan.kernel_name) == deterministic
    tA, tB, tb = (torch.from_numpy(x).to(cuda) for x in (A, B, b))
    ws = plan.workspace(cuda)
    hA, hB, hb = (x.cpu().pin_memory() for x in (tA, tB, tb))
    staging = (torch.empty_like(tA), torch.empty_like(tB), torch.empty_like(tb),
               torch.empty((M, N), dtype=torch.float16, device=cuda))
    dev_runs, host_runs = [], []
    for _ in range(3):
        dev_runs.append(plan.run(tA, tB, tb, workspace=ws).cpu())
        sync_check()
        hC = torch.empty((M, N), dtype=torch.float16).pin_memory()
        plan.run_host(hA, hB, hb, hC, staging, workspace=ws, chunks=3)
        sync_check()
        host_runs.append(hC.clone())
    ref = oracle.gemm(A, B, b, M, N, K, rows=(0, 8), threads=oracle.default_threads())
    ref_end = oracle.gemm(A, B, b, M, N, K, rows=(M - 8, M), threads=oracle.default_threads())
    for i, (c, h) in enumerate(zip(dev_runs, host_runs)):
        for name, got in (("device", c), ("host-buffer", h)):
            g = got.float().numpy()
            assert_close(g[:8], ref, f"{name} run {i}, first rows")
            assert_close(g[M - 8:], ref_end, f"{name} run {i}, last rows")
        assert_close(h.float().numpy(), dev_runs[0].float().numpy(), f"host-buffer run {i} vs device run")
        if deterministic:
            assert torch.equal(c, dev_runs[0]) and torch.equal(h, host_runs[0]), i
