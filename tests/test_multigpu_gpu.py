"""Fused multi-GPU split-K (SplitKGroup / mm4_gemm_splitk_group_run) on real GPUs.

One process per GPU (NCCL only for the setup's handle exchange and the test's
barriers); every rank runs the split-K plan on its own K shard and the root's
C must equal sum_r A_r B_r + bias within the BASELINE tolerance, over several
runs (the exchange buffers alternate halves by run parity). The group of one
rank runs on any single GPU; the 2-rank case needs two GPUs and is skipped
otherwise. NVLS is off (plain peer loads/stores only)."""
import multiprocessing as mp
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

from tolerance import assert_close  # noqa: E402

pytestmark = pytest.mark.gpu


def _shard(dev, M, N, Kr, r, it):
    import torch
    g = torch.Generator(device=dev)
    g.manual_seed(1000 + 17 * r + 101 * it)
    A = (torch.rand(M, Kr, generator=g, device=dev) * 2 - 1).half()
    B = (torch.rand(Kr, N, generator=g, device=dev) * 2 - 1).half()
    return A, B


def _bias(dev, N):
    import torch
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    return (torch.rand(N, generator=g, device=dev) * 2 - 1).half()


def _reference(dev, M, N, Kr, world, it):
    ref = _bias(dev, N).float().expand(M, N).clone()
    for r in range(world):
        A, B = _shard(dev, M, N, Kr, r, it)
        ref += A.float() @ B.float()
    return ref


def test_group_of_one_rank(cuda):
    import torch
    from example_matmul_metal4_b200 import BuildOptions, GEMMDimensions, GemmPlan
    from example_matmul_metal4_b200.parallel import SplitKGroup
    M, N, Kr = 512, 512, 8192
    plan = GemmPlan(GEMMDimensions(M, N, Kr), transpose=(False, False), bias=True,
                    buildOptions=BuildOptions(splitK=16))
    grp = SplitKGroup(plan)
    try:
        bias = _bias(cuda, N)
        for it in range(3):
            A, B = _shard(cuda, M, N, Kr, 0, it)
            grp.run(A, B, bias)
            torch.cuda.synchronize()
            assert_close(grp.C.float().cpu().numpy(), _reference(cuda, M, N, Kr, 1, it).cpu().numpy(),
                         f"run {it}")
    finally:
        grp.close()


def _worker(rank, world, port, q, M, N, Kr, split, runs, owners):
    try:
        import datetime

        import torch
        import torch.distributed as dist
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        os.environ["MM4_SPLITK_GROUP_OWNERS"] = owners
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        store = dist.TCPStore("127.0.0.1", port, world_size=world + 1, is_master=False,
                              timeout=datetime.timedelta(seconds=60))
        dist.init_process_group("nccl", store=store, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        sys.path.insert(0, str(ROOT))
        from example_matmul_metal4_b200 import BuildOptions, GEMMDimensions, GemmPlan
        from example_matmul_metal4_b200.parallel import SplitKGroup
        plan = GemmPlan(GEMMDimensions(M, N, Kr), transpose=(False, False), bias=True,
                        buildOptions=BuildOptions(splitK=split))
        grp = SplitKGroup(plan, root=0)
        bias = _bias(dev, N)
        worst = []
        for it in range(runs):
            A, B = _shard(dev, M, N, Kr, rank, it)
            grp.run(A, B, bias)
            torch.cuda.synchronize()
            if rank == 0:
                ref = _reference(dev, M, N, Kr, world, it)
                excess = ((grp.C.float() - ref).abs() - (2e-2 + 1e-2 * ref.abs())).max().item()
                worst.append(excess)
            dist.barrier()
        grp.close()
        dist.destroy_process_group()
        if rank == 0:
            q.put(("ok", worst))
    except Exception as e:  # noqa: BLE001
        import traceback
        q.put(("error", f"rank {rank}: {type(e).__name__}: {e}\n{traceback.format_exc()}"))


@pytest.mark.parametrize("M,N,Kr,split,owners", [(512, 512, 8192, 32, "root"), (256, 768, 4104, 8, "root"),
                                                  (512, 512, 8192, 32, "spread")])
def test_two_ranks_fused_splitk(M, N, Kr, split, owners):
    """owners="root": the root finishes every slice (groups of up to four); "spread": slice % world
    finishes it and writes the root's C over NVLink (larger groups)."""
    import datetime

    import torch
    import torch.distributed as dist
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    store = dist.TCPStore("127.0.0.1", 0, world_size=world + 1, is_master=True,
                          timeout=datetime.timedelta(seconds=60), wait_for_workers=False)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, store.port, q, M, N, Kr, split, 4, owners))
             for r in range(world)]
    for p in procs:
        p.start()
    try:
        kind, payload = q.get(timeout=240)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    assert kind == "ok", payload
    assert max(payload) <= 0.0, payload


def _comm_worker(rank, world, port, q, M, N, Kr, split, runs):
    try:
        import datetime

        import torch
        import torch.distributed as dist
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        store = dist.TCPStore("127.0.0.1", port, world_size=world + 1, is_master=False,
                              timeout=datetime.timedelta(seconds=60))
        sys.path.insert(0, str(ROOT))
        from example_matmul_metal4_b200 import BuildOptions, GEMMDimensions, GemmPlan
        from example_matmul_metal4_b200.parallel import Comm
        # NCCL bootstrap the C-ABI way: rank 0 makes the unique id, the store carries it.
        if rank == 0:
            store.set("mm4_nccl_id", Comm.unique_id())
        uid = store.get("mm4_nccl_id")
        comm = Comm(world, rank, uid)
        plan = GemmPlan(GEMMDimensions(M, N, Kr), transpose=(False, False), bias=True,
                        buildOptions=BuildOptions(splitK=split))
        bias = _bias(dev, N)
        C = torch.empty((M, N), dtype=torch.float16, device=dev) if rank == 0 else None
        worst = []
        for it in range(runs):
            A, B = _shard(dev, M, N, Kr, rank, it)
            comm.run(plan, A, B, bias, C=C)
            torch.cuda.synchronize()
            if rank == 0:
                ref = _reference(dev, M, N, Kr, world, it)
                worst.append(((C.float() - ref).abs() - (2e-2 + 1e-2 * ref.abs())).max().item())
        comm.close()
        if rank == 0:
            q.put(("ok", worst))
    except Exception as e:  # noqa: BLE001
        import traceback
        q.put(("error", f"rank {rank}: {type(e).__name__}: {e}\n{traceback.format_exc()}"))


def test_two_ranks_nccl_bootstrapped_comm():
    """mm4_comm_init from an NCCL unique id + mm4_gemm_splitk_run_distributed (the same fused kernel)."""
    import datetime

    import torch
    import torch.distributed as dist
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    store = dist.TCPStore("127.0.0.1", 0, world_size=world + 1, is_master=True,
                          timeout=datetime.timedelta(seconds=60), wait_for_workers=False)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_comm_worker, args=(r, world, store.port, q, 512, 512, 8192, 32, 3))
             for r in range(world)]
    for p in procs:
        p.start()
    try:
        kind, payload = q.get(timeout=240)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    assert kind == "ok", payload
    assert max(payload) <= 0.0, payload


@pytest.mark.parametrize("owners", ["root", "spread"])
def test_every_gpu_fused_splitk(owners):
    """The fused split-K group on every GPU of the box (at least three, at most eight): ranks 2 and up
    push into slots beyond the first two of the owner's staging, and with spread owners every rank owns
    slices."""
    import datetime

    import torch
    import torch.distributed as dist
    n = torch.cuda.device_count()
    if n < 3:
        pytest.skip("needs three or more GPUs")
    world = min(n, 8)
    store = dist.TCPStore("127.0.0.1", 0, world_size=world + 1, is_master=True,
                          timeout=datetime.timedelta(seconds=60), wait_for_workers=False)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, store.port, q, 512, 512, 8192, 32, 3, owners))
             for r in range(world)]
    for p in procs:
        p.start()
    try:
        kind, payload = q.get(timeout=240)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    assert kind == "ok", payload
    assert max(payload) <= 0.0, payload
