"""Multi-rank host logic on CPU with the gloo backend (world size 2):
K-shard arithmetic, the fp32 partial reduction of the split-K path, and
failure detection when a rank leaves (a short process-group timeout ends the
surviving rank's collective with an error instead of a hang)."""
import multiprocessing as mp
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

from example_matmul_metal4_b200.parallel import k_shard, shard, splitk_per_rank  # noqa: E402


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_k_shards_cover_and_align():
    for K, P in [(65536, 8), (65520, 8), (65520, 3), (1000, 4), (64, 8)]:
        spans = [k_shard(K, P, r) for r in range(P)]
        assert spans[0][0] == 0 and spans[-1][1] == K
        for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
            assert a1 == b0
        for k0, _ in spans:
            assert k0 % 8 == 0
    assert [shard(10, 3, i) for i in range(3)] == [(0, 3), (3, 6), (6, 10)]
    assert splitk_per_rank(32, 8) == 4 and splitk_per_rank(32, 64) == 1


def _worker(rank, world, port, M, N, K, q):
    import datetime
    import torch
    import torch.distributed as dist
    sys.path.insert(0, str(ROOT))
    from example_matmul_metal4_b200 import data
    from example_matmul_metal4_b200.parallel import k_shard, reduce_partials
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    A = data.uniform((M, K), -1, 1, 2, 0).astype(np.float32)
    B = data.uniform((K, N), -1, 1, 2, 1).astype(np.float32)
    k0, k1 = k_shard(K, world, rank)
    partial = torch.from_numpy(A[:, k0:k1] @ B[k0:k1])  # stands in for mm4_gemm_partial_run
    reduce_partials(partial, dst=0)
    if rank == 0:
        q.put(partial.numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_splitk_partials_reduce_to_full_product():
    M, N, K, world = 32, 24, 4104, 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, M, N, K, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = q.get(timeout=120)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    from example_matmul_metal4_b200 import data
    A = data.uniform((M, K), -1, 1, 2, 0).astype(np.float64)
    B = data.uniform((K, N), -1, 1, 2, 1).astype(np.float64)
    np.testing.assert_allclose(got, A @ B, rtol=1e-4, atol=1e-3)


def _leaver(rank, world, port, q):
    import datetime
    import torch
    import torch.distributed as dist
    sys.path.insert(0, str(ROOT))
    from example_matmul_metal4_b200.parallel import reduce_partials
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    t = torch.ones(16)
    reduce_partials(t, dst=0)  # step 1: both ranks take part
    if rank == 1:
        os._exit(0)  # rank 1 leaves between steps, with nothing in flight
    try:
        reduce_partials(t, dst=0)  # step 2: rank 0 must get an error, not hang
        q.put("no error")
    except Exception as e:  # noqa: BLE001
        q.put(f"error: {type(e).__name__}")
    os._exit(0)


def test_rank_leaving_is_detected_by_timeout():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaver, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    msg = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert msg.startswith("error"), msg
