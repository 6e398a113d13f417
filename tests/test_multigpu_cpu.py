"""Multi-rank host logic on CPU with the gloo backend (world size 2):
K-shard arithmetic, the fp32 partial reduction of the split-K path, and
failure detection when a rank leaves between steps (the survivors learn of it
on the host through a store heartbeat, before launching the next step's
collective, instead of hanging in it)."""
import multiprocessing as mp
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

from example_matmul_metal4_b200.parallel import k_shard, shard, splitk_per_rank  # noqa: E402


def _init_rank(rank, world, port, seconds):
    """Joins the gloo group through the parent's TCPStore on 127.0.0.1 (loopback transport)."""
    import datetime
    import torch.distributed as dist
    os.environ["GLOO_SOCKET_IFNAME"] = "lo"
    store = dist.TCPStore("127.0.0.1", port, world_size=world + 1, is_master=False,
                          timeout=datetime.timedelta(seconds=60))
    dist.init_process_group("gloo", store=store, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=seconds))
    return store


def _run_ranks(target, world, args, wait=120):
    """Runs `target(rank, world, port, q, *args)` in `world` spawned processes. The parent holds the
    rendezvous store (an OS-assigned port, so concurrent runs cannot collide) and returns the
    first message a rank puts on the queue; ranks report exceptions there instead of hanging."""
    import datetime
    import torch.distributed as dist
    store = dist.TCPStore("127.0.0.1", 0, world_size=world + 1, is_master=True,
                          timeout=datetime.timedelta(seconds=60), wait_for_workers=False)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=target, args=(r, world, store.port, q) + tuple(args)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        msg = q.get(timeout=wait)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    del store
    return msg, [p.exitcode for p in procs]


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


def _worker(rank, world, port, q, M, N, K):
    try:
        import torch
        import torch.distributed as dist
        sys.path.insert(0, str(ROOT))
        from example_matmul_metal4_b200 import data
        from example_matmul_metal4_b200.parallel import k_shard, reduce_partials
        _init_rank(rank, world, port, 30)
        A = data.uniform((M, K), -1, 1, 2, 0).astype(np.float32)
        B = data.uniform((K, N), -1, 1, 2, 1).astype(np.float32)
        k0, k1 = k_shard(K, world, rank)
        partial = torch.from_numpy(A[:, k0:k1] @ B[k0:k1])  # stands in for mm4_gemm_partial_run
        reduce_partials(partial, dst=0)
        if rank == 0:
            q.put(("ok", partial.numpy()))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        import traceback
        q.put(("error", f"rank {rank}: {type(e).__name__}: {e}\n{traceback.format_exc()}"))
        raise


def test_splitk_partials_reduce_to_full_product():
    M, N, K, world = 32, 24, 4104, 2
    (kind, got), codes = _run_ranks(_worker, world, (M, N, K))
    assert kind == "ok", got
    assert codes == [0] * world
    from example_matmul_metal4_b200 import data
    A = data.uniform((M, K), -1, 1, 2, 0).astype(np.float64)
    B = data.uniform((K, N), -1, 1, 2, 1).astype(np.float64)
    np.testing.assert_allclose(got, A @ B, rtol=1e-4, atol=1e-3)


def _put_and_exit(q, msg, code=0):
    """Delivers `msg` (Queue.put hands it to a feeder thread) before ending the process."""
    q.put(msg)
    q.close()
    q.join_thread()
    os._exit(code)


def _leaver(rank, world, port, q):
    import torch
    sys.path.insert(0, str(ROOT))
    from example_matmul_metal4_b200.parallel import RankLost, StepHeartbeat, reduce_partials
    try:
        store = _init_rank(rank, world, port, 30)
        hb = StepHeartbeat(store, rank, world, timeout=3.0)
        t = torch.ones(16)
        hb.beat(1)
        reduce_partials(t, dst=0)  # step 1: both ranks take part
    except Exception as e:  # noqa: BLE001
        _put_and_exit(q, f"setup failed on rank {rank}: {type(e).__name__}: {e}", 1)
    if rank == 1:
        os._exit(0)  # rank 1 leaves between steps, with nothing in flight
    try:
        hb.beat(2)  # rank 0 learns of it on the host, before launching step 2
        reduce_partials(t, dst=0)
        _put_and_exit(q, "no error")
    except RankLost as e:
        _put_and_exit(q, f"error: RankLost step={e.step} missing={e.missing}")
    except Exception as e:  # noqa: BLE001
        _put_and_exit(q, f"other error: {type(e).__name__}: {e}")


def test_rank_leaving_is_detected_on_the_host():
    msg, _ = _run_ranks(_leaver, 2, ())
    assert msg == "error: RankLost step=2 missing=[1]", msg
