"""The strong-scaled shard layouts that `bench.py --gpus N` runs, on two ranks.

One process per GPU (NCCL only for gathering the shards to rank 0 and for
the split-K group's set-up); both ranks draw the same full-size inputs from
the same seed and keep their own shard:

  attention   (batch, head) units: rank r owns a block of the B*H heads;
  GEMM        C column blocks: rank r owns B[:, cols_r], bias[cols_r], C[:, cols_r];
  conv2d      the batch;
  split-K     K shards on 64-element boundaries, the BASELINE K = 65520
              cut into 32768 + 32752, fp32 partials summed inside the
              split-K kernels over NVLink peer memory into rank 0's C.

Rank 0 assembles the shards and checks the whole result against the oracle
(the reference's CPU loops) and, for attention, bit for bit against the
unsharded kernel on one GPU (each (batch, head) unit is computed alone).
Skipped with fewer than two GPUs. NVLS is off (plain peer transport)."""
import multiprocessing as mp
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "oracle"))

pytestmark = pytest.mark.gpu


def _gather(t, world):
    import torch
    import torch.distributed as dist
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t.contiguous())
    return parts


def _excess(got, ref):
    """max(|got - ref| - (atol + rtol |ref|)): <= 0 means every element is within the BASELINE tolerance."""
    import numpy as np
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float((np.abs(got - ref) - (2e-2 + 1e-2 * np.abs(ref))).max())


def _worker(rank, world, port, q):
    try:
        import datetime

        import torch
        import torch.distributed as dist

        import bench
        import oracle
        from example_matmul_metal4_b200 import BuildOptions, GEMMDimensions, GemmPlan, sync_check
        from example_matmul_metal4_b200.attention import AttentionDimensions, AttentionPlan
        from example_matmul_metal4_b200.conv import WEIGHTS_OHWI, Conv2DDimensions, ConvPlan
        from example_matmul_metal4_b200.parallel import SplitKGroup
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        store = dist.TCPStore("127.0.0.1", port, world_size=world + 1, is_master=False,
                              timeout=datetime.timedelta(seconds=60))
        dist.init_process_group("nccl", store=store, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        threads = oracle.default_threads()
        out = {}

        def gen(seed):
            g = torch.Generator(device=dev)
            g.manual_seed(seed)
            return g

        # ---- attention: (batch, head) units
        B, H, S, D = 2, 4, 640, 128
        g = gen(3)
        Q, K, V = (torch.randn((B, H, S, D), generator=g, device=dev).half() for _ in range(3))
        u0, nu = bench.shard_range(B * H, world, rank)
        flat = lambda t: t.reshape(B * H, S, D)[u0:u0 + nu].reshape(1, nu, S, D).contiguous()  # noqa: E731
        plan = AttentionPlan(AttentionDimensions(S, S, D, nu, nu), batch=1)
        O = plan.run(flat(Q), flat(K), flat(V))
        sync_check()
        parts = _gather(O, world)
        if rank == 0:
            whole = torch.cat([p.reshape(-1, S, D) for p in parts]).reshape(B, H, S, D)
            full = AttentionPlan(AttentionDimensions(S, S, D, H, H), batch=B).run(Q, K, V)
            sync_check()
            hq, hk, hv = (t.cpu().numpy() for t in (Q, K, V))
            rows = [(0, 64), (S - 64, S)]
            ex = max(_excess(whole[:, :, r0:r1].float().cpu().numpy(),
                             oracle.attention(hq, hk, hv, B, H, H, S, S, D, plan.scale, rows=(r0, r1),
                                              threads=threads)) for r0, r1 in rows)
            out["attention"] = (ex, bool(torch.equal(whole, full)))

        # ---- GEMM + bias: C column blocks
        M, N, Kd = 1024, 1024, 1024
        g = gen(1)
        A = (torch.rand((M, Kd), generator=g, device=dev) * 2 - 1).half()
        Bm = (torch.rand((Kd, N), generator=g, device=dev) * 2 - 1).half()
        bias = (torch.rand((N,), generator=g, device=dev) * 2 - 1).half()
        n0, nr = bench.shard_range(N, world, rank, 8)
        plan = GemmPlan(GEMMDimensions(M, nr, Kd), transpose=(False, False), bias=True)
        C = plan.run(A, Bm[:, n0:n0 + nr].contiguous(), bias[n0:n0 + nr].contiguous())
        sync_check()
        parts = _gather(C, world)
        if rank == 0:
            whole = torch.cat(parts, dim=1)
            ref = oracle.gemm(A.cpu().numpy(), Bm.cpu().numpy(), bias.cpu().numpy(), M, N, Kd, threads=threads)
            out["gemm_columns"] = (_excess(whole.float().cpu().numpy(), ref), True)

        # ---- conv2d 3x3 pad 1: batch
        NB, Hh, Ww, Ci, Co = 4, 20, 24, 64, 128
        g = gen(4)
        x = torch.randn((NB, Hh, Ww, Ci), generator=g, device=dev).half()
        w = (torch.randn((Co, 3, 3, Ci), generator=g, device=dev) * 0.05).half()
        cb = ((torch.rand((Co,), generator=g, device=dev) * 2 - 1) * 0.1).half()
        b0, nb = bench.shard_range(NB, world, rank)
        plan = ConvPlan(Conv2DDimensions(nb, Hh, Ww, Ci, Co, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1), weight_layout=WEIGHTS_OHWI,
                        bias=True)
        y = plan.run(x[b0:b0 + nb].contiguous(), w, cb)
        sync_check()
        parts = _gather(y, world)
        if rank == 0:
            whole = torch.cat(parts)
            ref = oracle.conv2d(x.cpu().numpy(), w.cpu().numpy(), cb.cpu().numpy(), N=NB, H=Hh, W=Ww, C=Ci, O=Co,
                                KH=3, KW=3, pad_top=1, pad_bottom=1, pad_left=1, pad_right=1, layout=1,
                                threads=threads)
            out["conv2d_batch"] = (_excess(whole.float().cpu().numpy(), ref), True)

        # ---- split-K (K = 65520): K shards with an uneven tail, fused group reduce
        M, N, Kd, split = 512, 512, 65520, 32
        g = gen(2)
        A = (torch.rand((M, Kd), generator=g, device=dev) * 2 - 1).half()
        Bm = (torch.rand((Kd, N), generator=g, device=dev) * 2 - 1).half()
        bias = (torch.rand((N,), generator=g, device=dev) * 2 - 1).half()
        k0, kr = bench.shard_range(Kd, world, rank, 64)
        plan = GemmPlan(GEMMDimensions(M, N, kr), transpose=(False, False), bias=True,
                        buildOptions=BuildOptions(splitK=split))
        grp = SplitKGroup(plan, root=0)
        Ar, Br = A[:, k0:k0 + kr].contiguous(), Bm[k0:k0 + kr].contiguous()
        worst = -1e30
        for _ in range(3):  # the exchange halves alternate by run parity
            grp.run(Ar, Br, bias)
            torch.cuda.synchronize()
            if rank == 0:
                got = grp.C.float().cpu().numpy()
                rows = (0, 24)
                ref = oracle.gemm(A.cpu().numpy(), Bm.cpu().numpy(), bias.cpu().numpy(), M, N, Kd, rows=rows,
                                  threads=threads)
                prev = torch.backends.cuda.matmul.allow_tf32
                torch.backends.cuda.matmul.allow_tf32 = False
                full = (A.float() @ Bm.float() + bias.float()).cpu().numpy()
                torch.backends.cuda.matmul.allow_tf32 = prev
                worst = max(worst, _excess(got[rows[0]:rows[1]], ref), _excess(got, full))
            dist.barrier()
        grp.close()
        if rank == 0:
            out["splitk_k_shards"] = (worst, True)
            out["splitk_shard_sizes"] = [bench.shard_range(Kd, world, r, 64)[1] for r in range(world)]
        dist.destroy_process_group()
        if rank == 0:
            q.put(("ok", out))
    except Exception as e:  # noqa: BLE001
        import traceback
        q.put(("error", f"rank {rank}: {type(e).__name__}: {e}\n{traceback.format_exc()}"))


def test_two_rank_strong_scaling_shards():
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
    procs = [ctx.Process(target=_worker, args=(r, world, store.port, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        kind, payload = q.get(timeout=300)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    assert kind == "ok", payload
    assert payload["splitk_shard_sizes"] == [32768, 32752]
    for layout in ("attention", "gemm_columns", "conv2d_batch", "splitk_k_shards"):
        excess, exact = payload[layout]
        assert excess <= 0.0, (layout, payload)
        assert exact, (layout, "sharded attention differs from the unsharded kernel")
