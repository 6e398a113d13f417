#!/usr/bin/env python
"""Benchmark of the mm4 tensor-op contraction path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl mm4|reference]

Prints ONE JSON line (rank 0). A "step" is one pass of the hot path over one
batch of synthetic input (seeded torch generators, fp16, BASELINE shapes and
distributions):

  attention (default)  BASELINE configs[2]: B=4, H=16, S=4096, D=128,
                    non-causal, fp16 out (the largest config, tensor-bound).
  attention_bwd     its backward: dQ, dK, dV from O, dO and the forward's LSE.
  splitk            BASELINE configs[1]: C = A*B + bias, M=N=512, K=65536,
                    split-K 32, fp32 partials reduced in-kernel, fp16 out.
  splitk65520       the K=65520 variant of configs[1].
  gemm1024          BASELINE configs[0] (1024^3 GEMM+bias, NN).
  gemm8192          the north-star target shape, 8192^3 GEMM+bias, NN.
  conv2d            BASELINE configs[3]: N=32, 56x56, 256->256, 3x3, pad 1.
  conv3d            BASELINE configs[4]: N=8, D=16, 64x64, 128->128, 3x3x3, pad 1.

N>1 (torchrun, one rank per GPU) splits ONE copy of the named shape over the
ranks along its natural shards (strong scaling; `value` is the whole shape's
rate over the slowest rank's time):
  attention(_bwd)   the B*H = 64 (batch, head) units, 64/N per rank;
  gemm*             N-column blocks: rank r owns B[:, cols_r], bias[cols_r]
                    and C[:, cols_r]; A is replicated;
  conv*             the batch, N/P images per rank;
  splitk*           K shards on 64-element boundaries (65536 -> 8 x 8192;
                    65520 -> 7 x 8192 + 8176); each rank runs the split-K
                    kernel on its shard and the ranks' fp32 partials meet
                    inside those kernels over NVLink peer memory (one fused
                    launch per GPU, no separate collective) in rank 0's C.
No other workload has a data-path collective.

Timing: W untimed warm-up steps, then K timed steps, each bracketed by CUDA
events on the launching stream, with every step's inputs out of L2: HBM-bound
and small workloads read the next of several device copies of their inputs
each step (together well over the 126 MB L2), the others get a 512 MiB write
between steps that flushes L2 outside the events (--l2 rotate|flush forces
either). Barrier + synchronize on both sides; the reported time is the max
over ranks. `launch_only` times `steps` launches issued by ONE call through
the C ABI's duplicated_count (the reference's duplicatedCount loop), which
separates the kernels from per-call host issue.

`--impl reference` times the reference's CPU implementation of the path (the
C restatement of its Swift validation loops under oracle/, all host threads)
on a bounded sample of the same workload, extrapolated to the full workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PEAKS_FILE = ROOT / "MEASURED_PEAKS.json"
TRAFFIC_FILE = ROOT / "profiles" / "dram_traffic.json"
METRIC = "TFLOP/s per GPU & % of fp16 tensor peak (GEMM/attn/conv)"


def shard_range(total, parts, index, align=1):
    """[start, start + count) of shard `index` when `total` is cut into `parts` shards whose boundaries
    fall on multiples of `align`; the last shard takes what is left (65520 over 8 on 64-element
    boundaries: 7 x 8192 + 8176)."""
    per = -(-total // parts)
    per = -(-per // align) * align
    start = min(total, index * per)
    end = total if index == parts - 1 else min(total, start + per)
    return start, end - start


def load_peaks():
    try:
        p = json.loads(PEAKS_FILE.read_text())
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "bf16_tflops_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])),
                "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def load_traffic(name):
    try:
        return json.loads(TRAFFIC_FILE.read_text()).get(name)
    except Exception:
        return None


# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------

class GemmWorkload:
    def __init__(self, M, N, K, split, seed, bound, config_index):
        self.M, self.N, self.K, self.split, self.seed = M, N, K, split, seed
        self.bound = bound
        self.config_index = config_index
        self.name = (f"splitk_gemm_bias_{M}x{N}x{K}_s{split}_nn" if split > 1 else f"gemm_bias_{M}x{N}x{K}_nn")

    def flops(self):
        return 2.0 * self.M * self.N * self.K

    def bytes(self):
        return 2.0 * (self.M * self.K + self.K * self.N + self.N + self.M * self.N)

    def config(self):
        return {"workload": self.name, "M": self.M, "N": self.N, "K": self.K, "split_k": self.split,
                "layout": "row-major NN (A[M][K], B[K][N])", "bias": True, "inputs": "U[-1,1] fp16"}

    def inputs(self, dev, gen, N=None, K=None):
        """A [M][K], B [K][N], bias [N]; N or K narrowed to a rank's shard when given."""
        import torch
        N, K = N or self.N, K or self.K
        A = (torch.rand((self.M, K), generator=gen, device=dev) * 2 - 1).half()
        B = (torch.rand((K, N), generator=gen, device=dev) * 2 - 1).half()
        bias = (torch.rand((N,), generator=gen, device=dev) * 2 - 1).half()
        return {"A": A, "B": B, "bias": bias}


class AttentionWorkload:
    name = "attention_fwd_b4_h16_s4096_d128_noncausal"
    bound = "tensor"
    config_index = 2
    B, H, S, D = 4, 16, 4096, 128
    seed = 3

    def flops(self):
        return 4.0 * self.B * self.H * self.S * self.S * self.D

    def bytes(self):
        return 4.0 * self.B * self.H * self.S * self.D * 2

    def config(self):
        return {"workload": self.name, "batch": self.B, "heads": self.H, "seq_len": self.S, "head_dim": self.D,
                "layout": "[B][H][S][D]", "scale": 1 / math.sqrt(self.D), "inputs": "N(0,1) fp16",
                "reference_flop_count_(2D+5)S^2H": (2 * self.D + 5) * self.S * self.S * self.H * self.B}

    def shard(self, parts, index):
        """(batch, heads) of this rank's block of the B*H (batch, head) units, in [B][H] order."""
        u0, nu = shard_range(self.B * self.H, parts, index)
        if nu % self.H == 0 and u0 % self.H == 0:
            return nu // self.H, self.H
        return 1, nu

    def inputs(self, dev, gen, shape=None):
        import torch
        shp = shape or (self.B, self.H, self.S, self.D)
        return {k: torch.randn(shp, generator=gen, device=dev).half() for k in ("Q", "K", "V")}


class AttentionBwdWorkload(AttentionWorkload):
    """The backward of the attention config: dQ, dK, dV from Q, K, V, the forward's O and LSE, and dO."""
    name = "attention_bwd_b4_h16_s4096_d128_noncausal"

    def flops(self):
        # five S-sized GEMMs (S, dP, dV, dK, dQ); the kernels also recompute S and dP once more for dQ
        return 10.0 * self.B * self.H * self.S * self.S * self.D

    def bytes(self):
        # Q, K, V, O, dO read and dQ, dK, dV written, fp16; LSE read (fp32)
        return 8.0 * self.B * self.H * self.S * self.D * 2 + self.B * self.H * self.S * 4

    def config(self):
        c = super().config()
        c.update({"workload": self.name, "pass": "backward: dQ, dK, dV of sum(dO * O) (Network.swift:328-401)",
                  "inputs": "Q, K, V, dO N(0,1) fp16; O and LSE from the forward, outside the timed steps"})
        return c

    def inputs(self, dev, gen, shape=None):
        import torch
        shp = shape or (self.B, self.H, self.S, self.D)
        return {k: torch.randn(shp, generator=gen, device=dev).half() for k in ("Q", "K", "V", "dO")}


class ConvWorkload:
    def __init__(self, three_d):
        self.three_d = three_d
        if three_d:
            self.name = "conv3d_ndhwc_n8_d16_64x64_c128_k128_3x3x3_pad1"
            self.config_index = 4
            self.N, self.D, self.H, self.W, self.C, self.O, self.k = 8, 16, 64, 64, 128, 128, 3
            self.wsig, self.seed = 0.03, 5
        else:
            self.name = "conv2d_nhwc_n32_56x56_c256_k256_3x3_pad1"
            self.config_index = 3
            self.N, self.D, self.H, self.W, self.C, self.O, self.k = 32, 1, 56, 56, 256, 256, 3
            self.wsig, self.seed = 0.05, 4
        self.bound = "tensor"

    def taps(self):
        return self.k ** 3 if self.three_d else self.k ** 2

    def flops(self):
        return 2.0 * self.N * self.D * self.H * self.W * self.O * self.taps() * self.C

    def bytes(self):
        return 2.0 * (self.N * self.D * self.H * self.W * (self.C + self.O) + self.O * self.taps() * self.C + self.O)

    def config(self):
        c = {"workload": self.name, "batch": self.N, "H": self.H, "W": self.W, "Cin": self.C, "Cout": self.O,
             "kernel": self.k, "stride": 1, "padding": 1, "bias": True,
             "layout": "NDHWC x [Cout][3][3][3][Cin]" if self.three_d else "NHWC x [Cout][3][3][Cin]",
             "inputs": f"x N(0,1), w N(0,{self.wsig}), bias U[-0.1,0.1], fp16"}
        if self.three_d:
            c["D"] = self.D
        return c

    def weight_shape(self):
        return (self.O, self.k, self.k, self.k, self.C) if self.three_d else (self.O, self.k, self.k, self.C)

    def inputs(self, dev, gen, batch=None):
        import torch
        n = batch or self.N
        xs = (n, self.D, self.H, self.W, self.C) if self.three_d else (n, self.H, self.W, self.C)
        x = torch.randn(xs, generator=gen, device=dev).half()
        w = (torch.randn(self.weight_shape(), generator=gen, device=dev) * self.wsig).half()
        bias = ((torch.rand((self.O,), generator=gen, device=dev) * 2 - 1) * 0.1).half()
        return {"x": x, "w": w, "bias": bias}


WORKLOADS = {
    "splitk": lambda: GemmWorkload(512, 512, 65536, 32, 2, "hbm", 1),
    "splitk65520": lambda: GemmWorkload(512, 512, 65520, 32, 2, "hbm", 1),
    "gemm1024": lambda: GemmWorkload(1024, 1024, 1024, 1, 1, "tensor", 0),
    "gemm8192": lambda: GemmWorkload(8192, 8192, 8192, 1, 11, "tensor", None),
    "attention": AttentionWorkload,
    "attention_bwd": AttentionBwdWorkload,
    "conv2d": lambda: ConvWorkload(False),
    "conv3d": lambda: ConvWorkload(True),
}


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------

class Dist:
    def __init__(self, n_gpus):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        if self.world != n_gpus:
            raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={self.world}; launch N>1 under torchrun")
        self.pg = None

    def init(self, backend):
        import datetime
        import torch.distributed as dist
        if self.world > 1:
            # The bench's collectives are a few bytes (barriers, timing max, set-up handles): NVLink
            # multicast (NVLS) buys nothing here, so keep NCCL on plain peer transport.
            os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
            dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=60))
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, value):
        if not self.pg:
            return value
        import torch
        t = torch.tensor([value], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.barrier()
            self.pg.destroy_process_group()


# ---------------------------------------------------------------------------
# clocks sampler (nvidia-smi during the timed region)
# ---------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu_index = gpu_index
        self.proc = None
        self.file = None

    def start(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu_index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.file, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.file.flush()
        rows = []
        for line in Path(self.file.name).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append(dict(sm=float(parts[1]), max=float(parts[2]), power=float(parts[3]),
                                 hw=parts[5], hw_thermal=parts[6], sw_thermal=parts[7], sw_power=parts[8]))
            except ValueError:
                continue
        os.unlink(self.file.name)
        if not rows:
            return None
        loaded = [r for r in rows if r["power"] > 250.0] or rows
        reasons = set()
        for r in rows:
            for key, name in (("hw", "hw_slowdown"), ("hw_thermal", "hw_thermal_slowdown"),
                              ("sw_thermal", "sw_thermal_slowdown"), ("sw_power", "sw_power_cap")):
                if r[key].lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r["sm"] for r in loaded), "sm_max_mhz": max(r["max"] for r in rows),
                "power_w_max": max(r["power"] for r in rows), "samples": len(rows),
                "samples_under_load": len(loaded), "reasons": sorted(reasons)}


# ---------------------------------------------------------------------------
# timing helpers
# ---------------------------------------------------------------------------

def time_steps(step, steps, warmup, flush, stream, dist):
    """Per-step CUDA events on `stream`; with `flush`, an L2 flush between steps outside the events
    (without it the step rotates its inputs, see input_sets)."""
    import torch
    for _ in range(warmup):
        if flush is not None:
            flush.zero_()
        step()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    events = []
    for _ in range(steps):
        if flush is not None:
            flush.zero_()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record(stream)
        step()
        e.record(stream)
        events.append((s, e))
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    return [s.elapsed_time(e) for s, e in events]


def burn(step, flush, seconds, dist):
    """Repeats the step (with L2 flushes) for about `seconds`, untimed. Ranks run the same number of
    steps (the step may hold a collective): after every block of 4 they agree, by a MAX all-reduce,
    whether any rank still wants to continue."""
    import torch
    t_end = time.perf_counter() + seconds
    while True:
        for _ in range(4):
            if flush is not None:
                flush.zero_()
            step()
        torch.cuda.synchronize()
        more = 1.0 if time.perf_counter() < t_end else 0.0
        if dist.max(more) == 0.0:
            return


# ---------------------------------------------------------------------------
# mm4 arm: per-workload step builders
# Each returns (step, e2e_step, (h2d, d2h) bytes, kernel name, launches/step, scaling, input sets).
# ---------------------------------------------------------------------------

L2_BYTES = 126 * 1000 * 1000  # B200 L2


def input_sets(first, l2):
    """Device copies of a step's inputs for cold-L2 timing without a flush.

    l2 == "rotate": 1 + ceil(2 * L2 / bytes) copies (at least 2); a step uses the next copy, so
    between two uses of one copy at least twice the L2 size of other inputs has been read and the
    copy is evicted. l2 == "flush": just `first` (the caller flushes L2 between steps)."""
    import torch
    if l2 != "rotate":
        return [first]
    nbytes = sum(t.numel() * t.element_size() for t in first.values())
    n = max(2, 1 + math.ceil(2 * L2_BYTES / nbytes))
    return [first] + [{k: v.clone() for k, v in first.items()} for _ in range(n - 1)]


def check_rotation(w, dist, sets):
    """The config line states rotated_input_bytes(); fail loudly if a builder rotates something else."""
    got = sum(t.numel() * t.element_size() for t in sets[0].values())
    want = rotated_input_bytes(w, dist.world, dist.rank)
    if got != want:
        raise SystemExit(f"rotated inputs are {got} bytes, rotated_input_bytes() says {want}")


def cycling(sets):
    """Returns a function giving the next input set on each call."""
    state = [0]

    def nxt():
        cur = sets[state[0]]
        state[0] = (state[0] + 1) % len(sets)
        return cur
    return nxt


def shard_splits(w, n):
    """Split-K count within each K shard: the named shape's split, reduced so that every split still covers
    at least SPLIT_MIN_K of the shard (each split reduces a full fp32 M x N partial, so thin splits cost more
    reduction traffic than they save main-loop time): 32 on 1-4 GPUs at K = 65536, 16 on 8."""
    k = shard_range(w.K, n, 0, align=64)[1]
    return max(1, min(w.split, k // SPLIT_MIN_K))


SPLIT_MIN_K = 512


def _same_on_every_rank(value, what):
    """Raises unless every rank passes the same `value` (plans whose tiles must agree across ranks)."""
    import torch.distributed as tdist
    if not tdist.is_initialized() or tdist.get_world_size() == 1:
        return
    allv = [None] * tdist.get_world_size()
    tdist.all_gather_object(allv, value)
    if any(v != allv[0] for v in allv):
        raise SystemExit(f"{what} differs across ranks: {allv}")


def build_gemm(w, dist, dev, gen, l2):
    import torch
    from example_matmul_metal4_b200 import BuildOptions, GEMMDimensions, GemmPlan
    P, r = dist.world, dist.rank
    M, N, K = w.M, w.N, w.K
    if P > 1 and w.split > 1:
        # K shards of the named shape on 64-element boundaries; the shards' fp32 partials meet inside the
        # split-K kernels over peer memory (SplitKGroup): one launch per GPU per step, no separate
        # collective; the root's C holds the result.
        import torch.distributed as tdist
        from example_matmul_metal4_b200.parallel import SplitKGroup
        k0, Kr = shard_range(K, P, r, align=64)
        t = w.inputs(dev, gen, K=Kr)
        A, B = t["A"], t["B"]
        bias = t["bias"]
        tdist.broadcast(bias, src=0)  # one bias for the whole problem
        plan = GemmPlan(GEMMDimensions(M, N, Kr), transpose=(False, False), bias=True,
                        buildOptions=BuildOptions(splitK=shard_splits(w, P)))
        _same_on_every_rank((plan.kernel_name, plan.workspace_bytes), "split-K group plan")
        grp = SplitKGroup(plan, root=0)
        sets = input_sets({"A": A, "B": B}, l2)
        nxt = cycling(sets)

        def step():
            t = nxt()
            grp.run(t["A"], t["B"], bias)
        step.close = grp.close
        step.shard = f"K rows [{k0}, {k0 + Kr})"

        hA, hB = A.cpu().pin_memory(), B.cpu().pin_memory()
        hC = torch.empty((M, N), dtype=torch.float16).pin_memory() if r == 0 else None

        def e2e_step():
            A.copy_(hA, non_blocking=True)
            B.copy_(hB, non_blocking=True)
            grp.run(A, B, bias)
            if r == 0:
                hC.copy_(grp.C, non_blocking=True)
        e2e_bytes = (A.numel() * 2 + B.numel() * 2, M * N * 2 if r == 0 else 0)
        return (step, e2e_step, e2e_bytes, plan.kernel_name + " + in-kernel cross-GPU reduce over peer memory", 1,
                "strong", sets)
    n0, Nr = shard_range(N, P, r, align=8)  # column blocks of whole 16-byte groups
    t = w.inputs(dev, gen, N=Nr)
    A, B, bias = t["A"], t["B"], t["bias"]
    sets = input_sets({"A": A, "B": B}, l2)
    nxt = cycling(sets)
    plan = GemmPlan(GEMMDimensions(M, Nr, K), transpose=(False, False), bias=True,
                    buildOptions=BuildOptions(splitK=w.split))
    C = torch.empty((M, Nr), dtype=torch.float16, device=dev)
    ws = plan.workspace(dev)

    def step():
        t = nxt()
        plan.run(t["A"], t["B"], bias, C=C, workspace=ws)

    def launch_only(n):
        t = nxt()
        plan.run(t["A"], t["B"], bias, C=C, workspace=ws, duplicatedCount=n)
    step.launch_only = launch_only
    if P > 1:
        step.shard = f"C columns [{n0}, {n0 + Nr})"

    Ct = torch.empty_like(C)

    def torch_step():
        t = nxt()
        torch.addmm(bias, t["A"], t["B"], out=Ct)
    step.comparator = ("torch.addmm (cuBLAS, fp16 in/out)", torch_step, lambda: C, lambda: Ct)

    hA, hB, hb = A.cpu().pin_memory(), B.cpu().pin_memory(), bias.cpu().pin_memory()
    hC = torch.empty((M, Nr), dtype=torch.float16).pin_memory()

    def e2e_step():
        # Host buffers in and out through the host-buffer entry point (mm4_gemm_run_host): B and bias
        # first, then A's row blocks, their GEMMs and C's row blocks pipelined over 16 chunks.
        plan.run_host(hA, hB, hb, hC, (A, B, bias, C), workspace=ws)
    e2e_bytes = (A.numel() * 2 + B.numel() * 2 + bias.numel() * 2, C.numel() * 2)
    return step, e2e_step, e2e_bytes, plan.kernel_name, 1, "strong", sets


def _attention_shard(w, dist):
    from example_matmul_metal4_b200.attention import AttentionDimensions, AttentionPlan
    nb, nh = w.shard(dist.world, dist.rank)
    plan = AttentionPlan(AttentionDimensions(w.S, w.S, w.D, nh, nh), batch=nb)
    u0, nu = shard_range(w.B * w.H, dist.world, dist.rank)
    return plan, (nb, nh, w.S, w.D), f"(batch, head) units [{u0}, {u0 + nu}) of {w.B * w.H}"


def build_attention(w, dist, dev, gen, l2):
    import torch
    plan, shape, shard = _attention_shard(w, dist)
    t = w.inputs(dev, gen, shape)
    Q, K, V = t["Q"], t["K"], t["V"]
    O = torch.empty_like(Q)
    sets = input_sets({"Q": Q, "K": K, "V": V}, l2)
    nxt = cycling(sets)

    def step():
        t = nxt()
        plan.run(t["Q"], t["K"], t["V"], O=O)

    def launch_only(n):
        t = nxt()
        plan.run(t["Q"], t["K"], t["V"], O=O, duplicatedCount=n)
    step.launch_only = launch_only
    if dist.world > 1:
        step.shard = shard

    Ot = [None]

    def torch_step():
        t = nxt()
        Ot[0] = torch.nn.functional.scaled_dot_product_attention(t["Q"], t["K"], t["V"])
    step.comparator = ("torch scaled_dot_product_attention (fp16)", torch_step, lambda: O, lambda: Ot[0])

    hQ, hK, hV = Q.cpu().pin_memory(), K.cpu().pin_memory(), V.cpu().pin_memory()
    hO = torch.empty(O.shape, dtype=O.dtype).pin_memory()

    def e2e_step():
        # Host buffers in and out through the host-buffer entry point: copies in, kernels and copies out
        # pipelined over 16 chunks of (batch, head) units (mm4_attention_fwd_host).
        plan.run_host(hQ, hK, hV, hO, (Q, K, V, O))
    return step, e2e_step, (3 * Q.numel() * 2, O.numel() * 2), plan.kernel_name, 1, "strong", sets


def build_attention_bwd(w, dist, dev, gen, l2):
    import torch
    plan, shape, shard = _attention_shard(w, dist)
    t = w.inputs(dev, gen, shape)
    Q, K, V, dO = t["Q"], t["K"], t["V"], t["dO"]
    lse = torch.empty(plan.lse_shape(), dtype=torch.float32, device=dev)
    O = plan.run(Q, K, V, lse=lse)
    dQ, dK, dV = torch.empty_like(Q), torch.empty_like(K), torch.empty_like(V)
    ws = torch.empty(plan.backward_workspace_bytes(), dtype=torch.uint8, device=dev)
    sets = input_sets({"Q": Q, "K": K, "V": V, "O": O, "dO": dO, "lse": lse}, l2)
    nxt = cycling(sets)

    def step():
        t = nxt()
        plan.backward(t["Q"], t["K"], t["V"], t["O"], t["dO"], t["lse"], dQ=dQ, dK=dK, dV=dV, workspace=ws)
    if dist.world > 1:
        step.shard = shard

    # torch: SDPA's own backward on a retained graph (its forward runs once, outside the timed steps)
    q, k, v = (x.detach().clone().requires_grad_(True) for x in (Q, K, V))
    o = torch.nn.functional.scaled_dot_product_attention(q, k, v)
    gq = [None]

    def torch_step():
        gq[0] = torch.autograd.grad(o, (q, k, v), dO, retain_graph=True)[0]
    step.comparator = ("torch scaled_dot_product_attention backward (fp16)", torch_step, lambda: dQ,
                       lambda: gq[0])

    host = {k: v.cpu().pin_memory() for k, v in sets[0].items()}
    hout = [torch.empty(x.shape, dtype=x.dtype).pin_memory() for x in (dQ, dK, dV)]
    names = ("Q", "K", "V", "O", "dO", "lse")

    def e2e_step():
        # Host buffers in and out through the host-buffer entry point (mm4_attention_bwd_host): copies in,
        # the backward and copies out pipelined over 16 chunks of key/value heads.
        f = sets[0]
        plan.backward_host(*(host[k] for k in names), *hout, tuple(f[k] for k in names), (dQ, dK, dV), ws)
    h2d = sum(v.numel() * v.element_size() for v in sets[0].values())
    d2h = 3 * Q.numel() * 2
    return (step, e2e_step, (h2d, d2h), "attention_bwd_sm100 (prep + dK/dV + dQ kernels)", 3, "strong",
            sets)


def build_conv(w, dist, dev, gen, l2):
    import torch
    from example_matmul_metal4_b200.conv import (WEIGHTS_ODHWI, WEIGHTS_OHWI, Conv2DDimensions, Conv3DDimensions,
                                                 ConvPlan)
    b0, nb = shard_range(w.N, dist.world, dist.rank)
    if w.three_d:
        dims = Conv3DDimensions(nb, w.D, w.H, w.W, w.C, w.O, 3, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1)
        plan = ConvPlan(dims, weight_layout=WEIGHTS_ODHWI, bias=True)
    else:
        dims = Conv2DDimensions(nb, w.H, w.W, w.C, w.O, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1)
        plan = ConvPlan(dims, weight_layout=WEIGHTS_OHWI, bias=True)
    t = w.inputs(dev, gen, batch=nb)
    x, wt, bias = t["x"], t["w"], t["bias"]
    y = torch.empty(plan.out_shape, dtype=torch.float16, device=dev)
    sets = input_sets({"x": x, "w": wt}, l2)
    nxt = cycling(sets)

    def step():
        t = nxt()
        plan.run(t["x"], t["w"], bias, y=y)

    def launch_only(n):
        t = nxt()
        plan.run(t["x"], t["w"], bias, y=y, duplicatedCount=n)
    step.launch_only = launch_only
    if dist.world > 1:
        step.shard = f"images [{b0}, {b0 + nb}) of {w.N}"

    yt = [None]
    F = torch.nn.functional
    # NHWC / NDHWC tensors as channels-last views of the NCHW / NCDHW shapes cuDNN takes.
    perm_x = (0, 4, 1, 2, 3) if w.three_d else (0, 3, 1, 2)
    perm_y = (0, 2, 3, 4, 1) if w.three_d else (0, 2, 3, 1)
    conv = F.conv3d if w.three_d else F.conv2d

    def torch_step():
        t = nxt()
        yt[0] = conv(t["x"].permute(*perm_x), t["w"].permute(*perm_x), bias, padding=1).permute(*perm_y)
    step.comparator = (f"torch {conv.__name__} (cuDNN, fp16, channels-last)", torch_step, lambda: y, lambda: yt[0])

    hx, hw, hb = x.cpu().pin_memory(), wt.cpu().pin_memory(), bias.cpu().pin_memory()
    hy = torch.empty(plan.out_shape, dtype=torch.float16).pin_memory()

    def e2e_step():
        # Host buffers in and out through the host-buffer entry point (mm4_conv_run_host): weights and bias
        # first, then the images' copies in, convolutions and copies out pipelined over 16 chunks.
        plan.run_host(hx, hw, hb, hy, (x, wt, bias, y))
    return (step, e2e_step, ((x.numel() + wt.numel() + bias.numel()) * 2, y.numel() * 2), plan.kernel_name, 1,
            "strong", sets)


def run_mm4(args, w, dist, peaks):
    import torch
    from example_matmul_metal4_b200 import sync_check
    dev = torch.device("cuda", dist.local_rank)
    torch.cuda.set_device(dev)
    dist.init("nccl")
    stream = torch.cuda.current_stream()
    gen = torch.Generator(device=dev)
    gen.manual_seed(w.seed * 1000003 + dist.rank)
    builder = (build_gemm if isinstance(w, GemmWorkload) else
               build_attention_bwd if isinstance(w, AttentionBwdWorkload) else
               build_attention if isinstance(w, AttentionWorkload) else build_conv)
    step, e2e_step, e2e_bytes, kernel_name, launches, scaling, sets = builder(w, dist, dev, gen, args.l2)
    nsets = len(sets)
    if args.l2 == "rotate":
        check_rotation(w, dist, sets)
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=dev) if args.l2 == "flush" else None

    step()
    torch.cuda.synchronize()
    sync_check()

    clocks = ClockSampler(dist.local_rank)
    clocks.start()
    burn(step, flush, args.burn_seconds, dist)
    per_step = time_steps(step, args.steps, args.warmup, flush, stream, dist)
    burn(step, flush, args.burn_seconds / 2, dist)
    clk = clocks.stop()
    sync_check()
    ms = dist.max(sum(per_step) / len(per_step))

    # The ranks split one copy of the named shape (strong scaling): the whole job completes w.flops() per
    # step, in the slowest rank's time.
    units = 1 if scaling == "strong" else dist.world
    value = units * w.flops() / (ms * 1e-3) / 1e12

    launch_only = None
    if hasattr(step, "launch_only"):
        # `steps` launches from ONE call through the C ABI (duplicated_count, the reference's
        # duplicatedCount loop): the kernels without per-call host issue. One input copy is reused, so
        # L2 may hold part of it between launches.
        n = max(1, args.steps)
        step.launch_only(2)
        torch.cuda.synchronize()
        dist.barrier()
        s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if flush is not None:
            flush.zero_()
        s_ev.record(stream)
        step.launch_only(n)
        e_ev.record(stream)
        torch.cuda.synchronize()
        lo_ms = dist.max(s_ev.elapsed_time(e_ev) / n)
        launch_only = {"ms_per_launch": lo_ms, "launches_in_one_call": n,
                       "value": units * w.flops() / (lo_ms * 1e-3) / 1e12, "unit": "TFLOP/s"}

    e2e = None
    if e2e_step is not None:
        n_e2e = max(3, args.steps // 2)
        e2e_ms = dist.max(sum(time_steps(e2e_step, n_e2e, 2, flush, stream, dist)) / n_e2e)
        e2e = {"value": units * w.flops() / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": int(e2e_bytes[0]), "d2h_bytes_per_step": int(e2e_bytes[1])}
    comparator = None
    if dist.world == 1 and hasattr(step, "comparator") and not args.no_comparator:
        # B200 analogue of the reference's MPSGraph agreement check: the same op through torch
        # (cuBLAS / SDPA / cuDNN) on the same inputs, timed the same way, outputs compared.
        name, torch_step, ours, theirs = step.comparator
        torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False  # fp32 accumulation
        # Same thermal state as the mm4 arm: the same untimed burn before and after the timed steps, and
        # its own clock record (a long dense run settles at power-capped clocks; a cold one boosts).
        cmp_clocks = ClockSampler(dist.local_rank)
        cmp_clocks.start()
        burn(torch_step, flush, args.burn_seconds, dist)
        cmp_ms = sum(time_steps(torch_step, args.steps, args.warmup, flush, stream, dist)) / args.steps
        burn(torch_step, flush, args.burn_seconds / 2, dist)
        cmp_clk = cmp_clocks.stop()
        step()
        torch_step()  # every input copy holds the same values, so both outputs are comparable
        torch.cuda.synchronize()
        a, b = ours().float(), theirs().float()
        diff = (a - b).abs()
        comparator = {"impl": name, "ms_per_step": cmp_ms, "value": w.flops() / (cmp_ms * 1e-3) / 1e12,
                      "unit": "TFLOP/s", "max_abs_diff_vs_mm4": float(diff.max().item()),
                      "mismatches_vs_mm4": int((diff > 2e-2 + 1e-2 * b.abs()).sum().item()),
                      "clocks": cmp_clk}
    if hasattr(step, "close"):
        step.close()  # collective on every rank (peer mappings, exchange buffers)

    roof = None
    if dist.world == 1:
        if w.bound == "hbm":
            achieved, peak, unit = w.bytes() / (ms * 1e-3) / 1e9, peaks["hbm_gbs"], "GB/s"
        else:
            achieved, peak, unit = value, peaks["bf16_tflops"], "TFLOP/s"
        roof = {"bound": w.bound, "achieved": achieved, "peak": peak, "unit": unit, "frac": achieved / peak,
                "peak_source": ("measured, MEASURED_PEAKS.json (burst)" if peaks["source"] == "measured"
                                else "fallback"),
                "algorithmic_bytes": w.bytes(), "algorithmic_flops": w.flops(),
                "traffic": load_traffic(w.name), "kernel": kernel_name, "kernel_ms": ms}
    return dict(value=value, ms=ms, clocks=clk, e2e=e2e, roofline=roof, launches=launches * args.steps,
                kernel=kernel_name, scaling=scaling, nsets=nsets, comparator=comparator, launch_only=launch_only,
                shard=getattr(step, "shard", None))


# ---------------------------------------------------------------------------
# CPU legs (oracle = the reference's CPU loops restated in C)
# ---------------------------------------------------------------------------

def whole_rounds(rows, threads, total):
    """A row count for a sample on `threads` threads: a whole number of rows per thread, so that no thread
    idles at the end and the rate does not depend on how the last round splits (at most `total`)."""
    if total <= threads:
        return total
    return min(total // threads * threads, max(threads, rows // threads * threads))


def cpu_sample(w, seconds_hint=10.0, threads=None):
    """Times the oracle on a bounded sample of workload `w`, extrapolated to the full workload."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import numpy as np
    import oracle
    threads = threads or oracle.max_threads()
    rng = np.random.default_rng(12345)

    def timed(fn):
        t0 = time.perf_counter()
        fn()
        return time.perf_counter() - t0

    def h(shape, scale=1.0, uniform=False):
        if uniform:
            a = rng.uniform(-scale, scale, size=shape).astype(np.float32)
        else:
            a = rng.standard_normal(shape, dtype=np.float32) * scale
        return a.astype(np.float16)

    if isinstance(w, GemmWorkload):
        M, N, K = w.M, w.N, w.K
        A, B, bias = h((M, K), uniform=True), h((K, N), uniform=True), h((N,), uniform=True)
        # An untimed round of one row per thread warms the pages and threads and sizes the sample.
        one = timed(lambda: oracle.gemm(A, B, bias, M, N, K, rows=(0, min(M, threads)), threads=threads))
        rows = whole_rounds(int(seconds_hint / max(one, 1e-6)) * threads, threads, M)
        dt = timed(lambda: oracle.gemm(A, B, bias, M, N, K, rows=(0, rows), threads=threads))
        flops = 2.0 * rows * N * K
        sample = (f"{rows} of {M} output rows of the {M}x{N}x{K} GEMM+bias (fp32 loop of matmul.swift:499-510), "
                  f"{dt:.2f} s")
    elif isinstance(w, AttentionBwdWorkload):
        S, D = w.S, w.D
        H = threads  # one head per thread: a block of query rows of each, against all S keys
        Kt, V = h((1, H, S, D)), h((1, H, S, D))

        def run(rows, heads, nthreads):
            Qs, dOs = h((1, heads, rows, D)), h((1, heads, rows, D))
            return timed(lambda: oracle.attention_bwd(Qs, Kt[:, :heads].copy(), V[:, :heads].copy(), dOs, 1, heads,
                                                      heads, rows, S, D, 1 / math.sqrt(D), threads=nthreads))
        one = run(1, 1, 1)
        rows = max(1, min(S, int(seconds_hint / max(one, 1e-6))))
        dt = run(rows, H, threads)
        flops = 10.0 * H * rows * S * D
        sample = (f"{rows} query rows x {H} heads against S={S} keys, D={D} attention backward "
                  f"(Network.swift:181-401 restated), {dt:.2f} s")
    elif isinstance(w, AttentionWorkload):
        S, D = w.S, w.D
        H = threads  # one head per thread, a block of query rows of each
        Q, Kt, V = h((1, H, S, D)), h((1, H, S, D)), h((1, H, S, D))
        one = timed(lambda: oracle.attention(Q, Kt, V, 1, 1, 1, S, S, D, 1 / math.sqrt(D), rows=(0, 1), threads=1))
        rows = max(1, min(S, int(seconds_hint / max(one, 1e-6))))
        dt = timed(lambda: oracle.attention(Q, Kt, V, 1, H, H, S, S, D, 1 / math.sqrt(D), rows=(0, rows),
                                            threads=threads))
        flops = 4.0 * H * rows * S * D
        sample = (f"{rows} query rows x {H} heads of S={S}, D={D} attention (Network.swift:134-179, :286-311), "
                  f"{dt:.2f} s")
    else:
        b = np.zeros(w.O, dtype=np.float16)
        if w.three_d:
            x, wt = h((1, w.D, w.H, w.W, w.C)), h((w.O, 3, 3, 3, w.C), w.wsig)
            kw = dict(N=1, D=w.D, H=w.H, W=w.W, C=w.C, O=w.O, KD=3, KH=3, KW=3, pad_front=1, pad_back=1,
                      pad_top=1, pad_bottom=1, pad_left=1, pad_right=1, layout=4)
            total_rows, per_row_flops, fn = w.D * w.H, 2.0 * w.W * w.O * 27 * w.C, oracle.conv3d
        else:
            x, wt = h((1, w.H, w.W, w.C)), h((w.O, 3, 3, w.C), w.wsig)
            kw = dict(N=1, H=w.H, W=w.W, C=w.C, O=w.O, KH=3, KW=3, pad_top=1, pad_bottom=1, pad_left=1,
                      pad_right=1, layout=1)
            total_rows, per_row_flops, fn = w.H, 2.0 * w.W * w.O * 9 * w.C, oracle.conv2d
        one = timed(lambda: fn(x, wt, b, rows=(0, min(total_rows, threads)), threads=threads, **kw))
        rows = whole_rounds(int(seconds_hint / max(one, 1e-6)) * threads, threads, total_rows)
        dt = timed(lambda: fn(x, wt, b, rows=(0, rows), threads=threads, **kw))
        flops = per_row_flops * rows
        sample = (f"{rows} output rows ({w.W} pixels x {w.O} channels each) of one image of the {w.name} conv "
                  f"(ConvolutionShared.swift:4994-5096), {dt:.2f} s")
    return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": sample + "; the sample's rate stands for the full workload"}


# ---------------------------------------------------------------------------
# main
# ---------------------------------------------------------------------------

def parallelism(w, n):
    """How N GPUs split the named shape (the same text on both arms)."""
    if n == 1:
        return "single GPU"
    if isinstance(w, GemmWorkload) and w.split > 1:
        return (f"{n} K shards of K = {w.K} on 64-element boundaries, split-K {shard_splits(w, n)} within each "
                "shard (every split at least 512 deep); fp32 "
                "partials summed inside the split-K kernels over peer memory (NVLink) into rank 0's C; one launch "
                "per GPU per step")
    axis = ("(batch, head) units" if isinstance(w, AttentionWorkload) else
            "C column blocks (A replicated)" if isinstance(w, GemmWorkload) else "batch")
    return f"{n} shards of one named shape along {axis}, no collective"


def rotated_input_bytes(w, n, rank=0):
    """Bytes of the device inputs a step of rank `rank` reads and rotation copies (see the builders)."""
    if isinstance(w, GemmWorkload):
        if n > 1 and w.split > 1:
            k = shard_range(w.K, n, rank, align=64)[1]
            return 2 * (w.M * k + k * w.N)
        cols = shard_range(w.N, n, rank, align=8)[1]
        return 2 * (w.M * w.K + w.K * cols)
    if isinstance(w, AttentionWorkload):
        nb, nh = w.shard(n, rank)
        per = nb * nh * w.S * w.D * 2
        if isinstance(w, AttentionBwdWorkload):
            return 5 * per + nb * nh * w.S * 4  # Q, K, V, O, dO and the fp32 LSE
        return 3 * per
    nb = shard_range(w.N, n, rank)[1]
    return 2 * (nb * w.D * w.H * w.W * w.C + w.O * w.taps() * w.C)


def rotate_copies(w, n):
    """Device copies of rank 0's inputs that input_sets() makes when rotating (the same rule)."""
    return max(2, 1 + math.ceil(2 * L2_BYTES / rotated_input_bytes(w, n)))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="attention", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="mm4", choices=["mm4", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-comparator", action="store_true", help="skip the torch (cuBLAS/SDPA/cuDNN) comparator")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--burn-seconds", type=float, default=0.6,
                    help="untimed repetitions of the step before (and half as long after) the timed steps, so they "
                         "run at the clocks a sustained run settles at; small values keep profiler captures short")
    ap.add_argument("--l2", default="auto", choices=["auto", "rotate", "flush"],
                    help="keep inputs out of L2 by rotating device copies of them or by a 512 MiB write between "
                         "steps; auto: rotate for HBM-bound and small workloads (a write flush leaves ~126 MB of "
                         "dirty lines whose write-back would land inside the timed kernel), flush for the rest")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    w = WORKLOADS[args.workload]()
    if args.l2 == "auto":
        # Rotate for HBM-bound workloads and for small ones: the write flush leaves ~126 MB of dirty
        # L2 lines whose write-back (~20 us) lands inside the next timed kernel.
        args.l2 = "rotate" if (w.bound == "hbm" or w.bytes() < L2_BYTES / 4) else "flush"
    dist = Dist(args.gpus)
    peaks = load_peaks()
    base = {"metric": METRIC, "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "vs_baseline": None, "dtype": "fp16 (fp32 accumulate)",
            "data": "synthetic (seeded torch generator; BASELINE shapes and distributions)"}
    # The workload's configuration, identical on both arms (the reference arm runs the same named shape on
    # the host, where the L2 handling does not apply).
    cfg = dict(w.config(), l2="flushed between steps (512 MiB write outside the timed events)",
               baseline_config_index=w.config_index, parallelism=parallelism(w, args.gpus))
    if args.l2 == "rotate":
        cfg["l2"] = (f"inputs larger than L2: each step reads the next of {rotate_copies(w, args.gpus)} device "
                     "copies of its inputs, so at least 2 x 126 MB of other inputs pass through L2 between two "
                     "uses of a copy; no flush")

    if args.impl == "reference":
        if dist.rank != 0:
            return
        vals, cb = [], None
        per_step = max(1.0, min(8.0, 120.0 / (args.warmup + args.steps)))
        for i in range(args.warmup + args.steps):
            cb = cpu_sample(w, seconds_hint=per_step if i >= args.warmup else 0.5)
            if i >= args.warmup:
                vals.append(cb["value"])
        value = statistics.mean(vals)
        line = dict(base, impl="reference", value=value, ms_per_step=w.flops() / (value * 1e12) * 1e3,
                    scaling="strong", config=cfg, kernel="C restatement of the reference's CPU loops (host)",
                    cpu_baseline={"value": value, "unit": "TFLOP/s", "cores": cb["cores"], "kind": "port",
                                  "sample": cb["sample"]},
                    e2e={"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
                    gpu_launches=0)
        print(json.dumps(line), flush=True)
        return

    res = run_mm4(args, w, dist, peaks)
    if dist.rank == 0:
        cpu = None
        if args.gpus == 1 and not args.no_cpu_baseline:
            cpu = cpu_sample(w, seconds_hint=args.cpu_seconds)
            # The reference's own CPU check runs single-threaded; time that too on a smaller sample.
            one = cpu_sample(w, seconds_hint=max(1.0, args.cpu_seconds / 4), threads=1)
            cpu["single_thread"] = {"value": one["value"], "unit": one["unit"], "cores": 1, "sample": one["sample"]}
        line = dict(base, value=res["value"], ms_per_step=res["ms"], scaling=res["scaling"], config=cfg,
                    kernel=res["kernel"], shard_of_rank0=res["shard"],
                    pct_of_measured_bf16_peak=res["value"] / args.gpus / peaks["bf16_tflops"],
                    clocks=res["clocks"], e2e=res["e2e"], roofline=res["roofline"], cpu_baseline=cpu,
                    gpu_launches=res["launches"], launch_only=res["launch_only"], comparator=res["comparator"])
        print(json.dumps(line), flush=True)
    dist.close()


if __name__ == "__main__":
    main()
