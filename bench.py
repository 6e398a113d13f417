#!/usr/bin/env python
"""Benchmark of the mm4 tensor-op contraction path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl mm4|reference]

Prints ONE JSON line (rank 0). A "step" is one pass of the hot path over
one batch of synthetic input:

  splitk (default)  BASELINE configs[1]: C = A*B + bias, M=N=512, K=65536,
                    split-K 32, fp32 partials reduced in-kernel, fp16 out.
                    N>1: K is sharded over ranks; every rank computes its fp32
                    partial, the partials are summed with an NCCL reduce over
                    NVLink and rank 0 adds bias and rounds (strong scaling).
  gemm1024          BASELINE configs[0] (1024^3 GEMM+bias, NN).
  gemm8192          the north-star target shape 8192^3 GEMM+bias, NN.
  attention, conv2d, conv3d   BASELINE configs[2..4] (when built).

Timing: W untimed warm-up steps, then K timed steps, each bracketed by CUDA
events on the launching stream, with a 512 MiB write between steps to flush
L2 (126 MB) outside the events. Barrier + synchronize on both sides; the
reported time is the max over ranks.

`--impl reference` times the reference's CPU implementation of the path (the
C restatement of its Swift validation loops, oracle/) on the host cores, on a
bounded sample of the same workload, extrapolated to the full workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PEAKS_FILE = ROOT / "MEASURED_PEAKS.json"
TRAFFIC_FILE = ROOT / "profiles" / "dram_traffic.json"

# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------

WORKLOADS = {
    "splitk": dict(kind="gemm", M=512, N=512, K=65536, split=32, seed=2, bound="hbm",
                   name="splitk_gemm_bias_512x512x65536_s32_nn", config_index=1),
    "splitk65520": dict(kind="gemm", M=512, N=512, K=65520, split=32, seed=2, bound="hbm",
                        name="splitk_gemm_bias_512x512x65520_s32_nn", config_index=1),
    "gemm1024": dict(kind="gemm", M=1024, N=1024, K=1024, split=1, seed=1, bound="tensor",
                     name="gemm_bias_1024x1024x1024_nn", config_index=0),
    "gemm8192": dict(kind="gemm", M=8192, N=8192, K=8192, split=1, seed=11, bound="tensor",
                     name="gemm_bias_8192x8192x8192_nn", config_index=None),
}


def gemm_flops(w):
    return 2.0 * w["M"] * w["N"] * w["K"]


def gemm_bytes(w):
    # algorithmic: A + B + bias read once, C written once (fp16); the split-K
    # fp32 workspace is not algorithmic traffic.
    return 2.0 * (w["M"] * w["K"] + w["K"] * w["N"] + w["N"] + w["M"] * w["N"])


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
            dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=120))
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, value):
        if not self.pg:
            return value
        import torch
        t = torch.tensor([value], dtype=torch.float64, device="cuda" if torch.cuda.is_available() else "cpu")
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
        reasons = set()
        for r in rows:
            for key, name in (("hw", "hw_slowdown"), ("hw_thermal", "hw_thermal_slowdown"),
                              ("sw_thermal", "sw_thermal_slowdown"), ("sw_power", "sw_power_cap")):
                if r[key].lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r["sm"] for r in rows), "sm_max_mhz": max(r["max"] for r in rows),
                "power_w_max": max(r["power"] for r in rows), "samples": len(rows), "reasons": sorted(reasons)}


# ---------------------------------------------------------------------------
# inputs
# ---------------------------------------------------------------------------

def gemm_inputs(w, tl=False, tr=False):
    """Seeded U[-1,1] fp16 A[M][K], B[K][N], bias[N]."""
    from example_matmul_metal4_b200 import data
    A = data.uniform((w["M"], w["K"]), -1.0, 1.0, w["seed"], 0)
    B = data.uniform((w["K"], w["N"]), -1.0, 1.0, w["seed"], 1)
    bias = data.uniform((w["N"],), -1.0, 1.0, w["seed"], 2)
    return A, B, bias


# ---------------------------------------------------------------------------
# mm4 arm
# ---------------------------------------------------------------------------

def time_steps(step, steps, warmup, flush, stream, dist):
    """Per-step CUDA events on `stream`; L2 flush between steps outside events."""
    import torch
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    events = []
    for _ in range(steps):
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
    per_step = [s.elapsed_time(e) for s, e in events]
    return per_step


def burn(step, flush, seconds):
    """Repeats the step (with L2 flushes) for about `seconds`, untimed."""
    import torch
    t_end = time.perf_counter() + seconds
    while time.perf_counter() < t_end:
        for _ in range(8):
            flush.zero_()
            step()
        torch.cuda.synchronize()


def run_gemm_mm4(args, w, dist, peaks):
    import torch
    from example_matmul_metal4_b200 import BuildOptions, GEMMDimensions, GemmPlan, lib, sync_check
    from example_matmul_metal4_b200.gemm import splitk_finalize

    dev = torch.device("cuda", dist.local_rank)
    torch.cuda.set_device(dev)
    dist.init("nccl")
    stream = torch.cuda.current_stream()
    A, B, bias = gemm_inputs(w)
    M, N, K = w["M"], w["N"], w["K"]
    P, r = dist.world, dist.rank
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=dev)
    launches_per_step = 1

    if P == 1:
        plan = GemmPlan(GEMMDimensions(M, N, K), transpose=(False, False), bias=True,
                        buildOptions=BuildOptions(splitK=w["split"]))
        tA, tB, tb = (torch.from_numpy(x).to(dev) for x in (A, B, bias))
        C = torch.empty((M, N), dtype=torch.float16, device=dev)
        ws = plan.workspace(dev)

        def step():
            plan.run(tA, tB, tb, C=C, workspace=ws)
        kernel_name = plan.kernel_name
    else:
        if w["split"] <= 1:
            # N-column shards, no collective (weak in N: every rank owns N columns).
            plan = GemmPlan(GEMMDimensions(M, N, K), transpose=(False, False), bias=True,
                            buildOptions=BuildOptions(splitK=1))
            tA, tB, tb = (torch.from_numpy(x).to(dev) for x in (A, B, bias))
            C = torch.empty((M, N), dtype=torch.float16, device=dev)

            def step():
                plan.run(tA, tB, tb, C=C)
            kernel_name = plan.kernel_name
        else:
            # K shards + fp32 NCCL reduce to rank 0 + bias/cast on rank 0.
            k0, k1 = (K * r) // P, (K * (r + 1)) // P
            shard_split = max(1, w["split"] // P)
            plan = GemmPlan(GEMMDimensions(M, N, k1 - k0), transpose=(False, False), bias=False,
                            buildOptions=BuildOptions(splitK=shard_split))
            tA = torch.from_numpy(A[:, k0:k1].copy()).to(dev)
            tB = torch.from_numpy(B[k0:k1].copy()).to(dev)
            tb = torch.from_numpy(bias).to(dev)
            C32 = torch.empty((M, N), dtype=torch.float32, device=dev)
            C = torch.empty((M, N), dtype=torch.float16, device=dev)
            ws = plan.workspace(dev)
            import torch.distributed as tdist

            def step():
                plan.partial(tA, tB, C32=C32, workspace=ws)
                tdist.reduce(C32, dst=0, op=tdist.ReduceOp.SUM)
                if r == 0:
                    splitk_finalize(C32, tb, C=C)
            launches_per_step = 2 if r == 0 else 1
            kernel_name = plan.kernel_name + "+nccl_reduce+finalize"

    # correctness spot-check outside timing (rank 0 full output vs fp32 cuBLAS)
    step()
    torch.cuda.synchronize()
    sync_check()

    clocks = ClockSampler(dist.local_rank)
    clocks.start()
    burn(step, flush, 0.6)  # load the GPU so the sampler sees clocks under load
    per_step = time_steps(step, args.steps, args.warmup, flush, stream, dist)
    burn(step, flush, 0.3)
    clk = clocks.stop()
    ms = dist.max(sum(per_step) / len(per_step))

    flops = gemm_flops(w)
    value = flops / (ms * 1e-3) / 1e12  # whole-job TFLOP/s (one problem per step across all ranks)

    # e2e through the public API from pinned host buffers (rank 0, single GPU)
    e2e = None
    if P == 1:
        hA = torch.from_numpy(A).pin_memory()
        hB = torch.from_numpy(B).pin_memory()
        hb = torch.from_numpy(bias).pin_memory()
        hC = torch.empty((M, N), dtype=torch.float16).pin_memory()

        def e2e_step():
            tA.copy_(hA, non_blocking=True)
            tB.copy_(hB, non_blocking=True)
            tb.copy_(hb, non_blocking=True)
            plan.run(tA, tB, tb, C=C, workspace=ws)
            hC.copy_(C, non_blocking=True)
        e2e_ms = sum(time_steps(e2e_step, max(3, args.steps // 2), 2, flush, stream, dist)) / max(3, args.steps // 2)
        h2d = A.nbytes + B.nbytes + bias.nbytes
        e2e = {"value": flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(M * N * 2)}

    roof = None
    if P == 1:
        if w["bound"] == "hbm":
            achieved = gemm_bytes(w) / (ms * 1e-3) / 1e9
            peak = peaks["hbm_gbs"]
            unit = "GB/s"
        else:
            achieved = value
            peak = peaks["bf16_tflops"]
            unit = "TFLOP/s"
        roof = {"bound": w["bound"], "achieved": achieved, "peak": peak, "unit": unit, "frac": achieved / peak,
                "peak_source": f"{peaks['source']} (MEASURED_PEAKS.json)" if peaks["source"] == "measured"
                else "fallback", "algorithmic_bytes": gemm_bytes(w), "algorithmic_flops": flops,
                "traffic": load_traffic(w["name"]), "kernel": kernel_name}
    return dict(value=value, ms=ms, clocks=clk, e2e=e2e, roofline=roof, launches=launches_per_step * args.steps,
                kernel=kernel_name, flops=flops, pct_of_bf16_peak=value / peaks["bf16_tflops"])


# ---------------------------------------------------------------------------
# CPU baseline (the reference's CPU loops, restated in oracle/)
# ---------------------------------------------------------------------------

def cpu_gemm_sample(w, seconds_hint=10.0, threads=None):
    """Times the oracle on a bounded row sample and extrapolates to the full GEMM."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle
    threads = threads or oracle.max_threads()
    A, B, bias = gemm_inputs(w)
    M, N, K = w["M"], w["N"], w["K"]
    # calibrate with one row, then size the sample to ~seconds_hint
    t0 = time.perf_counter()
    oracle.gemm(A, B, bias, M, N, K, False, False, rows=(0, 1), threads=1)
    one_row = time.perf_counter() - t0
    rows = int(max(threads, min(M, seconds_hint * threads / max(one_row, 1e-6))))
    rows = max(1, min(M, (rows // threads) * threads or threads))
    t0 = time.perf_counter()
    oracle.gemm(A, B, bias, M, N, K, False, False, rows=(0, rows), threads=threads)
    dt = time.perf_counter() - t0
    flops = 2.0 * rows * N * K
    return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{rows} of {M} output rows of the {M}x{N}x{K} GEMM+bias (fp32 loop of matmul.swift:499-510), "
                      f"{dt:.2f} s, extrapolated linearly"}


# ---------------------------------------------------------------------------
# main
# ---------------------------------------------------------------------------

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="splitk", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="mm4", choices=["mm4", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    w = WORKLOADS[args.workload]
    dist = Dist(args.gpus)
    peaks = load_peaks()

    base = {"metric": "TFLOP/s per GPU & % of fp16 tensor peak (GEMM/attn/conv)", "unit": "TFLOP/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "vs_baseline": None, "dtype": "fp16 (fp32 accumulate)", "data": "synthetic (seeded Philox, U[-1,1])"}

    if args.impl == "reference":
        if dist.rank != 0:
            return
        cores = None
        vals = []
        sample = None
        for i in range(args.warmup + args.steps):
            cb = cpu_gemm_sample(w, seconds_hint=2.0 if i >= args.warmup else 0.5, threads=cores)
            cores = cb["cores"]
            sample = cb["sample"]
            if i >= args.warmup:
                vals.append(cb["value"])
        value = statistics.mean(vals)
        line = dict(base, impl="reference", value=value, ms_per_step=gemm_flops(w) / (value * 1e12) * 1e3,
                    scaling="strong", config={"workload": w["name"], "M": w["M"], "N": w["N"], "K": w["K"],
                                              "split_k": w["split"], "l2": "n/a (CPU)"},
                    cpu_baseline={"value": value, "unit": "TFLOP/s", "cores": cores, "kind": "port", "sample": sample},
                    e2e={"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
                    gpu_launches=0)
        print(json.dumps(line), flush=True)
        return

    res = run_gemm_mm4(args, w, dist, peaks)
    if dist.rank == 0:
        cpu = None
        if args.gpus == 1 and not args.no_cpu_baseline:
            cpu = cpu_gemm_sample(w, seconds_hint=10.0)
        line = dict(base, value=res["value"], ms_per_step=res["ms"],
                    scaling="strong" if (args.gpus > 1 and w["split"] > 1) else "weak",
                    config={"workload": w["name"], "M": w["M"], "N": w["N"], "K": w["K"], "split_k": w["split"],
                            "layout": "row-major NN (A[M][K], B[K][N])", "bias": True,
                            "l2": "flushed between steps (512 MiB write outside the timed events)",
                            "kernel": res["kernel"],
                            "parallelism": ("K-shard + NCCL fp32 reduce" if w["split"] > 1 else "N-column shards")
                            if args.gpus > 1 else "single GPU"},
                    pct_of_measured_bf16_peak=res["pct_of_bf16_peak"],
                    clocks=res["clocks"], e2e=res["e2e"], roofline=res["roofline"], cpu_baseline=cpu,
                    gpu_launches=res["launches"])
        print(json.dumps(line), flush=True)
    dist.close()


if __name__ == "__main__":
    main()
