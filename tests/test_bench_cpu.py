"""bench.py's output contract, checked on the CPU: the reference arm prints one
JSON line with every key the driver reads, the mm4 arm fails loudly when no
GPU is present (no silent CPU fallback), and every workload's accounting is
well formed."""
import json
import math
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _no_gpu():
    import torch
    return not torch.cuda.is_available()


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "3", "--workload", "gemm1024"],
                       capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e", "gpu_launches"):
        assert key in d, key
    assert d["impl"] == "reference"
    assert d["steps"] == 1 and d["warmup"] >= 3 and d["n_gpus"] == 1
    assert d["value"] > 0 and math.isclose(d["cpu_baseline"]["value"], d["value"])
    assert d["config"]["workload"] == "gemm_bias_1024x1024x1024_nn"
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1 and d["cpu_baseline"]["sample"]
    assert d["e2e"]["unit"] == d["unit"] and d["e2e"]["h2d_bytes_per_step"] == 0
    assert d["e2e"]["d2h_bytes_per_step"] == 0


@pytest.mark.skipif(not _no_gpu(), reason="checks the no-GPU failure")
def test_mm4_arm_fails_loudly_without_a_gpu():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--steps", "1", "--warmup", "3"],
                       capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert r.returncode != 0
    assert not r.stdout.strip(), "no JSON line may be printed without a GPU"


def test_workload_accounting():
    sys.path.insert(0, str(ROOT))
    import bench
    for name, make in bench.WORKLOADS.items():
        w = make()
        cfg = w.config()
        assert cfg["workload"] == w.name, name
        assert w.flops() > 0 and w.bytes() > 0, name
        assert w.bound in ("hbm", "tensor"), name
    # the split-K default is HBM-bound (arithmetic intensity below the ridge), the rest tensor-bound
    assert bench.WORKLOADS["splitk"]().bound == "hbm"
    att, bwd = bench.WORKLOADS["attention"](), bench.WORKLOADS["attention_bwd"]()
    assert bwd.flops() == 2.5 * att.flops()


def test_strong_scaling_shards_cover_each_named_shape_once():
    """The N>1 shards split ONE copy of each named shape: K shards on 64-element boundaries for split-K
    (65536 -> 8 x 8192, 65520 -> 7 x 8192 + 8176), C column blocks for the GEMMs, the 64 (batch, head)
    units for attention, the batch for conv."""
    sys.path.insert(0, str(ROOT))
    import bench
    assert [bench.shard_range(65536, 8, r, 64) for r in range(8)] == [(8192 * r, 8192) for r in range(8)]
    assert [bench.shard_range(65520, 8, r, 64)[1] for r in range(8)] == [8192] * 7 + [8176]
    att = bench.WORKLOADS["attention"]()
    for parts in (1, 2, 3, 4, 5, 8):
        for total, align in ((65536, 64), (65520, 64), (1024, 8), (8192, 8), (32, 1), (8, 1), (64, 1)):
            ranges = [bench.shard_range(total, parts, r, align) for r in range(parts)]
            assert sum(c for _, c in ranges) == total
            assert all(s == (ranges[i - 1][0] + ranges[i - 1][1]) for i, (s, _) in enumerate(ranges) if i)
            assert all(s % align == 0 for s, _ in ranges)
        units = 0
        for r in range(parts):
            nb, nh = att.shard(parts, r)
            units += nb * nh
        assert units == att.B * att.H
    assert att.shard(2, 1) == (2, 16) and att.shard(8, 3) == (1, 8)


def test_cpu_sample_rows_are_whole_rounds_per_thread():
    """The CPU baseline's row samples give every thread the same number of rows (no idle thread in the
    last round), and never exceed the workload."""
    sys.path.insert(0, str(ROOT))
    import bench
    assert bench.whole_rounds(198, 16, 512) == 192
    assert bench.whole_rounds(5, 16, 512) == 16
    assert bench.whole_rounds(10**6, 16, 512) == 512
    assert bench.whole_rounds(100, 16, 56) == 48
    assert bench.whole_rounds(100, 16, 10) == 10
