"""Multi-GPU partitioning of the contraction path (one process per GPU).

The path shards naturally (no collective) except split-K, whose K shards
meet in one fp32 reduction:

- GEMM: N-column blocks; attention: batch x heads; conv: batch.
- split-K GEMM: rank r owns K[k_shard(K, P, r)], computes an fp32 [M][N]
  partial (mm4_gemm_partial_run), the partials are summed over NCCL, and the
  destination rank adds bias and rounds to fp16 (mm4_splitk_finalize).
"""
from __future__ import annotations


def shard(n: int, parts: int, index: int) -> tuple[int, int]:
    """[begin, end) of part `index` of `n` items split as evenly as possible."""
    if parts <= 0 or not 0 <= index < parts:
        raise ValueError("bad shard request")
    return (n * index) // parts, (n * (index + 1)) // parts


def k_shard(K: int, world: int, rank: int, align: int = 8) -> tuple[int, int]:
    """K range of `rank`; boundaries rounded to `align` elements so every
    shard's A/B row pitch stays 16-byte aligned for TMA (the last shard takes
    the tail, e.g. K = 65520 over 8 ranks)."""
    k0, k1 = shard(K, world, rank)
    k0 = (k0 // align) * align if rank > 0 else 0
    k1 = K if rank == world - 1 else (k1 // align) * align
    return k0, k1


def splitk_per_rank(split_k: int, world: int) -> int:
    """In-kernel split count per rank, keeping the total number of K
    partitions at the requested split_k."""
    return max(1, split_k // world)


def reduce_partials(partial, dst: int = 0, group=None, async_op: bool = False):
    """Sums the fp32 K-shard partials of all ranks into `partial` on `dst`."""
    import torch.distributed as dist
    return dist.reduce(partial, dst=dst, op=dist.ReduceOp.SUM, group=group, async_op=async_op)


class RankLost(RuntimeError):
    """A rank did not reach a step: raised on the host before any collective of that step."""

    def __init__(self, step: int, missing: list[int]):
        super().__init__(f"ranks {missing} did not reach step {step}")
        self.step = step
        self.missing = missing


class StepHeartbeat:
    """Host-side liveness check between steps, over a c10d store.

    Before launching step `s` (its kernels and collectives) every rank calls
    `beat(s)`: it posts its own key for `s` and waits at most `timeout`
    seconds for every other rank's. A rank that left between steps is
    reported as RankLost on the survivors before they launch anything, so no
    collective is left waiting on a missing peer and no GPU work is in
    flight when the error surfaces."""

    def __init__(self, store, rank: int, world: int, timeout: float = 5.0, prefix: str = "mm4/hb"):
        self.store, self.rank, self.world, self.timeout, self.prefix = store, rank, world, timeout, prefix

    def _key(self, step: int, rank: int) -> str:
        return f"{self.prefix}/{step}/{rank}"

    def beat(self, step: int) -> None:
        import time
        self.store.set(self._key(step, self.rank), "1")
        waiting = [r for r in range(self.world) if r != self.rank]
        deadline = time.monotonic() + self.timeout
        # Poll with check() (non-blocking) rather than a store wait with a
        # timeout: a wait that runs out can leave the client connection
        # unusable for the report that follows.
        while waiting:
            waiting = [r for r in waiting if not self.store.check([self._key(step, r)])]
            if not waiting:
                return
            if time.monotonic() > deadline:
                raise RankLost(step, waiting)
            time.sleep(0.002)
