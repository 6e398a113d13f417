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


class _DeviceArray:
    """__cuda_array_interface__ over a raw device pointer (for a zero-copy torch view)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": tuple(shape), "typestr": typestr,
                                         "strides": None, "version": 3}


class SplitKGroup:
    """Fused multi-GPU split-K GEMM (mm4_gemm_splitk_group_run): every rank runs `plan` on its own K
    shard and the ranks' fp32 partials are summed inside the kernels over peer memory (CUDA IPC
    mappings over NVLink) into the root's C: one launch per GPU, no separate collective.

    Construction is collective (every rank of the default process group, same plan shape): each rank
    allocates its exchange buffer, the root also its C, and the handles are exchanged with
    all_gather_object / broadcast_object_list. `C` is the root's [M][N] fp16 output (None elsewhere);
    after `run` returns on the root's stream, the root's later work on that stream sees all of C.
    Every rank must call `run` the same number of times. Call `close()` on every rank when done."""

    def __init__(self, plan, root: int = 0):
        import ctypes

        import torch
        import torch.distributed as dist

        from . import _lib
        L = _lib.lib()
        self._L, self._lib, self.plan, self.root = L, _lib, plan, root
        self.world = dist.get_world_size() if dist.is_initialized() else 1
        self.rank = dist.get_rank() if dist.is_initialized() else 0
        M, N = plan.dims.M, plan.dims.N
        nbytes = ctypes.c_size_t()
        _lib.check(L.mm4_splitk_group_exchange_bytes(plan._h, self.world, ctypes.byref(nbytes)))
        self._own, self._c_own, self._opened, self._g = ctypes.c_void_p(), None, [], None
        h, hc = _lib.PeerHandle(), _lib.PeerHandle()
        _lib.check(L.mm4_peer_alloc(nbytes.value, ctypes.byref(self._own), ctypes.byref(h)))
        if self.rank == root:
            self._c_own = ctypes.c_void_p()
            _lib.check(L.mm4_peer_alloc(M * N * 2, ctypes.byref(self._c_own), ctypes.byref(hc)))
        handles = [bytes(h.bytes)]
        c_handle = bytes(hc.bytes)
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(h.bytes))
            obj = [c_handle if self.rank == root else None]
            dist.broadcast_object_list(obj, src=root)
            c_handle = obj[0]
        ptrs = (ctypes.c_void_p * self.world)()
        for r in range(self.world):
            if r == self.rank:
                ptrs[r] = self._own.value
            else:
                ptrs[r] = self._open(handles[r]).value
        c_root = self._c_own if self.rank == root else self._open(c_handle)
        g = ctypes.c_void_p()
        _lib.check(L.mm4_splitk_group_create(ctypes.byref(g), plan._h, self.world, self.rank, root, ptrs, c_root))
        self._g = g
        self.C = None
        if self.rank == root:
            self.C = torch.as_tensor(_DeviceArray(self._c_own.value, (M, N), "<f2"), device="cuda")

    def _open(self, handle_bytes):
        import ctypes
        ph = self._lib.PeerHandle.from_buffer_copy(handle_bytes)
        p = ctypes.c_void_p()
        self._lib.check(self._L.mm4_peer_open(ctypes.byref(ph), ctypes.byref(p)))
        self._opened.append(p)
        return p

    def run(self, A, B, bias=None, stream=None):
        """One fused step: this rank's K shard (A [M][K_r], B [K_r][N], fp16) into the root's C. The
        group owns its split-K scratch (in the exchange buffers), so no workspace is passed."""
        from .gemm import _check_tensor
        _check_tensor(A, self.plan.a_shape(), "A")
        _check_tensor(B, self.plan.b_shape(), "B")
        if self.plan.bias:
            _check_tensor(bias, (self.plan.dims.N,), "bias")
        self._lib.check(self._L.mm4_gemm_splitk_group_run(
            self.plan._h, self._g, A.data_ptr(), B.data_ptr(), bias.data_ptr() if self.plan.bias else None,
            self._lib.stream_handle(stream)))
        return self.C

    def close(self):
        """Collective: releases the group, the peer mappings and this rank's buffers."""
        import torch
        import torch.distributed as dist
        if self._g is None:
            return
        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier()  # no rank still runs a kernel that maps our buffers
        self._L.mm4_splitk_group_destroy(self._g)
        self._g = None
        self.C = None
        for p in self._opened:
            self._L.mm4_peer_close(p)
        self._opened = []
        if self.world > 1:
            dist.barrier()  # every rank has unmapped before the owners free
        self._L.mm4_peer_free(self._own)
        if self._c_own is not None:
            self._L.mm4_peer_free(self._c_own)


class Comm:
    """NCCL-bootstrapped communicator for the fused multi-GPU split-K (mm4_comm_init +
    mm4_gemm_splitk_run_distributed): the C-ABI form a caller with an NCCL unique id binds. NCCL
    only exchanges the exchange-buffer handles at set-up; every run is one fused launch per GPU."""

    def __init__(self, nranks: int, rank: int, unique_id: bytes):
        import ctypes

        from . import _lib
        self._lib, self._L = _lib, _lib.lib()
        self.nranks, self.rank = nranks, rank
        buf = ctypes.create_string_buffer(bytes(unique_id), 128)
        h = ctypes.c_void_p()
        _lib.check(self._L.mm4_comm_init(ctypes.byref(h), nranks, rank, buf))
        self._h = h

    @staticmethod
    def unique_id() -> bytes:
        import ctypes

        from . import _lib
        buf = ctypes.create_string_buffer(128)
        _lib.check(_lib.lib().mm4_comm_unique_id(buf))
        return buf.raw

    @classmethod
    def from_torch(cls):
        """Collective over the default torch.distributed group: rank 0 makes the id, all ranks join."""
        import torch.distributed as dist
        obj = [cls.unique_id() if dist.get_rank() == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        return cls(dist.get_world_size(), dist.get_rank(), obj[0])

    def run(self, plan, A, B, bias=None, C=None, stream=None, duplicatedCount: int = 1):
        """This rank's K shard of `plan` into rank 0's C (first call per plan is collective)."""
        import torch

        from .gemm import _check_tensor
        _check_tensor(A, plan.a_shape(), "A")
        _check_tensor(B, plan.b_shape(), "B")
        if plan.bias:
            _check_tensor(bias, (plan.dims.N,), "bias")
        if self.rank == 0 and C is None:
            C = torch.empty((plan.dims.M, plan.dims.N), dtype=torch.float16, device=A.device)
        self._lib.check(self._L.mm4_gemm_splitk_run_distributed(
            plan._h, self._h, A.data_ptr(), B.data_ptr(), bias.data_ptr() if plan.bias else None,
            C.data_ptr() if C is not None else None, self._lib.stream_handle(stream), int(duplicatedCount)))
        return C

    def close(self):
        """Collective: releases the communicator and every plan's group."""
        if self._h is not None:
            self._L.mm4_comm_destroy(self._h)
            self._h = None
