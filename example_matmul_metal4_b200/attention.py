"""Attention host interface: the reference's attention descriptors on the mm4 C ABI.

Mirrors Sources/attention/attention.swift: `AttentionDimensions(R, C, K, Hq,
Hk)` (:15-21; R = query rows, C = key/value rows, K = head dimension),
`BlockDimenions` / `BuildOptions` (:4-13; accepted as tuning hints), and
createSource + run(...) (:23-382, :398-541) as `AttentionPlan`. Tensors are
fp16 torch CUDA tensors in [B][H][S][D] (BHSD) or [B][S][H][D] (BSHD, the
reference's [S][H][D] packing with batch outermost).
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

from . import _lib
from ._lib import MM4_ATTN_BHSD, MM4_ATTN_BSHD  # noqa: F401


@dataclass
class AttentionDimensions:
    R: int
    C: int
    K: int
    Hq: int
    Hk: int


@dataclass
class BlockDimenions:  # (sic) the reference's spelling, attention.swift:9
    R: int = 128
    C: int = 128
    K: int = 128


@dataclass
class BuildOptions:
    executionSIMDGroups: int = 4
    bypassThreadgroupMemory: bool = True


class AttentionPlan:
    """Non-causal flash attention for one (batch, dims, layout): the forward (`run`, optionally with the
    per-row log-sum-exp) and the backward (`backward`: dQ, dK, dV of the loss sum(dO * O), the GPU form of
    Network.swift derivativeQ / derivativeK / derivativeV, :328-401)."""

    def __init__(self, dims: AttentionDimensions, batch: int = 1, layout: int = MM4_ATTN_BHSD,
                 scale: float | None = None, blockDimensions: BlockDimenions | None = None,
                 buildOptions: BuildOptions | None = None):
        self._L = _lib.lib()
        self.dims = dims
        self.batch = batch
        self.layout = layout
        self.scale = scale if scale is not None else 1.0 / math.sqrt(dims.K)
        d = _lib.AttentionDesc(batch, dims.Hq, dims.Hk, dims.R, dims.C, dims.K, float(self.scale), layout)
        h = ctypes.c_void_p()
        _lib.check(self._L.mm4_attention_plan_create(ctypes.byref(h), ctypes.byref(d)))
        self._h = h
        self.kernel_name = self._L.mm4_attention_plan_kernel_name(h).decode()

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            self._L.mm4_attention_plan_destroy(h)
            self._h = None

    def shape(self, rows: int, heads: int):
        if self.layout == MM4_ATTN_BHSD:
            return (self.batch, heads, rows, self.dims.K)
        return (self.batch, rows, heads, self.dims.K)

    def flops(self) -> float:
        """4*B*Hq*R*C*D (two GEMMs); the reference counts (2D+5)*S^2*H (attention.swift:513)."""
        return 4.0 * self.batch * self.dims.Hq * self.dims.R * self.dims.C * self.dims.K

    def _check(self, **tensors):
        import torch
        d = self.dims
        shapes = {"Q": self.shape(d.R, d.Hq), "O": self.shape(d.R, d.Hq), "dO": self.shape(d.R, d.Hq),
                  "K": self.shape(d.C, d.Hk), "V": self.shape(d.C, d.Hk)}
        for n, t in tensors.items():
            shp = shapes[n]
            if tuple(t.shape) != shp or t.dtype != torch.float16 or not t.is_cuda or not t.is_contiguous():
                raise ValueError(f"{n} must be a contiguous CUDA fp16 tensor of shape {shp}")

    def lse_shape(self):
        return (self.batch, self.dims.Hq, self.dims.R)

    def run(self, Q, K, V, O=None, stream=None, duplicatedCount: int = 1, lse=None):
        """O = softmax(scale Q K^T) V. With `lse` (fp32 [B][Hq][R] CUDA tensor) also writes each row's
        natural-log sum of exp(scale * S) (Network.swift createLTerm), which `backward` takes."""
        import torch
        d = self.dims
        self._check(Q=Q, K=K, V=V)
        if O is None:
            O = torch.empty(self.shape(d.R, d.Hq), dtype=torch.float16, device=Q.device)
        if lse is not None:
            if tuple(lse.shape) != self.lse_shape() or lse.dtype != torch.float32 or not lse.is_contiguous():
                raise ValueError(f"lse must be a contiguous fp32 tensor of shape {self.lse_shape()}")
            if duplicatedCount != 1:
                raise ValueError("duplicatedCount must be 1 when lse is requested")
            _lib.check(self._L.mm4_attention_fwd_lse(self._h, Q.data_ptr(), K.data_ptr(), V.data_ptr(),
                                                     O.data_ptr(), lse.data_ptr(), _lib.stream_handle(stream)))
            return O
        _lib.check(self._L.mm4_attention_fwd(self._h, Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(),
                                             _lib.stream_handle(stream), int(duplicatedCount)))
        return O

    def run_host(self, Q, K, V, O, staging, chunks: int = 16, stream=None):
        """O = softmax(scale Q K^T) V for CPU tensors (pinned for the copies to overlap): Q, K, V are copied
        in through the CUDA tensors `staging` = (dQ, dK, dV, dO) of the full shapes, and O is copied out,
        as a pipeline over `chunks` pieces of the (batch, head) units (mm4_attention_fwd_host). Ordered on
        `stream`; the result is in O once the stream reaches the end of the call."""
        import torch
        d = self.dims
        dQ, dK, dV, dO = staging
        self._check(Q=dQ, K=dK, V=dV, O=dO)
        shapes = {"Q": self.shape(d.R, d.Hq), "K": self.shape(d.C, d.Hk), "V": self.shape(d.C, d.Hk),
                  "O": self.shape(d.R, d.Hq)}
        for n, t in (("Q", Q), ("K", K), ("V", V), ("O", O)):
            if t.is_cuda or t.dtype != torch.float16 or not t.is_contiguous() or tuple(t.shape) != shapes[n]:
                raise ValueError(f"{n} must be a contiguous CPU fp16 tensor of shape {shapes[n]}")
        _lib.check(self._L.mm4_attention_fwd_host(self._h, Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(),
                                                  dQ.data_ptr(), dK.data_ptr(), dV.data_ptr(), dO.data_ptr(),
                                                  int(chunks), _lib.stream_handle(stream)))
        return O

    def backward_host(self, Q, K, V, O, dO, lse, dQ, dK, dV, staging_in, staging_out, workspace, chunks: int = 16,
                      stream=None):
        """dQ, dK, dV (CPU fp16 outputs) of sum(dO * O) from CPU Q, K, V, O, dO (fp16) and lse (fp32), pinned
        for the copies to overlap, through the CUDA tensors staging_in = (Q, K, V, O, dO, lse) and
        staging_out = (dQ, dK, dV) of the full shapes: copies in, the backward and copies out run as a
        pipeline over `chunks` pieces (mm4_attention_bwd_host). Ordered on `stream`."""
        import torch
        host_in, host_out = (Q, K, V, O, dO, lse), (dQ, dK, dV)
        for t in host_in + host_out:
            if t.is_cuda or not t.is_contiguous():
                raise ValueError("host tensors must be contiguous CPU tensors")
        for h, dv in zip(host_in + host_out, tuple(staging_in) + tuple(staging_out)):
            if not dv.is_cuda or tuple(h.shape) != tuple(dv.shape) or h.dtype != dv.dtype or not dv.is_contiguous():
                raise ValueError("staging tensors must be contiguous CUDA copies of the host tensors' shapes")
        self._check(Q=staging_in[0], K=staging_in[1], V=staging_in[2], O=staging_in[3], dO=staging_in[4])
        if tuple(lse.shape) != self.lse_shape() or lse.dtype != torch.float32:
            raise ValueError(f"lse must be fp32 of shape {self.lse_shape()}")
        arr = lambda ts: (ctypes.c_void_p * len(ts))(*[t.data_ptr() for t in ts])  # noqa: E731
        _lib.check(self._L.mm4_attention_bwd_host(self._h, arr(host_in), arr(host_out), arr(tuple(staging_in)),
                                                  arr(tuple(staging_out)), workspace.data_ptr(), workspace.numel(),
                                                  int(chunks), _lib.stream_handle(stream)))
        return dQ, dK, dV

    def backward_workspace_bytes(self) -> int:
        """Bytes of scratch `backward` needs (any contents, 16-byte aligned)."""
        return int(self._L.mm4_attention_bwd_workspace_size(self._h))

    def backward(self, Q, K, V, O, dO, lse, stream=None, dQ=None, dK=None, dV=None, workspace=None):
        """dQ, dK, dV (fp16, the layouts of Q, K, V) of sum(dO * O), from the forward's O and lse."""
        import torch
        d = self.dims
        self._check(Q=Q, K=K, V=V, O=O, dO=dO)
        if tuple(lse.shape) != self.lse_shape() or lse.dtype != torch.float32 or not lse.is_contiguous():
            raise ValueError(f"lse must be a contiguous fp32 tensor of shape {self.lse_shape()}")
        dQ = torch.empty_like(Q) if dQ is None else dQ
        dK = torch.empty_like(K) if dK is None else dK
        dV = torch.empty_like(V) if dV is None else dV
        if workspace is None:
            workspace = torch.empty(self.backward_workspace_bytes(), dtype=torch.uint8, device=Q.device)
        _lib.check(self._L.mm4_attention_bwd(self._h, Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(),
                                             dO.data_ptr(), lse.data_ptr(), dQ.data_ptr(), dK.data_ptr(),
                                             dV.data_ptr(), workspace.data_ptr(), workspace.numel(),
                                             _lib.stream_handle(stream)))
        return dQ, dK, dV


def run(sequenceDimension: int, headDimension: int, Hq: int, Hk: int,
        buildOptions: BuildOptions | None = None, duplicatedCount: int = 1, seed: int = 3, log=print):
    """The reference's attention run(sequenceDimension:headDimension:Hq:Hk:buildOptions:duplicatedCount:)
    (attention.swift:398-541): Q, K, V N(0,1) by Box-Muller (Network.swift:90-129; seeded here) in the
    [S][H][D] packing; `duplicatedCount` launches; "GFlops" with the reference's (2D+5) S^2 Hq count over
    their GPU time (:507-515); every element of O checked against the fp32 softmax(Q K^T / sqrt D) V with
    tolerance 5e-3 (:517-540), the expectation computed by torch on the host. Returns the same record as
    gemm.run."""
    import torch

    from . import data
    from .gemm import RunResult, _check, _gpu_time
    S, D = sequenceDimension, headDimension
    plan = AttentionPlan(AttentionDimensions(S, S, D, Hq, Hk), batch=1, layout=MM4_ATTN_BSHD,
                         buildOptions=buildOptions)
    Q = data.normal((1, S, Hq, D), 1.0, seed, 0)
    K = data.normal((1, S, Hk, D), 1.0, seed, 1)
    V = data.normal((1, S, Hk, D), 1.0, seed, 2)
    dev = torch.device("cuda", torch.cuda.current_device())
    tQ, tK, tV = (torch.from_numpy(x).to(dev) for x in (Q, K, V))
    O = torch.empty_like(tQ)
    seconds = _gpu_time(lambda: plan.run(tQ, tK, tV, O=O), duplicatedCount)
    ops = (2 * D + 5) * S * S * Hq * duplicatedCount
    gflops = ops / seconds / 1e9 if seconds > 0 else 0.0
    log(f"GFlops: {int(gflops)}")
    q = torch.from_numpy(Q[0]).float().permute(1, 0, 2)                     # [Hq][S][D]
    k = torch.from_numpy(K[0]).float().permute(1, 0, 2).repeat_interleave(Hq // Hk, dim=0)
    v = torch.from_numpy(V[0]).float().permute(1, 0, 2).repeat_interleave(Hq // Hk, dim=0)
    expected = (torch.softmax(q @ k.transpose(1, 2) * plan.scale, dim=-1) @ v).permute(1, 0, 2).numpy()
    max_err, bad = _check(expected, O[0].float().cpu().numpy(), "O", 5e-3, log)
    return RunResult(gflops, seconds * 1e3, max_err, bad, plan.kernel_name)


def profileCorrectness(sizes=range(1, 1024), log=print):
    """The reference's sweep (attention.swift:390-395): S = 1..1023, D = 128, Hq = Hk = 8."""
    out = []
    for i in sizes:
        log(f"Problem size: {i}")
        out.append(run(i, 128, 8, 8, BuildOptions(executionSIMDGroups=16, bypassThreadgroupMemory=True), 1,
                       log=log))
    return out
