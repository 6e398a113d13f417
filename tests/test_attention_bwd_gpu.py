"""Attention backward parity on the GPU: mm4 dQ / dK / dV and the forward's
log-sum-exp (through the C ABI) vs the C oracle restating Network.swift
derivativeQ / derivativeK / derivativeV / createLTerm (:181-203, :328-401),
which tests/test_oracle.py pins against finite differences of the loss."""
import numpy as np
import pytest

import oracle
from example_matmul_metal4_b200 import data, sync_check
from example_matmul_metal4_b200.attention import MM4_ATTN_BHSD, MM4_ATTN_BSHD, AttentionDimensions, AttentionPlan

pytestmark = pytest.mark.gpu

# Gradients of N(0,1) attention are O(1e-2), below the forward's absolute
# 2e-2 tolerance, so they are checked relative to their own scale instead:
# relative Frobenius error <= GRAD_REL_FRO, and every element within
# GRAD_REL_MAX * max|ref|. fp16 P, dS and outputs carry ~5e-4 relative
# rounding each.
GRAD_REL_FRO = 1e-2
GRAD_REL_MAX = 2e-2


def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _check_grad(got, ref, what):
    g = got.float().cpu().numpy().astype(np.float64)
    r = np.asarray(ref, dtype=np.float64)
    assert g.shape == r.shape, (what, g.shape, r.shape)
    rel = np.linalg.norm(g - r) / max(np.linalg.norm(r), 1e-30)
    worst = float(np.abs(g - r).max())
    scale = float(np.abs(r).max())
    assert rel <= GRAD_REL_FRO and worst <= GRAD_REL_MAX * scale, \
        f"{what}: relative Frobenius error {rel:.3e}, max abs error {worst:.3e}, max |ref| {scale:.3e}"


def _forward_backward(cuda, plan, Q, K, V, dO):
    import torch
    tQ, tK, tV, tdO = (_t(a, cuda) for a in (Q, K, V, dO))
    lse = torch.empty(plan.lse_shape(), dtype=torch.float32, device=cuda)
    O = plan.run(tQ, tK, tV, lse=lse)
    dQ, dK, dV = plan.backward(tQ, tK, tV, O, tdO, lse)
    sync_check()
    return lse, dQ, dK, dV


@pytest.mark.parametrize("D", [128, 64])
@pytest.mark.parametrize("B,Hq,Hk,R,C,layout", [
    (1, 2, 2, 256, 256, MM4_ATTN_BHSD),  # whole tiles
    (2, 4, 2, 200, 333, MM4_ATTN_BSHD),  # grouped-query heads, ragged R and C, [S][H][D] packing
    (1, 1, 1, 130, 129, MM4_ATTN_BHSD),  # one query row and one key past a tile
    (1, 2, 2, 64, 64, MM4_ATTN_BHSD),    # less than one tile: a single query and key half
])
def test_backward_vs_oracle(cuda, B, Hq, Hk, R, C, layout, D):
    plan = AttentionPlan(AttentionDimensions(R, C, D, Hq, Hk), batch=B, layout=layout)
    Q = data.normal(plan.shape(R, Hq), 1.0, 50 + R, 0)
    K = data.normal(plan.shape(C, Hk), 1.0, 50 + R, 1)
    V = data.normal(plan.shape(C, Hk), 1.0, 50 + R, 2)
    dO = data.normal(plan.shape(R, Hq), 1.0, 50 + R, 3)
    lse, dQ, dK, dV = _forward_backward(cuda, plan, Q, K, V, dO)
    rQ, rK, rV, rlse = oracle.attention_bwd(Q, K, V, dO, B, Hq, Hk, R, C, D, plan.scale, layout,
                                            threads=oracle.default_threads())
    np.testing.assert_allclose(lse.cpu().numpy(), rlse, rtol=1e-4, atol=1e-3, err_msg="lse")
    _check_grad(dQ, rQ, "dQ")
    _check_grad(dK, rK, "dK")
    _check_grad(dV, rV, "dV")


@pytest.mark.parametrize("D", [128, 64])
def test_backward_full_length_vs_fp32_autograd(cuda, D):
    """S = 4096 (the BASELINE sequence length) on two heads: every gradient
    element against fp32 torch autograd of softmax(scale Q K^T) V on the same
    fp16 inputs."""
    import torch
    B, H, S = 1, 2, 4096
    plan = AttentionPlan(AttentionDimensions(S, S, D, H, H), batch=B)
    Q, K, V, dO = (data.normal((B, H, S, D), 1.0, 61, i) for i in range(4))
    lse, dQ, dK, dV = _forward_backward(cuda, plan, Q, K, V, dO)
    for h in range(H):
        q, k, v = (_t(a[0, h], cuda).float().requires_grad_(True) for a in (Q, K, V))
        p = torch.softmax((q @ k.T) * plan.scale, dim=-1)
        o = p @ v
        o.backward(_t(dO[0, h], cuda).float())
        ref_lse = torch.logsumexp((q @ k.T) * plan.scale, dim=-1)
        np.testing.assert_allclose(lse[0, h].cpu().numpy(), ref_lse.detach().cpu().numpy(), rtol=1e-4, atol=1e-3)
        _check_grad(dQ[0, h], q.grad.cpu().numpy(), f"dQ h={h}")
        _check_grad(dK[0, h], k.grad.cpu().numpy(), f"dK h={h}")
        _check_grad(dV[0, h], v.grad.cpu().numpy(), f"dV h={h}")


def test_backward_repeated_calls_are_bitwise_identical(cuda):
    """No atomics and a fixed MMA order per output element: repeated backward calls on the same inputs give
    the same bits."""
    import torch
    B, H, S, D = 1, 4, 1024, 128
    plan = AttentionPlan(AttentionDimensions(S, S, D, H, H), batch=B)
    Q, K, V, dO = (data.normal((B, H, S, D), 1.0, 71, i) for i in range(4))
    tQ, tK, tV, tdO = (_t(a, cuda) for a in (Q, K, V, dO))
    lse = torch.empty(plan.lse_shape(), dtype=torch.float32, device=cuda)
    O = plan.run(tQ, tK, tV, lse=lse)
    first = [g.clone() for g in plan.backward(tQ, tK, tV, O, tdO, lse)]
    for _ in range(3):
        again = plan.backward(tQ, tK, tV, O, tdO, lse)
        sync_check()
        for a, b in zip(first, again):
            assert torch.equal(a, b)


@pytest.mark.parametrize("D", [128, 64])
@pytest.mark.parametrize("layout,B,Hq,Hk", [(MM4_ATTN_BHSD, 3, 4, 2), (MM4_ATTN_BSHD, 3, 4, 4)])
def test_host_buffer_backward_matches_device_backward(cuda, D, layout, B, Hq, Hk):
    """mm4_attention_bwd_host (pinned host inputs and outputs, pipelined over chunks of key/value heads or
    batch elements) gives mm4_attention_bwd's bits, for 1 chunk, a ragged split and more chunks than
    pieces."""
    import torch
    R, C = 200, 333
    plan = AttentionPlan(AttentionDimensions(R, C, D, Hq, Hk), batch=B, layout=layout)
    Q = _t(data.normal(plan.shape(R, Hq), 1.0, 6, 0), cuda)
    K = _t(data.normal(plan.shape(C, Hk), 1.0, 6, 1), cuda)
    V = _t(data.normal(plan.shape(C, Hk), 1.0, 6, 2), cuda)
    dO = _t(data.normal(plan.shape(R, Hq), 1.0, 6, 3), cuda)
    lse = torch.empty(plan.lse_shape(), dtype=torch.float32, device=cuda)
    O = plan.run(Q, K, V, lse=lse)
    ws = torch.empty(plan.backward_workspace_bytes(), dtype=torch.uint8, device=cuda)
    ref = [g.cpu() for g in plan.backward(Q, K, V, O, dO, lse, workspace=ws)]
    sync_check()
    host_in = tuple(x.cpu().pin_memory() for x in (Q, K, V, O, dO, lse))
    host_out = tuple(torch.empty(x.shape, dtype=x.dtype).pin_memory() for x in ref)
    staging_in = tuple(torch.empty_like(x) for x in (Q, K, V, O, dO, lse))
    staging_out = (torch.empty_like(Q), torch.empty_like(K), torch.empty_like(V))
    for chunks in (1, 4, 64):
        for h in host_out:
            h.fill_(float("nan"))
        plan.backward_host(*host_in, *host_out, staging_in, staging_out, ws, chunks=chunks)
        sync_check()
        for name, h, r in zip(("dQ", "dK", "dV"), host_out, ref):
            assert torch.equal(h, r), (chunks, name)
