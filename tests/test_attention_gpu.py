"""Attention parity on the GPU: mm4 flash-attention forward (through the C
ABI) vs the C oracle (Network.swift:134-179, :286-311 restated)."""
import numpy as np
import pytest

import oracle
from example_matmul_metal4_b200 import data, sync_check
from example_matmul_metal4_b200.attention import MM4_ATTN_BHSD, MM4_ATTN_BSHD, AttentionDimensions, AttentionPlan
from tolerance import assert_close

pytestmark = pytest.mark.gpu


def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _run(cuda, B, Hq, Hk, R, C, layout=MM4_ATTN_BHSD, seed=3, rows=None, D=128):
    plan = AttentionPlan(AttentionDimensions(R, C, D, Hq, Hk), batch=B, layout=layout)
    Q = data.normal(plan.shape(R, Hq), 1.0, seed, 0)
    K = data.normal(plan.shape(C, Hk), 1.0, seed, 1)
    V = data.normal(plan.shape(C, Hk), 1.0, seed, 2)
    O = plan.run(_t(Q, cuda), _t(K, cuda), _t(V, cuda))
    sync_check()
    got = O.float().cpu().numpy()
    ref = oracle.attention(Q, K, V, B, Hq, Hk, R, C, D, plan.scale, layout, rows=rows,
                           threads=oracle.default_threads())
    if layout == MM4_ATTN_BSHD:
        got = got.transpose(0, 2, 1, 3)
    if rows:
        got = got[:, :, rows[0]:rows[1]]
    return plan, got, ref


@pytest.mark.parametrize("D", [128, 64])
@pytest.mark.parametrize("S", [1, 7, 64, 127, 128, 129, 300, 1023])
def test_reference_sweep_points(cuda, S, D):
    """Points of the reference's S = 1..1023, Hq = Hk = 8 sweep (attention.swift:391-396) at its head
    dimension 128 and at 64 (run(...) takes headDimension as a parameter, attention.swift:398)."""
    plan, got, ref = _run(cuda, 1, 8, 8, S, S, D=D)
    assert_close(got, ref, f"S={S} D={D}")


@pytest.mark.parametrize("D", [128, 64])
@pytest.mark.parametrize("layout", [MM4_ATTN_BHSD, MM4_ATTN_BSHD])
def test_layouts_and_batch(cuda, layout, D):
    plan, got, ref = _run(cuda, 2, 4, 4, 256, 384, layout=layout, D=D)
    assert_close(got, ref, f"layout {layout} D={D}")


@pytest.mark.parametrize("D", [128, 64])
def test_gqa_and_rectangular(cuda, D):
    plan, got, ref = _run(cuda, 2, 8, 2, 200, 520, D=D)
    assert_close(got, ref, f"GQA 8/2, R=200 C=520, D={D}")


def test_repeated_launches_are_bitwise_identical(cuda):
    """Each output element is one fixed sequence of MMAs and softmax steps: 20 launches of one plan on the
    same inputs (the reference's duplicatedCount) give the same bits every time."""
    import torch
    B, H, S, D = 2, 4, 1024, 128
    plan = AttentionPlan(AttentionDimensions(S, S, D, H, H), batch=B)
    Q, K, V = (_t(data.normal((B, H, S, D), 1.0, 13, i), cuda) for i in range(3))
    first = plan.run(Q, K, V).clone()
    O = torch.empty_like(first)
    for _ in range(4):
        plan.run(Q, K, V, O=O, duplicatedCount=5)
        sync_check()
        assert torch.equal(O, first)


@pytest.mark.parametrize("D", [128, 64])
def test_large_logits_rescale_path(cuda, D):
    """Scaled inputs push the running max up across key tiles so the lazy
    rescale of O (max growth > 2^8) is exercised."""
    import torch
    B, H, R, C = 1, 2, 256, 1024
    plan = AttentionPlan(AttentionDimensions(R, C, D, H, H), batch=B)
    Q = data.normal((B, H, R, D), 1.0, 8, 0)
    Kn = data.normal((B, H, C, D), 1.0, 8, 1).astype(np.float32)
    Kn *= np.linspace(0.5, 4.0, C, dtype=np.float32)[None, None, :, None]  # later keys give larger logits
    K = Kn.astype(np.float16)
    V = data.normal((B, H, C, D), 1.0, 8, 2)
    O = plan.run(_t(Q, cuda), _t(K, cuda), _t(V, cuda))
    sync_check()
    ref = oracle.attention(Q, K, V, B, H, H, R, C, D, plan.scale, 0, threads=oracle.default_threads())
    assert_close(O.float().cpu().numpy(), ref, f"rescale path D={D}")


def test_baseline_config3_rows_sample(cuda):
    """B=4, H=16, S=4096, D=128, N(0,1), scale 1/sqrt(128).
    Oracle on a sample of query rows of every (b, h); all outputs also checked
    against an fp32 torch reference."""
    import torch
    B, H, S, D = 4, 16, 4096, 128
    plan, got, ref = _run(cuda, B, H, H, S, S, rows=(0, 8))
    assert_close(got, ref, "rows 0:8")
    plan2, got2, ref2 = _run(cuda, B, H, H, S, S, rows=(4090, 4096))
    assert_close(got2, ref2, "rows 4090:4096")
    # full-output property check against fp32 SDPA on the same fp16 inputs
    Q = _t(data.normal((B, H, S, D), 1.0, 3, 0), cuda)
    K = _t(data.normal((B, H, S, D), 1.0, 3, 1), cuda)
    V = _t(data.normal((B, H, S, D), 1.0, 3, 2), cuda)
    O = plan.run(Q, K, V)
    sync_check()
    for bh in range(0, B * H, 5):
        b, h = divmod(bh, H)
        s = (Q[b, h].float() @ K[b, h].float().T) * plan.scale
        p = torch.softmax(s, dim=-1)
        o = p @ V[b, h].float()
        assert_close(O[b, h].float().cpu().numpy(), o.cpu().numpy(), f"b={b} h={h} vs fp32 torch")


def test_head_dim_64_full_length_rows_sample(cuda):
    """The BASELINE attention shape at head_dim 64 (B=4, H=16, S=4096): oracle rows at both ends of every
    (b, h)."""
    B, H, S = 4, 16, 4096
    plan, got, ref = _run(cuda, B, H, H, S, S, rows=(0, 4), D=64)
    assert_close(got, ref, "D=64 rows 0:4")
    plan, got, ref = _run(cuda, B, H, H, S, S, rows=(4093, 4096), D=64)
    assert_close(got, ref, "D=64 rows 4093:4096")


def test_unsupported_head_dim_is_rejected():
    from example_matmul_metal4_b200 import MM4Error
    with pytest.raises(MM4Error):
        AttentionPlan(AttentionDimensions(64, 64, 96, 1, 1))


@pytest.mark.parametrize("D", [128, 64])
@pytest.mark.parametrize("layout,B,Hq,Hk", [(MM4_ATTN_BHSD, 3, 4, 2), (MM4_ATTN_BSHD, 3, 4, 4)])
def test_host_buffer_forward_matches_device_forward(cuda, D, layout, B, Hq, Hk):
    """mm4_attention_fwd_host (pinned host Q, K, V in, O out; pipelined over chunks of whole key/value
    heads or batch elements) gives the device forward's bits, for 1 chunk, a ragged split and more chunks
    than pieces."""
    import torch
    R, C = 200, 333
    plan = AttentionPlan(AttentionDimensions(R, C, D, Hq, Hk), batch=B, layout=layout)
    Q = _t(data.normal(plan.shape(R, Hq), 1.0, 5, 0), cuda)
    K = _t(data.normal(plan.shape(C, Hk), 1.0, 5, 1), cuda)
    V = _t(data.normal(plan.shape(C, Hk), 1.0, 5, 2), cuda)
    ref = plan.run(Q, K, V)
    sync_check()
    ref = ref.cpu()
    hQ, hK, hV = Q.cpu().pin_memory(), K.cpu().pin_memory(), V.cpu().pin_memory()
    hO = torch.empty(ref.shape, dtype=torch.float16).pin_memory()
    staging = (torch.empty_like(Q), torch.empty_like(K), torch.empty_like(V), torch.empty_like(Q))
    for chunks in (1, 4, 64):
        hO.fill_(float("nan"))
        plan.run_host(hQ, hK, hV, hO, staging, chunks=chunks)
        sync_check()
        assert torch.equal(hO, ref), chunks


@pytest.mark.parametrize("D", [128, 64])
def test_persistent_units_gqa_bshd_ragged(cuda, D):
    """More (batch, head, 256-row) units than SMs with grouped-query heads, the [B][S][H][D] layout and
    ragged rows and keys: every CTA of the persistent forward walks 2-3 units of different batches and
    heads, each ending on a partial query block. Oracle rows at the start, across the first block edge and
    at the end of R, for every (b, h)."""
    B, Hq, Hk, R, C = 5, 16, 4, 1000, 777
    for rows in ((0, 3), (254, 258), (997, 1000)):
        plan, got, ref = _run(cuda, B, Hq, Hk, R, C, layout=MM4_ATTN_BSHD, rows=rows, D=D)
        assert_close(got, ref, f"D={D} rows {rows}")
