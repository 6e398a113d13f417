"""The CUDA path against the committed golden fixtures (tests/golden/, made by
make_golden.py from the C oracle): GEMM + bias in NN / NT / TN, the attention
forward in both layouts with grouped-query heads, and the attention backward."""
from pathlib import Path

import numpy as np
import pytest

from example_matmul_metal4_b200 import GEMMDimensions, GemmPlan, sync_check
from example_matmul_metal4_b200.attention import AttentionDimensions, AttentionPlan
from tolerance import assert_close

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"


def _cases(name):
    z = np.load(GOLDEN / name)
    return z, sorted({k.split("/")[0] for k in z.files})


def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def test_gemm_fixtures(cuda):
    z, names = _cases("gemm_small.npz")
    for n in names:
        M, N, K, tl, tr = (int(v) for v in z[f"{n}/dims"])
        plan = GemmPlan(GEMMDimensions(M, N, K), transpose=(bool(tl), bool(tr)), bias=True)
        C = plan.run(_t(z[f"{n}/A"], cuda), _t(z[f"{n}/B"], cuda), _t(z[f"{n}/bias"], cuda))
        sync_check()
        assert_close(C.float().cpu().numpy(), z[f"{n}/out"], f"{n} {plan.kernel_name}")


def test_attention_forward_fixtures(cuda):
    z, names = _cases("attention_small.npz")
    for n in names:
        B, Hq, Hk, R, C, layout, D = (int(v) for v in z[f"{n}/dims"])
        plan = AttentionPlan(AttentionDimensions(R, C, D, Hq, Hk), batch=B, layout=layout)
        O = plan.run(_t(z[f"{n}/Q"], cuda), _t(z[f"{n}/K"], cuda), _t(z[f"{n}/V"], cuda))
        sync_check()
        got = O.float().cpu().numpy()
        if layout == 1:
            got = got.transpose(0, 2, 1, 3)  # the oracle writes [B][H][R][D]
        assert_close(got, z[f"{n}/out"], n)


def test_attention_backward_fixtures(cuda):
    """Gradients checked relative to their scale: relative Frobenius error <= 1e-2 and every element within
    2e-2 * max|ref| (fp16 P, dS and outputs)."""
    import torch
    z, names = _cases("attention_bwd_small.npz")
    for n in names:
        B, Hq, Hk, R, C, layout, D = (int(v) for v in z[f"{n}/dims"])
        plan = AttentionPlan(AttentionDimensions(R, C, D, Hq, Hk), batch=B, layout=layout)
        tQ, tK, tV, tdO = (_t(z[f"{n}/{k}"], cuda) for k in ("Q", "K", "V", "dO"))
        lse = torch.empty(plan.lse_shape(), dtype=torch.float32, device=cuda)
        O = plan.run(tQ, tK, tV, lse=lse)
        grads = plan.backward(tQ, tK, tV, O, tdO, lse)
        sync_check()
        np.testing.assert_allclose(lse.cpu().numpy(), z[f"{n}/lse"], rtol=1e-4, atol=1e-3, err_msg=f"{n} lse")
        for key, g in zip(("dQ", "dK", "dV"), grads):
            got = g.float().cpu().numpy().astype(np.float64)
            ref = z[f"{n}/{key}"].astype(np.float64)
            rel = np.linalg.norm(got - ref) / np.linalg.norm(ref)
            worst = np.abs(got - ref).max()
            assert rel <= 1e-2 and worst <= 2e-2 * np.abs(ref).max(), f"{n} {key}: rel {rel:.3e} max {worst:.3e}"
