"""The attention forward's software 2^x (ex2_poly2) against CUDA's exp2f.

The softmax computes 2^(scale*log2(e)*s - m) (the base-2 form of
attention.swift:24). Two of every eight elements take ex2_poly2, a cubic on
the FMA pipe: x = n + f with n = round(x), 2^f from the cubic on [-1/2, 1/2],
2^n added into the exponent field, inputs clamped at -125. The test sweeps
[-130, 10]: a dense grid, every fp32 exponent bucket of both signs, the
half-way points n +- 1/2 (where round-to-nearest-even picks n), and the
clamp. The reference output is torch.exp2 on the GPU (CUDA's exp2f); the
bound is the cubic's documented 7.5e-5 maximum relative error plus exp2f's
own 2-ulp error."""
import numpy as np
import pytest

from example_matmul_metal4_b200 import lib
from example_matmul_metal4_b200._lib import check, stream_handle

pytestmark = pytest.mark.gpu

POLY_REL = 7.5e-5
EXP2F_REL = 2 * 2.0 ** -23


def _sweep():
    grid = np.linspace(-130.0, 10.0, 1_400_001, dtype=np.float64)
    buckets = []
    for e in range(-40, 4):  # |x| from 2^-40 to 2^3 (10 lies in the 2^3 bucket)
        lo = 2.0 ** e
        buckets.append(np.linspace(lo, 2 * lo, 257)[:-1])
    buckets = np.concatenate(buckets)
    buckets = np.concatenate([buckets, -buckets, -buckets * 16])
    halves = np.arange(-130, 11, dtype=np.float64)
    halves = np.concatenate([halves + 0.5, halves - 0.5, halves,
                             np.nextafter(halves + 0.5, np.inf), np.nextafter(halves + 0.5, -np.inf)])
    x = np.concatenate([grid, buckets, halves, [0.0, -0.0, -125.0, -124.999, -125.001, -126.0, -200.0]])
    x = x[(x >= -200.0) & (x <= 10.0)]
    return x.astype(np.float32)


def _ex2(x, method, cuda):
    import torch
    tx = torch.from_numpy(x).to(cuda)
    ty = torch.empty_like(tx)
    check(lib().mm4_debug_ex2(tx.data_ptr(), ty.data_ptr(), tx.numel(), method, stream_handle()))
    torch.cuda.synchronize()
    return ty, tx


def test_ex2_poly2_against_exp2f(cuda):
    import torch
    x = _sweep()
    y, tx = _ex2(x, 1, cuda)
    ref = torch.exp2(tx).double().cpu().numpy()
    got = y.double().cpu().numpy()
    inside = x >= -125.0
    rel = np.abs(got[inside] - ref[inside]) / ref[inside]
    assert rel.max() <= POLY_REL + EXP2F_REL, (rel.max(), x[inside][np.argmax(rel)])
    # against the exact value as well (float64), with only fp32 rounding on top
    exact = np.exp2(x[inside].astype(np.float64))
    rel64 = np.abs(got[inside] - exact) / exact
    assert rel64.max() <= POLY_REL + 2.0 ** -24, rel64.max()
    # below the clamp every result is 2^-125 (within the cubic's error): a normal float, which rounds
    # to 0 in fp16 as a masked score must
    below = got[~inside]
    assert below.size > 0
    assert np.all(np.abs(below / 2.0 ** -125 - 1.0) <= POLY_REL + 2.0 ** -24), below
    assert np.all(below >= np.finfo(np.float32).tiny)
    assert np.all(torch.from_numpy(below.astype(np.float32)).half().numpy() == 0)
    # monotone up to the cubic's error: where f wraps from +1/2 to -1/2 the two ends' errors may differ
    g = np.argsort(x[inside], kind="stable")
    assert np.all(np.diff(got[inside][g]) >= -2 * POLY_REL * got[inside][g][1:])


def test_ex2_hardware_against_exp2f(cuda):
    """The MUFU path the other six of eight elements take; inputs that the softmax produces are <= 0."""
    import torch
    x = _sweep()
    x = x[(x >= -125.0) & (x <= 0.0)]
    y, tx = _ex2(x, 0, cuda)
    ref = torch.exp2(tx).double().cpu().numpy()
    rel = np.abs(y.double().cpu().numpy() - ref) / ref
    assert rel.max() <= 2.0 ** -20, rel.max()  # both are within a few ulp of 2^x
