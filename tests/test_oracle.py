"""Pins the C oracle (oracle/mm4_oracle.c) before any GPU result is trusted.

- fp16 <-> fp32 conversions against numpy, exhaustively / on random samples;
- known answers the reference itself holds: the 1-channel ramp with a centre
  tap (ConvolutionShared.swift:4876-4893), the set_offsets shift probe
  (convolution.swift:204-216, :372-392, AGENTS.md:67-70: an offset of +1
  samples the input one element later), and referenceForOffset(0,0) with the
  dense 1..9 kernel (convolution.swift:372-392);
- an independent float64 restatement of every loop (GEMM, attention, conv);
- the committed golden fixtures (tests/golden/make_golden.py).
"""
import numpy as np
import pytest

import oracle
from cases import (CONV2D_PADDED, CONV2D_VALID, CONV3D_HW_PADDED, CONV3D_LR_PADDED, CONV3D_VALID, oracle_kwargs2d,
                   oracle_kwargs3d)
from example_matmul_metal4_b200 import data
from pathlib import Path

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_half_to_float_exhaustive():
    L = oracle.lib()
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    ref = bits.view(np.float16).astype(np.float32)
    got = np.array([L.mm4o_half_to_float(int(b)) for b in bits[::7]], dtype=np.float32)
    r = ref[::7]
    both_nan = np.isnan(got) & np.isnan(r)
    assert np.array_equal(got[~both_nan], r[~both_nan])


def test_float_to_half_round_to_nearest_even():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(200000).astype(np.float32) * s for s in (1e-6, 1e-3, 1, 100, 3e4)])
    x = np.concatenate([x, np.array([0.0, -0.0, 65504, 65519.99, 65520, 1e9, -1e9, 5.96e-8, 2.98e-8, 2.99e-8],
                                    dtype=np.float32)])
    got = oracle.to_half(x).view(np.uint16)
    ref = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, ref)


# --------------------------------------------------------------- known answers

RAMP = np.arange(1, 26, dtype=np.float32).reshape(5, 5)


def _ramp_conv(kernel3x3, pt, pb, pl, pr):
    x = RAMP.astype(np.float16).reshape(1, 5, 5, 1)
    w = kernel3x3.astype(np.float16).reshape(3, 3, 1, 1)
    return oracle.conv2d(x, w, None, N=1, H=5, W=5, C=1, O=1, KH=3, KW=3, pad_top=pt, pad_bottom=pb,
                         pad_left=pl, pad_right=pr, layout=0).reshape(-1, RAMP.shape[1] if pl + pr == 2 else 3)


def test_kat_centre_tap_valid_is_centre_of_ramp():
    centre = np.zeros((3, 3), np.float32)
    centre[1, 1] = 1
    out = _ramp_conv(centre, 0, 0, 0, 0)
    assert np.array_equal(out, RAMP[1:4, 1:4])


def test_kat_centre_tap_same_padding_is_identity():
    centre = np.zeros((3, 3), np.float32)
    centre[1, 1] = 1
    assert np.array_equal(_ramp_conv(centre, 1, 1, 1, 1), RAMP)


@pytest.mark.parametrize("dx,dy", [(0, 0), (1, 1), (1, 0), (0, 1)])
def test_kat_set_offsets_shift(dx, dy):
    """An offset (dx, dy) samples input[h+dy][w+dx] with zero fill
    (convolution.swift inferShift :333-363); as a padded conv that is
    padding (1-dy, 1+dy) x (1-dx, 1+dx)."""
    centre = np.zeros((3, 3), np.float32)
    centre[1, 1] = 1
    out = _ramp_conv(centre, 1 - dy, 1 + dy, 1 - dx, 1 + dx)
    exp = np.zeros((5, 5), np.float32)
    exp[:5 - dy, :5 - dx] = RAMP[dy:, dx:]
    assert np.array_equal(out, exp)


def test_kat_dense_kernel_reference_for_offset_zero():
    """referenceForOffset(activation: 1...25, weights: 1...9, 0, 0)
    (convolution.swift:372-392) restated as literal loops."""
    dense = np.arange(1, 10, dtype=np.float32).reshape(3, 3)
    exp = np.zeros((5, 5), np.float32)
    for oh in range(5):
        for ow in range(5):
            s = 0.0
            for kh in range(3):
                for kw in range(3):
                    ih, iw = oh + kh - 1, ow + kw - 1
                    if 0 <= ih < 5 and 0 <= iw < 5:
                        s += RAMP[ih, iw] * dense[kh, kw]
            exp[oh, ow] = s
    assert exp[0, 0] == 5 * 1 + 6 * 2 + 8 * 6 + 9 * 7  # spot value of the literal loop
    assert np.array_equal(_ramp_conv(dense, 1, 1, 1, 1), exp)


# ---------------------------------------------------------- float64 restatements

def _gemm64(A, B, bias, tl, tr):
    a = A.astype(np.float64).T if tl else A.astype(np.float64)
    b = B.astype(np.float64).T if tr else B.astype(np.float64)
    return a @ b + (bias.astype(np.float64) if bias is not None else 0.0)


@pytest.mark.parametrize("tl,tr", [(False, False), (False, True), (True, False), (True, True)])
def test_gemm_oracle_vs_float64(tl, tr):
    M, N, K = 37, 29, 300
    A = data.uniform((K, M) if tl else (M, K), -1, 1, 5, 0)
    B = data.uniform((N, K) if tr else (K, N), -1, 1, 5, 1)
    bias = data.uniform((N,), -1, 1, 5, 2)
    got = oracle.gemm(A, B, bias, M, N, K, tl, tr, threads=2)
    np.testing.assert_allclose(got, _gemm64(A, B, bias, tl, tr), rtol=1e-5, atol=1e-4)


def test_gemm_oracle_row_sample_equals_full():
    M, N, K = 20, 16, 64
    A, B, bias = data.uniform((M, K), -1, 1, 6, 0), data.uniform((K, N), -1, 1, 6, 1), data.uniform((N,), -1, 1, 6, 2)
    full = oracle.gemm(A, B, bias, M, N, K)
    assert np.array_equal(full[5:9], oracle.gemm(A, B, bias, M, N, K, rows=(5, 9)))


def _attention64(Q, K, V, scale):
    s = Q.astype(np.float64) @ K.astype(np.float64).T * scale
    s -= s.max(axis=1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=1, keepdims=True)
    return p @ V.astype(np.float64)


@pytest.mark.parametrize("R,C", [(1, 1), (7, 129), (64, 300)])
def test_attention_oracle_vs_float64(R, C):
    D = 128
    Q, K, V = (data.normal((1, 1, n, D), 1.0, 7, i) for i, n in enumerate((R, C, C)))
    got = oracle.attention(Q, K, V, 1, 1, 1, R, C, D, 1 / np.sqrt(D))
    np.testing.assert_allclose(got[0, 0], _attention64(Q[0, 0], K[0, 0], V[0, 0], 1 / np.sqrt(D)), rtol=1e-4,
                               atol=1e-5)


def _bhsd(a, layout):
    return np.ascontiguousarray(a if layout == 0 else a.transpose(0, 2, 1, 3)).astype(np.float64)


def _attention_loss64(Q, K, V, dO, group, scale):
    """Network.loss (Network.swift:313-326) in float64: sum over heads of dO * softmax(scale Q K^T) V,
    [B][H][S][D] arrays, query head h reading key/value head h // group."""
    total = 0.0
    B, Hq = Q.shape[:2]
    for b in range(B):
        for h in range(Hq):
            s = Q[b, h] @ K[b, h // group].T * scale
            s -= s.max(axis=1, keepdims=True)
            p = np.exp(s)
            p /= p.sum(axis=1, keepdims=True)
            total += float((dO[b, h] * (p @ V[b, h // group])).sum())
    return total


@pytest.mark.parametrize("layout", [0, 1])
def test_attention_bwd_oracle_vs_finite_differences(layout):
    """The backward oracle (Network.derivativeQ / derivativeK / derivativeV restated in C, fp32) against
    central finite differences of the float64 loss, every input element, grouped-query heads (4 query
    heads on 2 key/value heads), ragged R != C, both layouts; and its LSE against float64 logsumexp."""
    B, Hq, Hk, R, C, D = 1, 4, 2, 5, 7, 8
    scale = 1 / np.sqrt(D)
    shp = (lambda S, H: (B, H, S, D)) if layout == 0 else (lambda S, H: (B, S, H, D))
    Q = data.normal(shp(R, Hq), 1.0, 41, 0)
    K = data.normal(shp(C, Hk), 1.0, 41, 1)
    V = data.normal(shp(C, Hk), 1.0, 41, 2)
    dO = data.normal(shp(R, Hq), 1.0, 41, 3)
    dQ, dK, dV, lse = oracle.attention_bwd(Q, K, V, dO, B, Hq, Hk, R, C, D, scale, layout)
    q, k, v, g = (_bhsd(a, layout) for a in (Q, K, V, dO))
    group = Hq // Hk
    eps = 1e-4
    for name, base, grad in (("Q", q, dQ), ("K", k, dK), ("V", v, dV)):
        fd = np.zeros_like(base)
        for idx in np.ndindex(base.shape):
            args = {"Q": q, "K": k, "V": v}
            plus, minus = base.copy(), base.copy()
            plus[idx] += eps
            minus[idx] -= eps
            args[name] = plus
            lp = _attention_loss64(args["Q"], args["K"], args["V"], g, group, scale)
            args[name] = minus
            lm = _attention_loss64(args["Q"], args["K"], args["V"], g, group, scale)
            fd[idx] = (lp - lm) / (2 * eps)
        np.testing.assert_allclose(_bhsd(grad, layout), fd, rtol=1e-3, atol=2e-4, err_msg=f"d{name}")
    for b in range(B):
        for h in range(Hq):
            s = q[b, h] @ k[b, h // group].T * scale
            m = s.max(axis=1)
            ref = m + np.log(np.exp(s - m[:, None]).sum(axis=1))
            np.testing.assert_allclose(lse[b, h], ref, rtol=1e-5, atol=1e-5)


def _conv64(x, w_hwio, bias, pads, strides, dils):
    """NDHWC x [KD][KH][KW][C][O], float64, zero padding."""
    N, D, H, W, C = x.shape
    KD, KH, KW, _, O = w_hwio.shape
    (pf, pb), (pt, pbo), (pl, pr) = pads
    xp = np.zeros((N, D + pf + pb, H + pt + pbo, W + pl + pr, C))
    xp[:, pf:pf + D, pt:pt + H, pl:pl + W] = x.astype(np.float64)
    sz, sy, sx = strides
    dz, dy, dx = dils
    OD = (D + pf + pb - ((KD - 1) * dz + 1)) // sz + 1
    OH = (H + pt + pbo - ((KH - 1) * dy + 1)) // sy + 1
    OW = (W + pl + pr - ((KW - 1) * dx + 1)) // sx + 1
    out = np.zeros((N, OD, OH, OW, O))
    w = w_hwio.astype(np.float64)
    for kd in range(KD):
        for kh in range(KH):
            for kw in range(KW):
                sl = xp[:, kd * dz: kd * dz + (OD - 1) * sz + 1: sz, kh * dy: kh * dy + (OH - 1) * sy + 1: sy,
                        kw * dx: kw * dx + (OW - 1) * sx + 1: sx]
                out += np.einsum("ndhwc,co->ndhwo", sl, w[kd, kh, kw])
    if bias is not None:
        out += bias.astype(np.float64)
    return out


@pytest.mark.parametrize("case", CONV2D_VALID + CONV2D_PADDED)
def test_conv2d_oracle_vs_float64_reference_cases(case):
    d = case
    x = data.conv2d_activation(d.batchSize, d.inputHeight, d.inputWidth, d.inputChannels, d.outputChannels,
                               d.kernelHeight, d.kernelWidth)
    w = data.conv2d_weights_hwio(d.inputChannels, d.outputChannels, d.kernelHeight, d.kernelWidth)
    got = oracle.conv2d(x, w, None, layout=0, **oracle_kwargs2d(d))
    ref = _conv64(x[:, None], w[None], None, ((0, 0), (d.paddingTop, d.paddingBottom),
                                             (d.paddingLeft, d.paddingRight)),
                  (1, d.strideY, d.strideX), (1, d.dilationY, d.dilationX))[:, 0]
    np.testing.assert_allclose(got, ref, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("case", CONV3D_VALID + CONV3D_HW_PADDED + CONV3D_LR_PADDED)
def test_conv3d_oracle_vs_float64_reference_cases(case):
    d = case
    x = data.conv3d_activation(d.batchSize, d.inputDepth, d.inputHeight, d.inputWidth, d.inputChannels)
    w = data.conv3d_weights_dhwio(d.inputChannels, d.outputChannels, d.kernelDepth, d.kernelHeight, d.kernelWidth)
    b = data.conv3d_bias(d.outputChannels)
    got = oracle.conv3d(x, w, b, layout=3, **oracle_kwargs3d(d))
    ref = _conv64(x, w, b, ((d.paddingFront, d.paddingBack), (d.paddingTop, d.paddingBottom),
                            (d.paddingLeft, d.paddingRight)),
                  (d.strideZ, d.strideY, d.strideX), (d.dilationZ, d.dilationY, d.dilationX))
    np.testing.assert_allclose(got, ref, rtol=1e-6, atol=1e-6)


def test_conv3d_reference_data_outputs_are_exact_in_fp32():
    """The formula data are multiples of 2^-4 and 2^-5, so every product and
    partial sum of these cases is exact in fp32: the oracle must equal float64
    bit for bit (the recorded device outcome maxAbsoluteError = 0.0 for the
    D=4 33x35 C4->8 case, AGENTS.md:124, rests on this)."""
    d = CONV3D_HW_PADDED[4]
    x = data.conv3d_activation(d.batchSize, d.inputDepth, d.inputHeight, d.inputWidth, d.inputChannels)
    w = data.conv3d_weights_dhwio(d.inputChannels, d.outputChannels, d.kernelDepth, d.kernelHeight, d.kernelWidth)
    got = oracle.conv3d(x, w, None, layout=3, **oracle_kwargs3d(d))
    ref = _conv64(x, w, None, ((0, 0), (1, 1), (1, 1)), (1, 1, 1), (1, 1, 1))
    assert np.array_equal(got.astype(np.float64), ref)


@pytest.mark.parametrize("src,dst,kd", [(5, 3, 3), (5, 4, 3), (3, 4, 3), (2, 0, 1), (0, 1, 1), (1, 2, 1)])
def test_permute_oracle_vs_numpy(src, dst, kd):
    O, C, KH, KW = 5, 3, 3, 2
    w = data.normal((O * C * kd * KH * KW,), 1.0, 9, 0)
    order = {0: "hwio", 1: "ohwi", 2: "oihw", 3: "dhwio", 4: "odhwi", 5: "oidhw"}
    shapes = {"o": O, "i": C, "d": kd, "h": KH, "w": KW}
    s_ax, d_ax = order[src], order[dst]
    if kd == 1 and "d" not in s_ax:
        s_ax5, d_ax5 = "d" + s_ax, "d" + d_ax
    else:
        s_ax5, d_ax5 = s_ax, d_ax
    canon = w.reshape([shapes[a] for a in s_ax5])
    ref = np.transpose(canon, [s_ax5.index(a) for a in d_ax5]).reshape(-1)
    got = oracle.permute_weights(w, src, dst, O, C, kd, KH, KW)
    assert np.array_equal(got.view(np.uint16), ref.view(np.uint16))


# ------------------------------------------------------------------ golden fixtures

def test_golden_gemm_fixtures():
    z = np.load(GOLDEN / "gemm_small.npz")
    names = sorted({k.split("/")[0] for k in z.files})
    assert names
    for n in names:
        M, N, K, tl, tr = (int(v) for v in z[f"{n}/dims"])
        got = oracle.gemm(z[f"{n}/A"], z[f"{n}/B"], z[f"{n}/bias"], M, N, K, bool(tl), bool(tr))
        assert np.array_equal(got, z[f"{n}/out"]), n
        # the fixture inputs are the seeded generator's output
        np.testing.assert_allclose(z[f"{n}/out"], _gemm64(z[f"{n}/A"], z[f"{n}/B"], z[f"{n}/bias"], tl, tr),
                                   rtol=1e-5, atol=1e-4)


def test_golden_attention_fixtures():
    z = np.load(GOLDEN / "attention_small.npz")
    names = sorted({k.split("/")[0] for k in z.files})
    for n in names:
        B, Hq, Hk, R, C, layout, D = (int(v) for v in z[f"{n}/dims"])
        got = oracle.attention(z[f"{n}/Q"], z[f"{n}/K"], z[f"{n}/V"], B, Hq, Hk, R, C, D, 1 / np.sqrt(D),
                               layout)
        np.testing.assert_allclose(got, z[f"{n}/out"], rtol=1e-6, atol=1e-7)


def test_golden_attention_backward_fixtures():
    """The backward oracle reproduces its committed fixtures (regression pin; the finite-difference test
    above is the mathematical one)."""
    z = np.load(GOLDEN / "attention_bwd_small.npz")
    names = sorted({k.split("/")[0] for k in z.files})
    assert len(names) == 4
    for n in names:
        B, Hq, Hk, R, C, layout, D = (int(v) for v in z[f"{n}/dims"])
        got = oracle.attention_bwd(z[f"{n}/Q"], z[f"{n}/K"], z[f"{n}/V"], z[f"{n}/dO"], B, Hq, Hk, R, C, D,
                                   1 / np.sqrt(D), layout)
        for i, key in enumerate(("dQ", "dK", "dV", "lse")):
            np.testing.assert_allclose(got[i], z[f"{n}/{key}"], rtol=1e-6, atol=1e-7, err_msg=f"{n} {key}")
