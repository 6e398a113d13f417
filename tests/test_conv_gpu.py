"""Conv parity on the GPU: mm4 implicit-GEMM conv (through the C ABI) vs the
C oracle (ConvolutionShared.swift:4994-5096 restated), on the reference's own
validation cases with its formula data, and on the BASELINE shapes."""
import numpy as np
import pytest

import oracle
from cases import (CONV2D_PADDED, CONV2D_VALID, CONV3D_HW_PADDED, CONV3D_LR_PADDED, CONV3D_VALID, oracle_kwargs2d,
                   oracle_kwargs3d)
from example_matmul_metal4_b200 import data, sync_check
from example_matmul_metal4_b200.conv import (WEIGHTS_DHWIO, WEIGHTS_HWIO, WEIGHTS_ODHWI, WEIGHTS_OHWI,
                                             WEIGHTS_OIDHW, WEIGHTS_OIHW, Conv2DDimensions, Conv3DDimensions,
                                             ConvPlan, permute_weights)
from tolerance import assert_close

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _no_tf32():
    import torch
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False


def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _run2d(cuda, d, x, w_hwio, bias=None, layout=WEIGHTS_HWIO):
    w = w_hwio
    if layout == WEIGHTS_OHWI:
        w = np.ascontiguousarray(np.transpose(w_hwio, (3, 0, 1, 2)))
    plan = ConvPlan(d, weight_layout=layout, bias=bias is not None)
    y = plan.run(_t(x, cuda), _t(w, cuda), _t(bias, cuda) if bias is not None else None)
    sync_check()
    ref = oracle.conv2d(x, np.ascontiguousarray(w_hwio), bias, layout=0, threads=oracle.default_threads(),
                        **oracle_kwargs2d(d))
    return plan, y.float().cpu().numpy(), ref


@pytest.mark.parametrize("idx", range(len(CONV2D_VALID)))
@pytest.mark.parametrize("layout", [WEIGHTS_HWIO, WEIGHTS_OHWI])
def test_conv2d_reference_valid_cases(cuda, idx, layout):
    d = CONV2D_VALID[idx]
    x = data.conv2d_activation(d.batchSize, d.inputHeight, d.inputWidth, d.inputChannels, d.outputChannels,
                               d.kernelHeight, d.kernelWidth)
    w = data.conv2d_weights_hwio(d.inputChannels, d.outputChannels, d.kernelHeight, d.kernelWidth)
    plan, got, ref = _run2d(cuda, d, x, w, layout=layout)
    assert_close(got, ref, f"conv2d valid case {idx} {plan.kernel_name}")


def test_conv2d_identity_kat(cuda):
    """1-channel ramp with a centre tap: the valid 3x3 conv of a 5x5 ramp picks
    the centre 3x3 of the ramp (ConvolutionShared.swift:4876-4893)."""
    d = CONV2D_VALID[0]
    x = data.conv2d_activation(1, 5, 5, 1, 1, 3, 3)
    w = data.conv2d_weights_hwio(1, 1, 3, 3)
    plan, got, ref = _run2d(cuda, d, x, w)
    expected = np.arange(1, 26, dtype=np.float32).reshape(5, 5)[1:4, 1:4]
    assert np.array_equal(got.reshape(3, 3), expected)


@pytest.mark.parametrize("idx", range(len(CONV2D_PADDED)))
def test_conv2d_reference_padded_cases(cuda, idx):
    d = CONV2D_PADDED[idx]
    x = data.padded_conv2d_activation(1, d.inputHeight, d.inputWidth, d.inputChannels)
    w = data.padded_conv2d_weights_hwio(d.inputChannels, d.outputChannels, d.kernelHeight, d.kernelWidth)
    plan, got, ref = _run2d(cuda, d, x, w)
    assert_close(got, ref, f"conv2d padded case {idx}")


def _run3d(cuda, d, x, w_dhwio, bias=None, layout=WEIGHTS_DHWIO):
    w = w_dhwio
    if layout == WEIGHTS_ODHWI:
        w = np.ascontiguousarray(np.transpose(w_dhwio, (4, 0, 1, 2, 3)))
    plan = ConvPlan(d, weight_layout=layout, bias=bias is not None)
    y = plan.run(_t(x, cuda), _t(w, cuda), _t(bias, cuda) if bias is not None else None)
    sync_check()
    ref = oracle.conv3d(x, np.ascontiguousarray(w_dhwio), bias, layout=3, threads=oracle.default_threads(),
                        **oracle_kwargs3d(d))
    return plan, y.float().cpu().numpy(), ref


def _data3d(d):
    x = data.conv3d_activation(d.batchSize, d.inputDepth, d.inputHeight, d.inputWidth, d.inputChannels)
    w = data.conv3d_weights_dhwio(d.inputChannels, d.outputChannels, d.kernelDepth, d.kernelHeight, d.kernelWidth)
    return x, w


@pytest.mark.parametrize("idx", range(len(CONV3D_VALID)))
@pytest.mark.parametrize("with_bias", [False, True])
def test_conv3d_reference_cases(cuda, idx, with_bias):
    d = CONV3D_VALID[idx]
    x, w = _data3d(d)
    b = data.conv3d_bias(d.outputChannels) if with_bias else None
    plan, got, ref = _run3d(cuda, d, x, w, b)
    assert_close(got, ref, f"conv3d case {idx} bias={with_bias}")


@pytest.mark.parametrize("idx", range(len(CONV3D_HW_PADDED)))
@pytest.mark.parametrize("layout", [WEIGHTS_DHWIO, WEIGHTS_ODHWI])
def test_conv3d_reference_padded_cases(cuda, idx, layout):
    d = CONV3D_HW_PADDED[idx]
    x, w = _data3d(d)
    plan, got, ref = _run3d(cuda, d, x, w, layout=layout)
    v = assert_close(got, ref, f"conv3d padded case {idx}")
    # The reference's recorded device outcomes (AGENTS.md:123-124): N=1 D=5 17x19 C8->12 gave
    # maxAbsoluteError 0.001953125 and N=1 D=4 33x35 C4->8 gave 0.0, both with 0 mismatches. The formula
    # data are multiples of 1/32, so the fp32 sums are exact and the only error left is the one rounding
    # to fp16: the kernel's output is the oracle's rounded bit for bit, and the recorded bounds hold as
    # written.
    if idx == 3:
        assert v["maxAbsoluteError"] <= 0.001953125 and v["mismatches"] == 0, v
    if idx == 4:
        assert v["maxAbsoluteError"] == 0.0 and v["mismatches"] == 0, v
    if idx in (3, 4):
        np.testing.assert_array_equal(got.astype(np.float16), oracle.to_half(ref))


@pytest.mark.parametrize("idx", range(len(CONV3D_LR_PADDED)))
@pytest.mark.parametrize("layout", [WEIGHTS_DHWIO, WEIGHTS_ODHWI])
def test_conv3d_left_right_padding_probe(cuda, idx, layout):
    """The left/right-only padding probe cases (convolution3d_padding.swift:676-742)."""
    d = CONV3D_LR_PADDED[idx]
    x, w = _data3d(d)
    plan, got, ref = _run3d(cuda, d, x, w, layout=layout)
    assert_close(got, ref, f"conv3d L/R padding probe case {idx} {plan.kernel_name}")


def test_conv3d_depth_padding_extension(cuda):
    d = Conv3DDimensions(1, 6, 9, 11, 16, 24, 3, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1)
    x = data.normal((1, 6, 9, 11, 16), 1.0, 5, 0)
    w = data.normal((3, 3, 3, 16, 24), 0.03, 5, 1)
    b = data.uniform((24,), -0.1, 0.1, 5, 2)
    for layout in (WEIGHTS_DHWIO, WEIGHTS_ODHWI):
        plan, got, ref = _run3d(cuda, d, x, w, b, layout=layout)
        assert "tma" in plan.kernel_name
        assert_close(got, ref, f"conv3d depth padding {plan.kernel_name}")


@pytest.mark.parametrize("C,O", [(24, 40), (64, 64), (72, 136), (128, 264)])
def test_conv2d_channel_blocks(cuda, C, O):
    """Cin not a multiple of 64 (partial channel slab), Cout tails, both layouts."""
    d = Conv2DDimensions(2, 13, 15, C, O, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1)
    x = data.normal((2, 13, 15, C), 1.0, 4, 0)
    w = data.normal((3, 3, C, O), 0.05, 4, 1)
    b = data.uniform((O,), -0.1, 0.1, 4, 2)
    for layout in (WEIGHTS_HWIO, WEIGHTS_OHWI):
        plan, got, ref = _run2d(cuda, d, x, w, b, layout=layout)
        assert_close(got, ref, f"C={C} O={O} {plan.kernel_name}")


def test_conv2d_strided_dilated_aligned(cuda):
    d = Conv2DDimensions(3, 20, 23, 32, 48, 3, 3, 2, 2, 2, 2, 2, 1, 0, 2)
    x = data.normal((3, 20, 23, 32), 1.0, 6, 0)
    w = data.normal((3, 3, 32, 48), 0.05, 6, 1)
    plan, got, ref = _run2d(cuda, d, x, w)
    assert_close(got, ref, "strided dilated asymmetric padding")


@pytest.mark.parametrize("mode", ["im2col", "rect"])
def test_stride1_activation_paths(cuda, mode, monkeypatch):
    """Stride-1 convs with 16-byte channels load activations by TMA: im2col
    tiles of 128 consecutive output pixels (default) or TH x TW rectangles
    (MM4_CONV_ACTIVATIONS=rect). Dilation, asymmetric and depth padding, tiles
    that cross rows and images, ragged last tile."""
    if mode == "rect":
        monkeypatch.setenv("MM4_CONV_ACTIVATIONS", "rect")
    else:
        monkeypatch.delenv("MM4_CONV_ACTIVATIONS", raising=False)
    d = Conv2DDimensions(3, 19, 21, 32, 48, 3, 3, 1, 1, 2, 2, 2, 1, 0, 2)
    x = data.normal((3, 19, 21, 32), 1.0, 7, 0)
    w = data.normal((3, 3, 32, 48), 0.05, 7, 1)
    b = data.uniform((48,), -0.1, 0.1, 7, 2)
    for layout in (WEIGHTS_HWIO, WEIGHTS_OHWI):
        plan, got, ref = _run2d(cuda, d, x, w, b, layout=layout)
        assert f"tma-{mode}" in plan.kernel_name, plan.kernel_name
        assert_close(got, ref, f"conv2d stride 1 {plan.kernel_name}")
    d3 = Conv3DDimensions(2, 5, 9, 11, 16, 24, 3, 3, 3, 1, 1, 1, 1, 1, 1, 2, 0, 1, 1, 1, 0)
    x3 = data.normal((2, 5, 9, 11, 16), 1.0, 8, 0)
    w3 = data.normal((3, 3, 3, 16, 24), 0.03, 8, 1)
    b3 = data.uniform((24,), -0.1, 0.1, 8, 2)
    plan, got, ref = _run3d(cuda, d3, x3, w3, b3, layout=WEIGHTS_DHWIO)
    assert f"tma-{mode}" in plan.kernel_name, plan.kernel_name
    assert_close(got, ref, f"conv3d stride 1 {plan.kernel_name}")


TAP_ROW_2D = [
    # (dims, x seed) -- KW 3 with left-only padding, ragged channel slab, BN 256 (O = 136)
    Conv2DDimensions(3, 19, 21, 72, 136, 3, 3, 1, 1, 1, 1, 1, 0, 2, 0),
    # KW 2, right padding only, one channel slab
    Conv2DDimensions(2, 17, 30, 32, 48, 2, 2, 1, 1, 1, 1, 1, 0, 0, 1),
    # dilated in H only (tap rows need dilation 1 in W)
    Conv2DDimensions(2, 15, 13, 24, 40, 3, 3, 1, 1, 2, 1, 2, 2, 1, 1),
]


@pytest.mark.parametrize("taprow", [True, False])
@pytest.mark.parametrize("idx", range(len(TAP_ROW_2D)))
def test_tap_rows(cuda, idx, taprow, monkeypatch):
    """Pair-path convs whose KW taps all read one activation box per (kd, kh,
    channel slab) (default), against one box per tap (MM4_CONV_TAPREUSE=0):
    virtual rows OW + KW - 1 wide, the overhang columns dropped in the
    epilogue, tiles crossing rows and images, ragged last tile."""
    if taprow:
        monkeypatch.delenv("MM4_CONV_TAPREUSE", raising=False)
    else:
        monkeypatch.setenv("MM4_CONV_TAPREUSE", "0")
    d = TAP_ROW_2D[idx]
    x = data.normal((d.batchSize, d.inputHeight, d.inputWidth, d.inputChannels), 1.0, 30 + idx, 0)
    w = data.normal((d.kernelHeight, d.kernelWidth, d.inputChannels, d.outputChannels), 0.05, 30 + idx, 1)
    b = data.uniform((d.outputChannels,), -0.1, 0.1, 30 + idx, 2)
    for layout in (WEIGHTS_HWIO, WEIGHTS_OHWI):
        plan, got, ref = _run2d(cuda, d, x, w, b, layout=layout)
        assert ("taprow" in plan.kernel_name) == taprow, plan.kernel_name
        assert_close(got, ref, f"conv2d tap rows case {idx} {plan.kernel_name}")
    if idx == 0:
        d3 = Conv3DDimensions(2, 5, 9, 11, 16, 24, 3, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 0)
        x3 = data.normal((2, 5, 9, 11, 16), 1.0, 9, 0)
        w3 = data.normal((3, 3, 3, 16, 24), 0.03, 9, 1)
        b3 = data.uniform((24,), -0.1, 0.1, 9, 2)
        for layout in (WEIGHTS_DHWIO, WEIGHTS_ODHWI):
            plan, got, ref = _run3d(cuda, d3, x3, w3, b3, layout=layout)
            assert ("taprow" in plan.kernel_name) == taprow, plan.kernel_name
            assert_close(got, ref, f"conv3d tap rows {plan.kernel_name}")


def test_baseline_config4_conv2d(cuda):
    """N=32, 56x56, 256->256, 3x3, pad 1, OHWI weights
    N(0,0.05), bias U[-0.1,0.1]. Oracle on a row sample; every output checked
    against an fp32 cuDNN conv as a second reference."""
    import torch
    d = Conv2DDimensions(32, 56, 56, 256, 256, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1)
    x = data.normal((32, 56, 56, 256), 1.0, 4, 0)
    w_ohwi = data.normal((256, 3, 3, 256), 0.05, 4, 1)
    b = data.uniform((256,), -0.1, 0.1, 4, 2)
    plan = ConvPlan(d, weight_layout=WEIGHTS_OHWI, bias=True)
    tx, tw, tb = _t(x, cuda), _t(w_ohwi, cuda), _t(b, cuda)
    y = plan.run(tx, tw, tb)
    sync_check()
    got = y.float().cpu().numpy()
    rows = [(0, 2), (55, 58), (900, 902), (32 * 56 - 2, 32 * 56)]
    for r0, r1 in rows:
        ref = oracle.conv2d(x, w_ohwi, b, layout=1, rows=(r0, r1), threads=oracle.default_threads(),
                            **oracle_kwargs2d(d))
        assert_close(got.reshape(-1, 56, 256)[r0:r1], ref, f"rows {r0}:{r1}")
    ref_t = torch.nn.functional.conv2d(tx.permute(0, 3, 1, 2).float(), tw.permute(0, 3, 1, 2).float(),
                                       tb.float(), padding=1).permute(0, 2, 3, 1)
    assert_close(got, ref_t.cpu().numpy(), "full output vs fp32 cuDNN")


def test_baseline_config5_conv3d(cuda):
    """N=8, D=16, 64x64, 128->128, 3x3x3, pad 1 in D/H/W,
    ODHWI weights N(0,0.03), bias U[-0.1,0.1]."""
    import torch
    d = Conv3DDimensions(8, 16, 64, 64, 128, 128, 3, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1)
    x = data.normal((8, 16, 64, 64, 128), 1.0, 5, 0)
    w = data.normal((128, 3, 3, 3, 128), 0.03, 5, 1)
    b = data.uniform((128,), -0.1, 0.1, 5, 2)
    plan = ConvPlan(d, weight_layout=WEIGHTS_ODHWI, bias=True)
    tx, tw, tb = _t(x, cuda), _t(w, cuda), _t(b, cuda)
    y = plan.run(tx, tw, tb)
    sync_check()
    got = y.float().cpu().numpy()
    for r0, r1 in [(0, 2), (64 * 16 - 1, 64 * 16 + 1), (8 * 16 * 64 - 2, 8 * 16 * 64)]:
        ref = oracle.conv3d(x, w, b, layout=4, rows=(r0, r1), threads=oracle.default_threads(),
                            **oracle_kwargs3d(d))
        assert_close(got.reshape(-1, 64, 128)[r0:r1], ref, f"rows {r0}:{r1}")
    ref_t = torch.nn.functional.conv3d(tx.permute(0, 4, 1, 2, 3).float(), tw.permute(0, 4, 1, 2, 3).float(),
                                       tb.float(), padding=1).permute(0, 2, 3, 4, 1)
    assert_close(got, ref_t.cpu().numpy(), "full output vs fp32 cuDNN")


@pytest.mark.parametrize("src,dst,kd", [(WEIGHTS_OIDHW, WEIGHTS_DHWIO, 3), (WEIGHTS_OIDHW, WEIGHTS_ODHWI, 3),
                                        (WEIGHTS_DHWIO, WEIGHTS_ODHWI, 3), (WEIGHTS_OIHW, WEIGHTS_HWIO, 1),
                                        (WEIGHTS_HWIO, WEIGHTS_OHWI, 1)])
def test_permute_weights_exact(cuda, src, dst, kd):
    """K10 permute_oidhw_to_dhwio and friends: bit-exact (ConvolutionShared.swift:5381-5406 uses tolerance 0)."""
    O, C, KH, KW = 12, 8, 3, 3
    w = data.normal((O * C * kd * KH * KW,), 1.0, 9, 0)
    got = permute_weights(_t(w, cuda), src, dst, (O, C, kd, KH, KW))
    sync_check()
    ref = oracle.permute_weights(w, src, dst, O, C, kd, KH, KW)
    assert np.array_equal(got.cpu().numpy().view(np.uint16), ref.view(np.uint16))


@pytest.mark.parametrize("three_d,chunks", [(False, 3), (True, 2), (False, 64)])
def test_host_buffer_conv_matches_device_conv(cuda, three_d, chunks):
    """mm4_conv_run_host (images copied in, convolved and copied out in batch chunks, ragged last chunk)
    writes the same bits as mm4_conv_run on device buffers."""
    import torch
    if three_d:
        d = Conv3DDimensions(5, 4, 12, 12, 64, 64, 3, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1)
        plan = ConvPlan(d, weight_layout=WEIGHTS_ODHWI, bias=True)
        w_shape = (64, 3, 3, 3, 64)
    else:
        d = Conv2DDimensions(7, 20, 20, 64, 128, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1)
        plan = ConvPlan(d, weight_layout=WEIGHTS_OHWI, bias=True)
        w_shape = (128, 3, 3, 64)
    x = torch.from_numpy(data.normal(plan.in_shape, 1.0, 6, 0)).pin_memory()
    w = torch.from_numpy(data.normal(w_shape, 0.05, 6, 1)).pin_memory()
    b = torch.from_numpy(data.uniform((d.outputChannels,), -0.1, 0.1, 6, 2)).pin_memory()
    y = torch.empty(plan.out_shape, dtype=torch.float16).pin_memory()
    staging = (torch.empty_like(x, device=cuda), torch.empty_like(w, device=cuda), torch.empty_like(b, device=cuda),
               torch.empty(plan.out_shape, dtype=torch.float16, device=cuda))
    plan.run_host(x, w, b, y, staging, chunks=chunks)
    torch.cuda.current_stream().synchronize()
    sync_check()
    ref = plan.run(x.to(cuda), w.to(cuda), b.to(cuda))
    sync_check()
    assert torch.equal(y, ref.cpu())
