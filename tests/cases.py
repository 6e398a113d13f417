"""The reference's own validation case lists.

conv2d valid cases, conv3d cases and the conv3d left/right (H/W) padding
cases come from ConvolutionHarness (the defaults of
ConvolutionShared.swift:2143-2211, :2693-2764, :2770-2878), which restates
them; the padded conv2d probe cases (convolution2d_padding.swift:313-388) and
the conv3d left/right-only padding probe cases
(convolution3d_padding.swift:676-742) are restated here.
"""
from example_matmul_metal4_b200.conv import Conv2DDimensions, Conv3DDimensions  # noqa: F401
from example_matmul_metal4_b200.harness import ConvolutionHarness

CONV2D_VALID = ConvolutionHarness.defaultValidationCases()

CONV2D_PADDED = [
    Conv2DDimensions(1, 5, 5, 1, 1, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1),
    Conv2DDimensions(1, 5, 5, 4, 8, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1),
    Conv2DDimensions(1, 17, 19, 8, 12, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1),
    Conv2DDimensions(1, 33, 35, 4, 8, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1),
]

CONV3D_VALID = ConvolutionHarness.defaultTensorOpConv3DValidationCases()

CONV3D_HW_PADDED = ConvolutionHarness.defaultTensorOpConv3DLeftRightPaddingValidationCases()

# The left/right-padding probe (convolution3d_padding.swift:676-742): pad 1 on W only, none on H or D;
# the same data formulas (:186-200) and CPU loop (:202-242) as the shared conv3d code.
CONV3D_LR_PADDED = [
    Conv3DDimensions(1, 5, 5, 5, 1, 1, 3, 3, 3, 1, 1, 1, 1, 1, 1, 0, 0, 1, 1),
    Conv3DDimensions(1, 4, 5, 5, 4, 8, 3, 3, 3, 1, 1, 1, 1, 1, 1, 0, 0, 1, 1),
    Conv3DDimensions(2, 7, 6, 7, 3, 5, 3, 3, 3, 2, 1, 1, 1, 1, 1, 0, 0, 1, 1),
]


def oracle_kwargs2d(d: Conv2DDimensions):
    return dict(N=d.batchSize, H=d.inputHeight, W=d.inputWidth, C=d.inputChannels, O=d.outputChannels,
                KH=d.kernelHeight, KW=d.kernelWidth, SY=d.strideY, SX=d.strideX, DY=d.dilationY, DX=d.dilationX,
                pad_top=d.paddingTop, pad_bottom=d.paddingBottom, pad_left=d.paddingLeft, pad_right=d.paddingRight)


def oracle_kwargs3d(d: Conv3DDimensions):
    return dict(N=d.batchSize, D=d.inputDepth, H=d.inputHeight, W=d.inputWidth, C=d.inputChannels,
                O=d.outputChannels, KD=d.kernelDepth, KH=d.kernelHeight, KW=d.kernelWidth, SZ=d.strideZ, SY=d.strideY,
                SX=d.strideX, DZ=d.dilationZ, DY=d.dilationY, DX=d.dilationX, pad_front=d.paddingFront,
                pad_back=d.paddingBack, pad_top=d.paddingTop, pad_bottom=d.paddingBottom, pad_left=d.paddingLeft,
                pad_right=d.paddingRight)
