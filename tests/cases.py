"""The reference's own validation case lists, restated as data.

conv2d valid cases: ConvolutionHarness.defaultValidationCases
(ConvolutionShared.swift:2143-2211); padded conv2d probe cases
(convolution2d_padding.swift:313-388); conv3d cases
defaultTensorOpConv3DValidationCases (ConvolutionShared.swift:2693-2764) and
the left/right (H/W) padding cases (:2770-2878).
"""
from example_matmul_metal4_b200.conv import Conv2DDimensions, Conv3DDimensions

CONV2D_VALID = [
    Conv2DDimensions(1, 5, 5, 1, 1, 3, 3, 1, 1, 1, 1),
    Conv2DDimensions(1, 5, 5, 4, 8, 3, 3, 1, 1, 1, 1),
    Conv2DDimensions(1, 6, 7, 3, 5, 3, 3, 1, 1, 1, 1),
    Conv2DDimensions(1, 7, 8, 3, 4, 3, 3, 2, 2, 1, 1),
    Conv2DDimensions(1, 9, 10, 2, 3, 3, 3, 1, 1, 2, 2),
]

CONV2D_PADDED = [
    Conv2DDimensions(1, 5, 5, 1, 1, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1),
    Conv2DDimensions(1, 5, 5, 4, 8, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1),
    Conv2DDimensions(1, 17, 19, 8, 12, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1),
    Conv2DDimensions(1, 33, 35, 4, 8, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1),
]

CONV3D_VALID = [
    Conv3DDimensions(1, 5, 5, 5, 1, 1, 3, 3, 3, 1, 1, 1, 1, 1, 1),
    Conv3DDimensions(1, 4, 5, 5, 4, 8, 3, 3, 3, 1, 1, 1, 1, 1, 1),
    Conv3DDimensions(2, 7, 6, 7, 3, 5, 3, 3, 3, 2, 1, 1, 1, 1, 1),
    Conv3DDimensions(1, 7, 7, 7, 2, 3, 3, 3, 3, 1, 1, 1, 2, 2, 2),
]

CONV3D_HW_PADDED = [
    Conv3DDimensions(1, 5, 5, 5, 1, 1, 3, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1),
    Conv3DDimensions(1, 4, 5, 5, 4, 8, 3, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1),
    Conv3DDimensions(2, 7, 6, 7, 3, 5, 3, 3, 3, 2, 1, 1, 1, 1, 1, 1, 1, 1, 1),
    Conv3DDimensions(1, 5, 17, 19, 8, 12, 3, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1),
    Conv3DDimensions(1, 4, 33, 35, 4, 8, 3, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1),
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
