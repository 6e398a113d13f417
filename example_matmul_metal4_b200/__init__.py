"""B200-native (sm_100a) tensor-op contraction path of liuliu/example_matmul_metal4.

GEMM (+bias, split-K, dynamic K), flash-attention forward and conv2d/conv3d
as hand-written tcgen05/TMA kernels in libmm4.so behind the C ABI of
include/mm4.h. This package is the Python host side: descriptor types named
after the reference's Swift structs and thin wrappers over the C entry
points. There is no CPU fallback.
"""
from ._lib import MM4Error, lib, sync_check  # noqa: F401
from .gemm import BuildOptions, GEMMDimensions, GemmPlan, splitk_finalize  # noqa: F401

__all__ = ["MM4Error", "lib", "sync_check", "BuildOptions", "GEMMDimensions", "GemmPlan", "splitk_finalize"]
