"""Python access to the C oracle (oracle/mm4_oracle.c) — TEST INFRASTRUCTURE ONLY.

Used by tests/, `__graft_entry__.smoke()` and the `cpu_baseline` / reference
arm of bench.py, and nothing else. Inputs are numpy float16 arrays; outputs
are float32 arrays of the fp32-accumulated reference result.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libmm4_oracle.so"

_lib = None
_u16p = ctypes.POINTER(ctypes.c_uint16)
_f32p = ctypes.POINTER(ctypes.c_float)
_i = ctypes.c_int


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        h = ctypes.CDLL(str(LIB_PATH))
        h.mm4o_gemm.argtypes = [_i, _i, _i, _u16p, _u16p, _u16p, _i, _i, _f32p, _i, _i, _i]
        h.mm4o_attention.argtypes = [_i, _i, _i, _i, _i, _i, ctypes.c_float, _i, _u16p, _u16p, _u16p, _f32p, _i,
                                     _i, _i, _f32p]
        h.mm4o_attention_bwd.argtypes = [_i, _i, _i, _i, _i, _i, ctypes.c_float, _i, _u16p, _u16p, _u16p, _u16p,
                                         _f32p, _f32p, _f32p, _f32p, _i, _f32p]
        h.mm4o_conv3d.argtypes = [_i] * 22 + [_u16p, _u16p, _u16p, _f32p, ctypes.c_int64, ctypes.c_int64, _i]
        h.mm4o_permute_weights.argtypes = [_i, _i, _i, _i, _i, _i, _i, _u16p, _u16p]
        h.mm4o_half_to_float.argtypes = [ctypes.c_uint16]
        h.mm4o_half_to_float.restype = ctypes.c_float
        h.mm4o_float_to_half.argtypes = [ctypes.c_float]
        h.mm4o_float_to_half.restype = ctypes.c_uint16
        h.mm4o_float_to_half_array.argtypes = [_f32p, _u16p, ctypes.c_int64]
        h.mm4o_max_threads.restype = ctypes.c_int
        _lib = h
    return _lib


def max_threads() -> int:
    return int(lib().mm4o_max_threads())


def _h(a: np.ndarray | None):
    if a is None:
        return None
    assert a.dtype == np.float16 and a.flags.c_contiguous
    return a.ctypes.data_as(_u16p)


def to_half(x: np.ndarray) -> np.ndarray:
    """fp32 -> fp16 with the oracle's round-to-nearest-even."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().mm4o_float_to_half_array(x.ctypes.data_as(_f32p), out.ctypes.data_as(_u16p), x.size)
    return out.view(np.float16)


def gemm(A: np.ndarray, B: np.ndarray, bias: np.ndarray | None, M: int, N: int, K: int, transpose_left: bool = False,
         transpose_right: bool = False, rows: tuple[int, int] | None = None, threads: int = 1) -> np.ndarray:
    """fp32 reference of matmul.swift:499-510 for rows [r0, r1): shape (r1-r0, N)."""
    r0, r1 = rows if rows else (0, M)
    out = np.empty((r1 - r0, N), dtype=np.float32)
    lib().mm4o_gemm(M, N, K, _h(A), _h(B), _h(bias), int(transpose_left), int(transpose_right),
                    out.ctypes.data_as(_f32p), r0, r1, threads)
    return out


def attention(Q: np.ndarray, K: np.ndarray, V: np.ndarray, batch: int, heads_q: int, heads_kv: int, R: int, C: int,
              D: int, scale: float, layout: int = 0, rows: tuple[int, int] | None = None,
              threads: int = 1) -> np.ndarray:
    """fp32 reference of Network.inferenceAttention: shape (batch, heads_q, r1-r0, D)."""
    r0, r1 = rows if rows else (0, R)
    out = np.empty((batch, heads_q, r1 - r0, D), dtype=np.float32)
    nthreads = max(1, threads)
    scratch = np.empty(nthreads * C, dtype=np.float32)
    lib().mm4o_attention(batch, heads_q, heads_kv, R, C, D, float(scale), layout, _h(Q), _h(K), _h(V),
                         out.ctypes.data_as(_f32p), r0, r1, nthreads, scratch.ctypes.data_as(_f32p))
    return out


def attention_bwd(Q: np.ndarray, K: np.ndarray, V: np.ndarray, dO: np.ndarray, batch: int, heads_q: int,
                  heads_kv: int, R: int, C: int, D: int, scale: float, layout: int = 0, threads: int = 1):
    """fp32 reference of Network.derivativeQ / derivativeK / derivativeV (and createLTerm): returns
    (dQ, dK, dV, lse) with dQ/dK/dV shaped like Q/K/V and lse shaped (batch, heads_q, R)."""
    nthreads = max(1, threads)
    dQ = np.empty(Q.shape, dtype=np.float32)
    dK = np.empty(K.shape, dtype=np.float32)
    dV = np.empty(V.shape, dtype=np.float32)
    lse = np.empty((batch, heads_q, R), dtype=np.float32)
    scratch = np.empty(nthreads * (2 * C + D), dtype=np.float32)
    f = lambda a: a.ctypes.data_as(_f32p)  # noqa: E731
    lib().mm4o_attention_bwd(batch, heads_q, heads_kv, R, C, D, float(scale), layout, _h(Q), _h(K), _h(V), _h(dO),
                             f(dQ), f(dK), f(dV), f(lse), nthreads, f(scratch))
    return dQ, dK, dV, lse


def conv_out_size(inp: int, pad_lo: int, pad_hi: int, k: int, stride: int, dil: int) -> int:
    return (inp + pad_lo + pad_hi - ((k - 1) * dil + 1)) // stride + 1


def conv3d(x: np.ndarray, w: np.ndarray, bias: np.ndarray | None, *, N, D, H, W, C, O, KD, KH, KW, SZ=1, SY=1, SX=1,
           DZ=1, DY=1, DX=1, pad_front=0, pad_back=0, pad_top=0, pad_bottom=0, pad_left=0, pad_right=0, layout=3,
           rows: tuple[int, int] | None = None, threads: int = 1) -> np.ndarray:
    """fp32 reference of ConvolutionShared.swift:4994-5096 (NDHWC, NDHWC out).

    Returns shape (rows, OW, O) over flattened (n, oz, oh) rows, or the full
    (N, OD, OH, OW, O) output when `rows` is None.
    """
    OD = conv_out_size(D, pad_front, pad_back, KD, SZ, DZ)
    OH = conv_out_size(H, pad_top, pad_bottom, KH, SY, DY)
    OW = conv_out_size(W, pad_left, pad_right, KW, SX, DX)
    total = N * OD * OH
    r0, r1 = rows if rows else (0, total)
    out = np.empty((r1 - r0, OW, O), dtype=np.float32)
    lib().mm4o_conv3d(N, D, H, W, C, O, KD, KH, KW, SZ, SY, SX, DZ, DY, DX, pad_front, pad_top, pad_left, OD, OH, OW,
                      layout, _h(x), _h(w), _h(bias), out.ctypes.data_as(_f32p), r0, r1, threads)
    if rows is None:
        return out.reshape(N, OD, OH, OW, O)
    return out


def conv2d(x: np.ndarray, w: np.ndarray, bias: np.ndarray | None, *, N, H, W, C, O, KH, KW, SY=1, SX=1, DY=1, DX=1,
           pad_top=0, pad_bottom=0, pad_left=0, pad_right=0, layout=0, rows=None, threads: int = 1) -> np.ndarray:
    """conv2d = conv3d with D = KD = 1 (weight layouts 0..2 are the 2-D ones)."""
    out = conv3d(x, w, bias, N=N, D=1, H=H, W=W, C=C, O=O, KD=1, KH=KH, KW=KW, SY=SY, SX=SX, DY=DY, DX=DX,
                 pad_top=pad_top, pad_bottom=pad_bottom, pad_left=pad_left, pad_right=pad_right, layout=layout,
                 rows=rows, threads=threads)
    if rows is None:
        return out.reshape(out.shape[0], out.shape[2], out.shape[3], out.shape[4])
    return out


def permute_weights(src: np.ndarray, from_layout: int, to_layout: int, O: int, C: int, KD: int, KH: int,
                    KW: int) -> np.ndarray:
    dst = np.empty(src.size, dtype=np.float16)
    lib().mm4o_permute_weights(from_layout, to_layout, O, C, KD, KH, KW, _h(np.ascontiguousarray(src).reshape(-1)),
                               _h(dst))
    return dst


def default_threads() -> int:
    return max(1, min(max_threads(), int(os.environ.get("MM4_ORACLE_THREADS", "0")) or max_threads()))
