"""Seeded synthetic inputs, rounded once to fp16.

- `uniform` / `normal`: counter-based Philox-4x32-10 (Salmon, Moraes, Dror,
  Shaw, "Parallel random numbers: as easy as 1, 2, 3", SC'11) keyed by
  (seed, tensor id), so every element is a pure function of
  (seed, tensor id, index) — the same values in every process and on every
  rank. Normals use the Box-Muller transform, as the reference's attention
  inputs do (Network.swift:115-129); sigma is the standard deviation.
- `conv*_activation` / `conv*_weights` / `conv3d_bias`: the reference's
  deterministic formula generators used by its conv validation suites
  (ConvolutionShared.swift:4874-4992, convolution2d_padding.swift:65-77).

All generators return numpy float16 arrays.
"""
from __future__ import annotations

import numpy as np

_M0 = np.uint64(0xD2511F53)
_M1 = np.uint64(0xCD9E8D57)
_W0 = np.uint32(0x9E3779B9)
_W1 = np.uint32(0xBB67AE85)
_MASK32 = np.uint64(0xFFFFFFFF)


def philox4x32_10(c0, c1, c2, c3, k0: int, k1: int) -> tuple[np.ndarray, ...]:
    """Philox-4x32-10 block function on uint32 counter arrays (c0..c3) and key (k0, k1)."""
    c0, c1, c2, c3 = (np.asarray(c, dtype=np.uint32) for c in (c0, c1, c2, c3))
    k0 &= 0xFFFFFFFF
    k1 &= 0xFFFFFFFF
    for _ in range(10):
        p0 = c0.astype(np.uint64) * _M0
        p1 = c2.astype(np.uint64) * _M1
        hi0 = (p0 >> np.uint64(32)).astype(np.uint32)
        lo0 = (p0 & _MASK32).astype(np.uint32)
        hi1 = (p1 >> np.uint64(32)).astype(np.uint32)
        lo1 = (p1 & _MASK32).astype(np.uint32)
        c0, c1, c2, c3 = hi1 ^ c1 ^ np.uint32(k0), lo1, hi0 ^ c3 ^ np.uint32(k1), lo0
        k0 = (k0 + int(_W0)) & 0xFFFFFFFF
        k1 = (k1 + int(_W1)) & 0xFFFFFFFF
    return c0, c1, c2, c3


def philox4x32(counter_lo: np.ndarray, counter_hi: np.ndarray, tensor_id: int, seed: int) -> tuple[np.ndarray, ...]:
    """Philox-4x32-10 on counters (lo, hi, tensor_id, 0) with key (seed, seed >> 32)."""
    lo = np.asarray(counter_lo, dtype=np.uint32)
    return philox4x32_10(lo, counter_hi, np.full_like(lo, np.uint32(tensor_id & 0xFFFFFFFF)), np.zeros_like(lo),
                         seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF)


def _random_words(n: int, tensor_id: int, seed: int) -> np.ndarray:
    """n uint32 words: word i is lane i%4 of the Philox block at counter i//4."""
    blocks = (n + 3) // 4
    idx = np.arange(blocks, dtype=np.uint64)
    lo = (idx & _MASK32).astype(np.uint32)
    hi = (idx >> np.uint64(32)).astype(np.uint32)
    w = np.stack(philox4x32(lo, hi, tensor_id, seed), axis=1).reshape(-1)
    return w[:n]


def _unit(words: np.ndarray) -> np.ndarray:
    """uint32 -> float64 in [0, 1) with 24 random bits."""
    return (words >> np.uint32(8)).astype(np.float64) * (1.0 / 16777216.0)


def uniform(shape, low: float, high: float, seed: int, tensor_id: int = 0) -> np.ndarray:
    n = int(np.prod(shape))
    u = _unit(_random_words(n, tensor_id, seed))
    return (low + (high - low) * u).astype(np.float32).astype(np.float16).reshape(shape)


def normal(shape, sigma: float, seed: int, tensor_id: int = 0) -> np.ndarray:
    n = int(np.prod(shape))
    pairs = (n + 1) // 2
    w = _random_words(2 * pairs, tensor_id, seed)
    u1 = ((w[0::2] >> np.uint32(8)).astype(np.float64) + 1.0) * (1.0 / 16777216.0)  # (0, 1]
    u2 = _unit(w[1::2])
    mag = np.sqrt(-2.0 * np.log(u1))
    ang = 2.0 * np.pi * u2
    z = np.empty(2 * pairs, dtype=np.float64)
    z[0::2] = mag * np.cos(ang)
    z[1::2] = mag * np.sin(ang)
    return (sigma * z[:n]).astype(np.float32).astype(np.float16).reshape(shape)


# --------------------------------------------------------------------------
# Reference formula generators (conv validation suites)
# --------------------------------------------------------------------------

def conv2d_activation(n: int, h: int, w: int, c: int, o: int, kh: int, kw: int) -> np.ndarray:
    """createActivationData(Conv2DDimensions) (ConvolutionShared.swift:4874-4884), NHWC."""
    count = n * h * w * c
    i = np.arange(count, dtype=np.int64)
    if c == 1 and o == 1 and kh == 3 and kw == 3:
        vals = (i + 1).astype(np.float32)
    else:
        vals = (((i * 7) + 3) % 19 - 9).astype(np.float32) * 0.0625
    return vals.astype(np.float16).reshape(n, h, w, c)


def conv2d_weights_hwio(c: int, o: int, kh: int, kw: int) -> np.ndarray:
    """createWeightData(Conv2DDimensions, .hwio) (ConvolutionShared.swift:4886-4908): [KH][KW][C][O]."""
    if c == 1 and o == 1 and kh == 3 and kw == 3:
        wgt = np.zeros((kh, kw, c, o), dtype=np.float16)
        wgt[1, 1, 0, 0] = 1.0
        return wgt
    idx = np.arange(kh * kw * c * o, dtype=np.int64)
    vals = ((((idx * 5) + 1) % 17) - 8).astype(np.float32) * 0.03125
    return vals.astype(np.float16).reshape(kh, kw, c, o)


def conv3d_activation(n: int, d: int, h: int, w: int, c: int) -> np.ndarray:
    """createActivationData(Conv3DDimensions) (ConvolutionShared.swift:4944-4950), NDHWC."""
    i = np.arange(n * d * h * w * c, dtype=np.int64)
    vals = (((i * 7) + 3) % 29 - 14).astype(np.float32) * 0.0625
    return vals.astype(np.float16).reshape(n, d, h, w, c)


def conv3d_weights_dhwio(c: int, o: int, kd: int, kh: int, kw: int) -> np.ndarray:
    """createWeightData(Conv3DDimensions, .dhwio) (ConvolutionShared.swift:4952-4983): [KD][KH][KW][C][O]."""
    idx = np.arange(kd * kh * kw * c * o, dtype=np.int64)
    vals = ((((idx * 5) + 1) % 23) - 11).astype(np.float32) * 0.03125
    return vals.astype(np.float16).reshape(kd, kh, kw, c, o)


def conv3d_bias(o: int) -> np.ndarray:
    """createBiasData(Conv3DDimensions) (ConvolutionShared.swift:4985-4990)."""
    i = np.arange(o, dtype=np.int64)
    return ((((i * 11) + 5) % 19 - 9).astype(np.float32) * 0.0625).astype(np.float16)


def padded_conv2d_activation(n: int, h: int, w: int, c: int) -> np.ndarray:
    """Activation formula of the padded conv2d probe (convolution2d_padding.swift:65-70), NHWC."""
    i = np.arange(n * h * w * c, dtype=np.int64)
    return ((((i * 7) + 3) % 29 - 14).astype(np.float32) * 0.0625).astype(np.float16).reshape(n, h, w, c)


def padded_conv2d_weights_hwio(c: int, o: int, kh: int, kw: int) -> np.ndarray:
    """Weight formula of the padded conv2d probe (convolution2d_padding.swift:72-77): [KH][KW][C][O]."""
    i = np.arange(kh * kw * c * o, dtype=np.int64)
    return ((((i * 5) + 1) % 23 - 11).astype(np.float32) * 0.03125).astype(np.float16).reshape(kh, kw, c, o)
