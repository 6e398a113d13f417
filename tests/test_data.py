"""Seeded input generators: Philox-4x32-10 known-answer vectors (Random123's
published KATs for the SC'11 generator) and the reference's formula data."""
import numpy as np

from example_matmul_metal4_b200 import data


def _block(ctr, key):
    out = data.philox4x32_10(*(np.array([c], dtype=np.uint32) for c in ctr), *key)
    return [int(v[0]) for v in out]


def test_philox_kat_zero():
    assert _block((0, 0, 0, 0), (0, 0)) == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]


def test_philox_kat_ones():
    assert _block((0xFFFFFFFF,) * 4, (0xFFFFFFFF, 0xFFFFFFFF)) == [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]


def test_philox_kat_pi():
    assert _block((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0)) == \
        [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]


def test_generators_deterministic_and_in_range():
    a = data.uniform((1000,), -1, 1, 7, 3)
    assert np.array_equal(a.view(np.uint16), data.uniform((1000,), -1, 1, 7, 3).view(np.uint16))
    assert a.min() >= -1 and a.max() <= 1
    assert not np.array_equal(a, data.uniform((1000,), -1, 1, 7, 4))
    n = data.normal((200000,), 1.0, 7, 0).astype(np.float64)
    assert abs(n.mean()) < 0.01 and abs(n.std() - 1.0) < 0.01
    assert abs(data.normal((200000,), 0.05, 7, 0).astype(np.float64).std() - 0.05) < 0.001


def test_prefix_stability():
    """Element i depends only on (seed, tensor id, i): a longer tensor extends a shorter one."""
    short = data.uniform((100,), 0, 1, 11, 0)
    long = data.uniform((1000,), 0, 1, 11, 0)
    assert np.array_equal(short.view(np.uint16), long[:100].view(np.uint16))


def test_reference_formula_values():
    # createActivationData: ((i*7+3)%19 - 9) * 0.0625 (ConvolutionShared.swift:4880-4883)
    x = data.conv2d_activation(1, 2, 2, 2, 3, 3, 3).reshape(-1)
    assert list(x.astype(np.float32)) == [((i * 7 + 3) % 19 - 9) * 0.0625 for i in range(8)]
    # 1-channel 3x3 special case: ramp 1..N and a centre-tap kernel
    assert list(data.conv2d_activation(1, 2, 2, 1, 1, 3, 3).reshape(-1)) == [1, 2, 3, 4]
    w = data.conv2d_weights_hwio(1, 1, 3, 3)
    assert w.sum() == 1 and w[1, 1, 0, 0] == 1
    # createBiasData: ((i*11+5)%19 - 9) * 0.0625
    assert list(data.conv3d_bias(3).astype(np.float32)) == [((i * 11 + 5) % 19 - 9) * 0.0625 for i in range(3)]
