"""Generates the committed golden fixtures under tests/golden/.

Each fixture holds seeded fp16 inputs (example_matmul_metal4_b200.data) and
the fp32 output of the C oracle (oracle/mm4_oracle.c, the restatement of the
reference's CPU validation loops). tests/test_oracle.py checks the oracle
against these fixtures and against an independent float64 restatement, and
the GPU tests compare the kernels with the same oracle.

    python tests/golden/make_golden.py
"""
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "oracle"))

import oracle  # noqa: E402
from example_matmul_metal4_b200 import data  # noqa: E402


def gemm_cases():
    out = {}
    for name, (M, N, K, tl, tr, seed) in {
        "nn_48x40x72": (48, 40, 72, False, False, 101),
        "nt_33x17x31": (33, 17, 31, False, True, 102),
        "tn_16x24x40": (16, 24, 40, True, False, 103),
    }.items():
        A = data.uniform((K, M) if tl else (M, K), -1, 1, seed, 0)
        B = data.uniform((N, K) if tr else (K, N), -1, 1, seed, 1)
        bias = data.uniform((N,), -1, 1, seed, 2)
        ref = oracle.gemm(A, B, bias, M, N, K, tl, tr)
        out.update({f"{name}/A": A, f"{name}/B": B, f"{name}/bias": bias, f"{name}/out": ref,
                    f"{name}/dims": np.array([M, N, K, int(tl), int(tr)])})
    return out


def attention_cases():
    out = {}
    for name, (B, Hq, Hk, R, C, layout, seed, D) in {
        "bhsd_1x2_r37_c45": (1, 2, 2, 37, 45, 0, 201, 128),
        "bshd_2x2_gqa_r20_c33": (2, 2, 1, 20, 33, 1, 202, 128),
        "bhsd_1x2_r37_c45_d64": (1, 2, 2, 37, 45, 0, 203, 64),
        "bshd_2x2_gqa_r20_c33_d64": (2, 2, 1, 20, 33, 1, 204, 64),
    }.items():
        qs = (B, Hq, R, D) if layout == 0 else (B, R, Hq, D)
        ks = (B, Hk, C, D) if layout == 0 else (B, C, Hk, D)
        Q = data.normal(qs, 1.0, seed, 0)
        K = data.normal(ks, 1.0, seed, 1)
        V = data.normal(ks, 1.0, seed, 2)
        ref = oracle.attention(Q, K, V, B, Hq, Hk, R, C, D, 1 / np.sqrt(D), layout)
        out.update({f"{name}/Q": Q, f"{name}/K": K, f"{name}/V": V, f"{name}/out": ref,
                    f"{name}/dims": np.array([B, Hq, Hk, R, C, layout, D])})
    return out


def attention_bwd_cases():
    """dQ, dK, dV and the row LSE of the loss sum(dO * O) (Network.swift:181-401 restated)."""
    out = {}
    for name, (B, Hq, Hk, R, C, layout, seed, D) in {
        "bhsd_1x2_r19_c23": (1, 2, 2, 19, 23, 0, 301, 128),
        "bshd_1x4_gqa_r12_c17": (1, 4, 2, 12, 17, 1, 302, 128),
        "bhsd_1x2_r19_c23_d64": (1, 2, 2, 19, 23, 0, 303, 64),
        "bshd_1x4_gqa_r12_c17_d64": (1, 4, 2, 12, 17, 1, 304, 64),
    }.items():
        qs = (B, Hq, R, D) if layout == 0 else (B, R, Hq, D)
        ks = (B, Hk, C, D) if layout == 0 else (B, C, Hk, D)
        Q = data.normal(qs, 1.0, seed, 0)
        K = data.normal(ks, 1.0, seed, 1)
        V = data.normal(ks, 1.0, seed, 2)
        dO = data.normal(qs, 1.0, seed, 3)
        dQ, dK, dV, lse = oracle.attention_bwd(Q, K, V, dO, B, Hq, Hk, R, C, D, 1 / np.sqrt(D), layout)
        out.update({f"{name}/Q": Q, f"{name}/K": K, f"{name}/V": V, f"{name}/dO": dO, f"{name}/dQ": dQ,
                    f"{name}/dK": dK, f"{name}/dV": dV, f"{name}/lse": lse,
                    f"{name}/dims": np.array([B, Hq, Hk, R, C, layout, D])})
    return out


def main():
    np.savez_compressed(HERE / "gemm_small.npz", **gemm_cases())
    np.savez_compressed(HERE / "attention_small.npz", **attention_cases())
    np.savez_compressed(HERE / "attention_bwd_small.npz", **attention_bwd_cases())
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
