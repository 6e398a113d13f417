"""Pass rule shared by the parity tests.

fp16 outputs within max relative error 1e-2 and max
absolute error 2e-2 of the fp32-accumulated CPU result, applied per element
in allclose form: |gpu - ref| <= ATOL + RTOL * |ref|. Reported like the
reference's ValidationResult (maxAbsoluteError, mismatches;
ConvolutionShared.swift:5174-5208).
"""
import numpy as np

ATOL = 2e-2
RTOL = 1e-2


def validation(gpu, ref, atol=ATOL, rtol=RTOL):
    gpu = np.asarray(gpu, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert gpu.shape == ref.shape, (gpu.shape, ref.shape)
    err = np.abs(gpu - ref)
    bad = ~(err <= atol + rtol * np.abs(ref))
    return {
        "maxAbsoluteError": float(err.max()) if err.size else 0.0,
        "maxRelativeError": float((err / np.maximum(np.abs(ref), 1e-6)).max()) if err.size else 0.0,
        "mismatches": int(bad.sum()),
        "count": int(err.size),
    }


def assert_close(gpu, ref, what="", atol=ATOL, rtol=RTOL):
    v = validation(gpu, ref, atol, rtol)
    assert v["mismatches"] == 0, f"{what}: {v}"
    return v
