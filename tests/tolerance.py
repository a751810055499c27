"""The parity tolerance for the fused GEMM's fp16 output.

The target states: max |kernel - oracle| <= 1e-2 absolute + 1e-3 relative to
the oracle, elementwise, on the fp16 output, where the oracle is the
reference's fp32-accumulated ``reference_w4a16`` on the same quantised
tensors. Since 1e-3*|y| exceeds one fp16 ulp (2^-10 |y|) this admits the
one-ulp differences of a different fp32 summation order and nothing larger.
"""
from __future__ import annotations

import numpy as np

ATOL = 1e-2
RTOL = 1e-3


def assert_gemm_close(out: np.ndarray, ref: np.ndarray, what: str = "") -> float:
    out = np.asarray(out, dtype=np.float32)
    ref = np.asarray(ref, dtype=np.float32)
    assert out.shape == ref.shape, f"{what}: shape {out.shape} != {ref.shape}"
    assert np.all(np.isfinite(out)), f"{what}: non-finite output"
    err = np.abs(out - ref)
    bound = ATOL + RTOL * np.abs(ref)
    bad = err > bound
    if bad.any():
        i = np.unravel_index(np.argmax(err - bound), err.shape)
        raise AssertionError(
            f"{what}: {int(bad.sum())} of {err.size} elements outside 1e-2 + 1e-3*|ref|; "
            f"worst at {i}: out={out[i]} ref={ref[i]}")
    return float(err.max()) if err.size else 0.0
