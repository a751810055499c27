"""CPU oracle for the W4A16 hot path (TEST INFRASTRUCTURE ONLY).

This package restates, in numpy, the reference's quantise / pack / unpack /
dequantise / fp32-accumulate GEMM algorithm so that the sm_100a kernels can be
checked against it. Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU
baseline leg of ``bench.py`` may import it; the product package never does.

Parity is pinned: ``tests/test_oracle.py`` checks every function here against
the worked examples of ``W4A16_SPEC.md`` and against golden vectors produced by
running the reference's own ``quant.py`` / ``reference.py`` (see
``tests/golden/make_golden.py``).
"""
from .w4a16_oracle import (  # noqa: F401
    pack_int4,
    unpack_int4,
    quantize_weight,
    dequantize_weight,
    reference_w4a16,
    dequant_then_matmul,
)
