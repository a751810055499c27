"""W4A16 fused dequant-GEMM for NVIDIA B200 (sm_100a).

4-bit group-wise asymmetric weights, fp16 activations. Same public API as the
reference package (w4a16-kernel/src/w4a16/__init__.py:18-39):

    quantize_weight / dequantize_weight / pack_int4 / unpack_int4   (quant.py)
    reference_w4a16 / dequant_then_matmul / fp16_matmul             (reference.py)
    w4a16_matmul                                                    (gemm.py)
    W4A16Linear                                                     (linear.py)

Tensor-parallel layers (column / row sharding over torch.distributed + NCCL)
live in ``w4a16.parallel``.

Everything computes in the hand-written sm_100a library ``libw4a16_b200.so``
(C ABI in ``include/w4a16_b200.h``) -- there is one backend and no CPU or
Triton fallback. Importing needs no GPU; calling needs a B200.
"""
from __future__ import annotations

from ._lib import W4A16Error, check_device_errors
from .gemm import (interleave_gate_up, repack_qweight, stage_copy, swiglu, to_fp16, w4a16_matmul,
                   w4a16_matmul_bf16, w4a16_matmul_f32, w4a16_matmul_host, w4a16_matmul_swiglu)
from .linear import W4A16Linear
from .quant import dequantize_weight, pack_int4, quantize_weight, unpack_int4
from .reference import dequant_then_matmul, fp16_matmul, reference_w4a16

__all__ = [
    "quantize_weight",
    "dequantize_weight",
    "pack_int4",
    "unpack_int4",
    "reference_w4a16",
    "dequant_then_matmul",
    "fp16_matmul",
    "w4a16_matmul",
    "W4A16Linear",
    "w4a16_matmul_f32",
    "swiglu",
    "w4a16_matmul_swiglu",
    "interleave_gate_up",
    "repack_qweight",
    "w4a16_matmul_bf16",
    "to_fp16",
    "stage_copy",
    "w4a16_matmul_host",
    "W4A16Error",
    "check_device_errors",
]

# The reference exported the fused GEMM only when its Triton backend imported
# (HAS_TRITON). The fused GEMM here is always present; the flag is kept, True,
# so code that tests it keeps working. There is no Triton in this package.
HAS_TRITON = True
