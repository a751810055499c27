"""Import-path compatibility: the reference exposed ``w4a16_matmul`` from
``w4a16.triton_kernel`` (w4a16-kernel/src/w4a16/triton_kernel.py:131). The
function lives in :mod:`w4a16.gemm` and runs the sm_100a CUDA library; no
Triton is involved."""
from .gemm import w4a16_matmul  # noqa: F401

__all__ = ["w4a16_matmul"]
