"""Import-path compatibility with the reference's CUDA extension wrapper
(w4a16-kernel/src/w4a16/cuda_kernel.py:35-87).

``load_cuda_module()`` returns the loaded sm_100a C-ABI library (built
ahead of time in-tree, never JIT-compiled at import), and
``w4a16_matmul_cuda`` is the same fused GEMM as :func:`w4a16.w4a16_matmul`.
"""
from __future__ import annotations

import ctypes

from . import _lib
from .gemm import w4a16_matmul

__all__ = ["w4a16_matmul_cuda", "load_cuda_module"]


def load_cuda_module(verbose: bool = False) -> ctypes.CDLL:
    lib = _lib.lib()
    if verbose:
        print(f"w4a16: loaded {_lib.LIB_PATH} (version {lib.w4a16_version()})")
    return lib


def w4a16_matmul_cuda(x, qweight, scales, zeros, group_size):
    return w4a16_matmul(x, qweight, scales, zeros, group_size)
