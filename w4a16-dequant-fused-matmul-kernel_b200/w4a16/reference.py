"""Baselines with the reference's names (w4a16-kernel/src/w4a16/reference.py:15-67).

* ``reference_w4a16``     dequantise, fp32-accumulated matmul, fp16 out
  (the reference's correctness oracle, reference.py:18-40);
* ``dequant_then_matmul`` materialise fp16 W, then an fp16 cuBLAS matmul
  (reference.py:43-53);
* ``fp16_matmul``         plain fp16 cuBLAS matmul on unquantised W (reference.py:56-67).

Here they are GPU comparison rows: the dequantisation is this library's
sm_100a kernel and the matmul is torch's (cuBLAS). They are not the fused
path, and the fused path never calls them. The CPU oracle the test-suite
checks against lives outside this package.
"""
from __future__ import annotations

import torch
from torch import Tensor

from .quant import dequantize_weight

__all__ = ["reference_w4a16", "dequant_then_matmul", "fp16_matmul"]


def reference_w4a16(X: Tensor, qweight: Tensor, scales: Tensor, zeros: Tensor, group_size: int) -> Tensor:
    """dequant -> fp32-accumulated matmul -> fp16, on X's device (CUDA)."""
    assert X.dtype == torch.float16, f"X must be fp16, got {X.dtype}"
    assert X.dim() == 2, f"X must be 2D [M, K], got {tuple(X.shape)}"
    M, K = X.shape
    W_dq = dequantize_weight(qweight, scales, zeros, group_size).to(X.device)
    assert W_dq.shape[0] == K, f"K mismatch: X K={K} vs weight K={W_dq.shape[0]}"
    Y = torch.matmul(X.to(torch.float32), W_dq.to(torch.float32))
    return Y.to(torch.float16)


def dequant_then_matmul(X: Tensor, qweight: Tensor, scales: Tensor, zeros: Tensor,
                        group_size: int) -> Tensor:
    """Naive baseline: materialise the fp16 weight (reads 4x the bytes), then matmul."""
    assert X.dtype == torch.float16
    W_dq = dequantize_weight(qweight, scales, zeros, group_size).to(X.device)
    return torch.matmul(X, W_dq)


def fp16_matmul(X: Tensor, W: Tensor) -> Tensor:
    """Unquantised fp16 matmul; ``W`` is the logical ``[K, N]`` weight."""
    assert X.dtype == torch.float16 and W.dtype == torch.float16
    assert X.shape[1] == W.shape[0], f"K mismatch: X {tuple(X.shape)} vs W {tuple(W.shape)}"
    return torch.matmul(X, W)
