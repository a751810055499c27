"""Test helpers: seeded GPU case builders and a plain-PyTorch fp32 reference
for full-size parity checks (too large for the numpy oracle to finish in
seconds). The torch reference restates the oracle's arithmetic -- unpack with
shift/mask, fp16 ``(q - z) * s``, fp32 matmul with TF32 off -- in torch ops on
the GPU; it is test infrastructure, never called by the package."""
from __future__ import annotations

import numpy as np
import torch


def gpu_case(M, K, N, G, sigma=1.0, seed=0, device="cuda", outlier_frac=0.0):
    """X ~ N(0,1) fp16 [M,K], W ~ sigma*N(0,1) fp16 [K,N] (optionally with a
    Bernoulli(outlier_frac) set redrawn from N(0, 0.2^2)), generated on the GPU."""
    gen = torch.Generator(device=device).manual_seed(seed)
    X = torch.randn(M, K, generator=gen, device=device, dtype=torch.float32).half()
    W = torch.randn(K, N, generator=gen, device=device, dtype=torch.float32) * sigma
    if outlier_frac > 0:
        mask = torch.rand(K, N, generator=gen, device=device) < outlier_frac
        W = torch.where(mask, torch.randn(K, N, generator=gen, device=device) * 0.2, W)
    return X, W.half()


def torch_dequant(qweight: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor, G: int) -> torch.Tensor:
    Kp, N = qweight.shape
    K = Kp * 8
    shifts = torch.arange(0, 32, 4, device=qweight.device, dtype=torch.int32).view(1, 8, 1)
    q = ((qweight.view(Kp, 1, N) >> shifts) & 0xF).reshape(K, N)
    qh = q.to(torch.float16).view(K // G, G, N)
    w = (qh - zeros.view(K // G, 1, N)) * scales.view(K // G, 1, N)   # fp16 arithmetic
    return w.reshape(K, N)


def torch_reference(X, qweight, scales, zeros, G) -> torch.Tensor:
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        W = torch_dequant(qweight, scales, zeros, G).float()
        return (X.float() @ W).half()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def np_(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy()


def bits16(t) -> np.ndarray:
    a = np_(t) if isinstance(t, torch.Tensor) else t
    return np.ascontiguousarray(a).view(np.uint16)
