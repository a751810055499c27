"""Quantise / pack / unpack / dequantise on the GPU (sm_100a kernels).

Same API, argument meaning and error behaviour as the reference's
``w4a16-kernel/src/w4a16/quant.py``:

* ``pack_int4(q)``                      quant.py:45-70
* ``unpack_int4(qweight, K=None)``      quant.py:73-95
* ``quantize_weight(W, group_size)``    quant.py:101-144 (bit-exact)
* ``dequantize_weight(qweight, scales, zeros, group_size)``  quant.py:147-178 (bit-exact)

Format: ``W`` is ``[K, N]`` (K = in_features); groups of ``G`` K-rows share one
fp16 scale and one integer fp16 zero-point per column; ``qweight[i, n]``
holds rows ``8i .. 8i+7`` with row ``8i + j`` in bits ``[4j, 4j+4)``.

Every function computes on a CUDA device. CUDA inputs stay on their device;
CPU inputs are copied to the current CUDA device, processed there, and the
results are copied back, so ``W4A16Linear.from_linear`` works on a CPU layer.
Without a CUDA device these functions raise ``RuntimeError``.
"""
from __future__ import annotations

import torch
from torch import Tensor

from . import _lib

__all__ = ["quantize_weight", "dequantize_weight", "pack_int4", "unpack_int4"]

_NIBBLES_PER_INT32 = 8
_MAX_UINT4 = 15


def _work_device(t: Tensor) -> torch.device:
    if t.is_cuda:
        return t.device
    if not torch.cuda.is_available():
        raise RuntimeError("W4A16 kernels need a CUDA (sm_100 / B200) device; none is available")
    return torch.device("cuda", torch.cuda.current_device())


def pack_int4(q: Tensor) -> Tensor:
    """Pack a ``[K, N]`` tensor of uint4 values (0..15) into int32 ``[K//8, N]``.

    Row ``k = 8*i + j`` maps to nibble ``j`` (bits ``[4*j : 4*j+4]``) of
    ``qweight[i, n]``. Raises ``AssertionError`` for a non-2D input, K not
    divisible by 8, or values outside [0, 15] (a one-time device->host check,
    as in the reference).
    """
    assert q.dim() == 2, f"pack_int4 expects 2D [K, N], got {tuple(q.shape)}"
    K, N = q.shape
    assert K % _NIBBLES_PER_INT32 == 0, f"K={K} must be divisible by 8 to pack int4"
    dev = _work_device(q)
    qi = q.to(device=dev, dtype=torch.int32).contiguous()
    if qi.numel():
        lo, hi = (int(v) for v in torch.aminmax(qi))
        assert 0 <= lo and hi <= _MAX_UINT4, f"uint4 values must be in [0,15], got [{lo},{hi}]"
    packed = torch.empty((K // _NIBBLES_PER_INT32, N), dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        st = _lib.lib().w4a16_pack_int4(qi.data_ptr(), packed.data_ptr(), K, N, _lib.stream_of(dev))
    _lib.check(st, "w4a16_pack_int4")
    return packed.to(q.device)


def unpack_int4(qweight: Tensor, K: int | None = None) -> Tensor:
    """Inverse of :func:`pack_int4`: int32 ``[K//8, N]`` -> int32 ``[K, N]`` in [0, 15]."""
    assert qweight.dim() == 2, f"unpack_int4 expects 2D [K//8, N], got {tuple(qweight.shape)}"
    assert qweight.dtype == torch.int32, f"qweight must be int32, got {qweight.dtype}"
    Kp, N = qweight.shape
    if K is None:
        K = Kp * _NIBBLES_PER_INT32
    assert K == Kp * _NIBBLES_PER_INT32, f"K={K} incompatible with qweight rows {Kp}"
    dev = _work_device(qweight)
    qw = qweight.to(dev).contiguous()
    out = torch.empty((K, N), dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        st = _lib.lib().w4a16_unpack_int4(qw.data_ptr(), out.data_ptr(), K, N, _lib.stream_of(dev))
    _lib.check(st, "w4a16_unpack_int4")
    return out.to(qweight.device)


def quantize_weight(W: Tensor, group_size: int = 128, *, symmetric: bool = False) -> tuple[Tensor, Tensor, Tensor]:
    """Group-wise asymmetric 4-bit quantisation of ``W`` along K (bit-exact with the reference).

    Args:
        W: weight tensor [K, N] (fp16, bf16 or fp32; other dtypes go through fp32).
        group_size: G, number of K-rows per quantisation group. Requires G | K, 8 | K.
        symmetric: (extension) symmetric codes as GPTQ-style checkpoints store them
            with sym=True: zero-point 8 and scale 2 * max|w| / 15 per group, in the
            same format (every GEMM takes it unchanged). The reference has no such mode.

    Returns:
        (qweight int32 [K//8, N], scales fp16 [K//G, N], zeros fp16 [K//G, N]),
        on ``W``'s device.

    Raises:
        ValueError: K not divisible by 8 or by group_size (quant.py:116-119).
        AssertionError: W not 2D, or non-finite weights (the reference's packer
            rejects the out-of-range codes they produce, quant.py:62-63).
    """
    assert W.dim() == 2, f"quantize_weight expects 2D [K, N], got {tuple(W.shape)}"
    K, N = W.shape
    if K % _NIBBLES_PER_INT32 != 0:
        raise ValueError(f"K={K} must be divisible by 8 (got remainder {K % 8})")
    if K % group_size != 0:
        raise ValueError(f"K={K} must be divisible by group_size={group_size}")
    G = group_size
    dev = _work_device(W)
    Wd = W.detach()
    if Wd.dtype not in _lib.DTYPE_CODES:
        Wd = Wd.to(torch.float32)
    Wd = Wd.to(dev).contiguous()
    if Wd.numel():
        assert bool(torch.isfinite(Wd).all()), "W contains non-finite values; they cannot be quantised"
    qweight = torch.empty((K // _NIBBLES_PER_INT32, N), dtype=torch.int32, device=dev)
    scales = torch.empty((K // G, N), dtype=torch.float16, device=dev)
    zeros = torch.empty((K // G, N), dtype=torch.float16, device=dev)
    with torch.cuda.device(dev):
        if symmetric:
            st = _lib.lib().w4a16_quantize_ex(
                Wd.data_ptr(), _lib.DTYPE_CODES[Wd.dtype], qweight.data_ptr(), scales.data_ptr(),
                zeros.data_ptr(), K, N, G, 1, _lib.stream_of(dev))
        else:
            st = _lib.lib().w4a16_quantize(
                Wd.data_ptr(), _lib.DTYPE_CODES[Wd.dtype], qweight.data_ptr(), scales.data_ptr(),
                zeros.data_ptr(), K, N, G, _lib.stream_of(dev))
    _lib.check(st, "w4a16_quantize")
    return qweight.to(W.device), scales.to(W.device), zeros.to(W.device)


def dequantize_weight(qweight: Tensor, scales: Tensor, zeros: Tensor, group_size: int) -> Tensor:
    """Dequantise packed uint4 weights back to fp16 ``[K, N]``: ``(q - z) * s`` in fp16."""
    assert qweight.dtype == torch.int32, f"qweight must be int32, got {qweight.dtype}"
    Kp, N = qweight.shape
    K = Kp * _NIBBLES_PER_INT32
    G = group_size
    assert K % G == 0, f"K={K} must be divisible by group_size={G}"
    num_groups = K // G
    assert scales.shape == (num_groups, N), f"scales shape {tuple(scales.shape)} != {(num_groups, N)}"
    assert zeros.shape == (num_groups, N), f"zeros shape {tuple(zeros.shape)} != {(num_groups, N)}"
    dev = _work_device(qweight)
    qw = qweight.to(dev).contiguous()
    s = scales.to(device=dev, dtype=torch.float16).contiguous()
    z = zeros.to(device=dev, dtype=torch.float16).contiguous()
    w = torch.empty((K, N), dtype=torch.float16, device=dev)
    with torch.cuda.device(dev):
        st = _lib.lib().w4a16_dequantize(qw.data_ptr(), s.data_ptr(), z.data_ptr(), w.data_ptr(),
                                         K, N, G, _lib.stream_of(dev))
    _lib.check(st, "w4a16_dequantize")
    return w.to(qweight.device)
