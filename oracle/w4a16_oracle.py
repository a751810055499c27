"""numpy restatement of the reference W4A16 algorithm (CPU oracle, test-only).

Reference being restated (paths inside the reference project):

* ``w4a16-kernel/src/w4a16/quant.py:45-70``   pack_int4
* ``w4a16-kernel/src/w4a16/quant.py:73-95``   unpack_int4
* ``w4a16-kernel/src/w4a16/quant.py:101-144`` quantize_weight
* ``w4a16-kernel/src/w4a16/quant.py:147-178`` dequantize_weight
* ``w4a16-kernel/src/w4a16/reference.py:18-40`` reference_w4a16 (the oracle)
* ``w4a16-kernel/src/w4a16/reference.py:43-53`` dequant_then_matmul (CPU baseline)

Format (``W4A16_SPEC.md`` sections 2-3): ``W`` is ``[K, N]`` (K = in_features).
Groups of ``G`` consecutive K-rows share one fp16 scale and one fp16 integer
zero-point per column. ``qweight[i, n]`` packs rows ``8i .. 8i+7`` of column
``n`` with row ``8i + j`` in bits ``[4j, 4j+4)``.

Numerics mirrored bit-for-bit:

* scale / zero / code arithmetic in fp32 with IEEE division and
  round-half-to-even (numpy ``np.rint`` == ``torch.round``);
* ``clamp`` keeps the sign of a zero (torch's CPU clamp returns ``-0.0`` for
  ``clamp(-0.0, 0, 15)``), so an all-zero group stores zero-point ``-0.0``;
* dequantisation is ``(q - z) * s`` rounded once to fp16: ``q - z`` is exact,
  and an fp16*fp16 product is exact in fp32, so computing in fp32 and rounding
  to fp16 once equals the reference's fp16 tensor arithmetic.

Every array argument is a numpy array; nothing here touches torch or a GPU.
"""
from __future__ import annotations

import numpy as np

_NIB = 8          # nibbles per int32 word (quant.py:33)
_QMAX = 15        # 2**4 - 1 (quant.py:34)


def pack_int4(q: np.ndarray) -> np.ndarray:
    """Pack ``[K, N]`` codes in 0..15 into int32 ``[K//8, N]`` (quant.py:45-70).

    Raises ``AssertionError`` for a non-2D input, ``K % 8 != 0`` or codes
    outside ``[0, 15]`` (quant.py:57-63).
    """
    assert q.ndim == 2, f"pack_int4 expects 2D [K, N], got {q.shape}"
    K, N = q.shape
    assert K % _NIB == 0, f"K={K} must be divisible by 8 to pack int4"
    qi = q.astype(np.int64)
    if qi.size:
        lo, hi = int(qi.min()), int(qi.max())
        assert 0 <= lo and hi <= _QMAX, f"uint4 values must be in [0,15], got [{lo},{hi}]"
    qi = qi.reshape(K // _NIB, _NIB, N)
    packed = np.zeros((K // _NIB, N), dtype=np.uint32)
    for j in range(_NIB):
        packed |= ((qi[:, j, :] & 0xF).astype(np.uint32)) << np.uint32(4 * j)
    return packed.view(np.int32)


def unpack_int4(qweight: np.ndarray, K: int | None = None) -> np.ndarray:
    """Inverse of :func:`pack_int4`: int32 ``[K//8, N]`` -> int32 ``[K, N]`` (quant.py:73-95)."""
    assert qweight.ndim == 2, f"unpack_int4 expects 2D [K//8, N], got {qweight.shape}"
    assert qweight.dtype == np.int32, f"qweight must be int32, got {qweight.dtype}"
    Kp, N = qweight.shape
    if K is None:
        K = Kp * _NIB
    assert K == Kp * _NIB, f"K={K} incompatible with qweight rows {Kp}"
    u = qweight.view(np.uint32)
    out = np.empty((Kp, _NIB, N), dtype=np.int32)
    for j in range(_NIB):
        out[:, j, :] = ((u >> np.uint32(4 * j)) & np.uint32(0xF)).astype(np.int32)
    return out.reshape(K, N)


def _clamp_keep_sign(x: np.ndarray, lo: float, hi: float) -> np.ndarray:
    """``min(max(x, lo), hi)`` with torch-CPU semantics: NaN and ``-0.0`` pass through."""
    y = np.where(x < lo, np.float32(lo), x)
    return np.where(y > hi, np.float32(hi), y).astype(np.float32)


def quantize_weight(W: np.ndarray, group_size: int = 128):
    """Group-wise asymmetric uint4 quantisation of ``W [K, N]`` (quant.py:101-144).

    Returns ``(qweight int32 [K//8, N], scales fp16 [K//G, N], zeros fp16 [K//G, N])``.
    Raises ``ValueError`` when ``K % 8`` or ``K % G`` is non-zero (quant.py:116-119).
    """
    assert W.ndim == 2, f"quantize_weight expects 2D [K, N], got {W.shape}"
    K, N = W.shape
    if K % _NIB != 0:
        raise ValueError(f"K={K} must be divisible by 8 (got remainder {K % 8})")
    if K % group_size != 0:
        raise ValueError(f"K={K} must be divisible by group_size={group_size}")
    G = group_size
    ng = K // G
    Wg = W.astype(np.float32).reshape(ng, G, N)
    gmax = Wg.max(axis=1)
    gmin = Wg.min(axis=1)
    scale = ((gmax - gmin) / np.float32(_QMAX)).astype(np.float32)          # quant.py:129
    scale = np.where(scale > 0, scale, np.float32(1.0)).astype(np.float32)   # quant.py:132
    with np.errstate(invalid="ignore", divide="ignore"):
        zero = _clamp_keep_sign(np.rint(-gmin / scale), 0, _QMAX)            # quant.py:134
        q = _clamp_keep_sign(np.rint(Wg / scale[:, None, :]) + zero[:, None, :], 0, _QMAX)
    q = q.reshape(K, N)
    assert np.all(np.isfinite(q)), "non-finite weights cannot be quantised"
    qweight = pack_int4(q.astype(np.int32))
    return qweight, scale.astype(np.float16), zero.astype(np.float16)


def dequantize_weight(qweight: np.ndarray, scales: np.ndarray, zeros: np.ndarray,
                      group_size: int) -> np.ndarray:
    """``W_dq = (q - z) * s`` rounded once to fp16, shape ``[K, N]`` (quant.py:147-178)."""
    assert qweight.dtype == np.int32
    Kp, N = qweight.shape
    K = Kp * _NIB
    G = group_size
    assert K % G == 0, f"K={K} must be divisible by group_size={G}"
    ng = K // G
    assert scales.shape == (ng, N) and zeros.shape == (ng, N)
    q = unpack_int4(qweight, K).astype(np.float32).reshape(ng, G, N)
    s = scales.astype(np.float16).astype(np.float32)[:, None, :]
    z = zeros.astype(np.float16).astype(np.float32)[:, None, :]
    # fp16(q) - fp16(z) is one fp16 rounding in the reference; for the integer
    # zero-points quantize_weight produces it is exact. Mirror it explicitly.
    d = (q - z).astype(np.float16).astype(np.float32)
    return (d * s).astype(np.float16).reshape(K, N)


def reference_w4a16(X: np.ndarray, qweight: np.ndarray, scales: np.ndarray,
                    zeros: np.ndarray, group_size: int) -> np.ndarray:
    """The correctness oracle: fp16 dequant -> fp32 matmul -> fp16 (reference.py:18-40)."""
    assert X.dtype == np.float16, f"X must be fp16, got {X.dtype}"
    assert X.ndim == 2
    W_dq = dequantize_weight(qweight, scales, zeros, group_size)
    assert W_dq.shape[0] == X.shape[1]
    Y = X.astype(np.float32) @ W_dq.astype(np.float32)
    return Y.astype(np.float16)


def dequant_then_matmul(X: np.ndarray, qweight: np.ndarray, scales: np.ndarray,
                        zeros: np.ndarray, group_size: int) -> np.ndarray:
    """CPU restatement of the reference's naive baseline (reference.py:43-53).

    Materialises the full fp16 weight, then multiplies. numpy has no fp16 BLAS,
    so the product runs through fp32 BLAS on the fp16 values (the same sums a
    CPU fp16 matmul accumulates in fp32) and rounds to fp16.
    """
    assert X.dtype == np.float16
    W_dq = dequantize_weight(qweight, scales, zeros, group_size)
    return (X.astype(np.float32) @ W_dq.astype(np.float32)).astype(np.float16)
