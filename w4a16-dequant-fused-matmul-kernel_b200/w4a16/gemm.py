"""``w4a16_matmul`` -- the fused W4A16 GEMM on B200 (sm_100a).

Drop-in for the reference's ``w4a16_matmul`` (w4a16-kernel/src/w4a16/triton_kernel.py:131-200):
same signature, same argument meaning, same ``AssertionError`` conditions and
messages, same fresh-or-``out`` output contract. The work runs in the
hand-written sm_100a library through its C ABI, on torch's current stream:

* ``M <= 32``  -> the memory-bound decode kernel (TMA-fed, tensor-core MMA on
  register-dequantised fragments, cluster split-K);
* ``M > 32``   -> the tcgen05/TMEM prefill kernel (128x256 tiles).

Group sizes: the reference requires every autotune ``BLOCK_K`` (32 and 64) to
divide ``group_size`` (triton_kernel.py:177-182), i.e. ``group_size % 64 == 0``;
the same rule holds here and raises the same ``AssertionError``.

Zero-points must be integers in ``[0, 15]`` as ``quantize_weight`` produces
them (the format's contract); the kernels subtract them exactly through the
fp16 magic-number trick, which relies on it.
"""
from __future__ import annotations

import torch
from torch import Tensor

from . import _lib

__all__ = ["w4a16_matmul"]

# The reference's smallest and largest BLOCK_K; every group size must be a multiple of both.
_BLOCK_K_RULE = 64
_F16, _I32 = torch.float16, torch.int32
_current_device = torch._C._cuda_getDevice if hasattr(torch._C, "_cuda_getDevice") else torch.cuda.current_device
_raw_stream = _lib.stream_of_index


def w4a16_matmul(
    x: Tensor,
    qweight: Tensor,
    scales: Tensor,
    zeros: Tensor,
    group_size: int,
    out: Tensor | None = None,
    *,
    bias: Tensor | None = None,
    kernel_order: bool = False,
) -> Tensor:
    """Fused W4A16 GEMM: ``Y = X @ dequant(qweight)`` (fp32 accumulate, fp16 out).

    Args:
        x: activations [M, K] fp16, contiguous, on CUDA.
        qweight: int32 [K//8, N], contiguous, on CUDA.
        scales: fp16 [K//G, N], contiguous, on CUDA.
        zeros: fp16 [K//G, N], contiguous, on CUDA.
        group_size: G. Must satisfy G | K, 8 | K and 64 | G.
        out: optional preallocated fp16 [M, N] output.
        bias: optional fp16 [N] (extension): the result is ``fp16(Y) + bias``
            rounded to fp16, fused into the kernel's epilogue.
        kernel_order: (extension) ``qweight`` holds the kernel nibble order written
            by :func:`repack_qweight` instead of the reference's.

    Returns:
        fp16 tensor [M, N].
    """
    # The common case in one expression (cheap tensor attributes, no temporaries);
    # anything unusual goes through the detailed checks below, which raise the
    # reference's AssertionError with its message.
    xs, qs = x.shape, qweight.shape
    d = x.get_device()
    if not (len(xs) == 2 and len(qs) == 2 and d >= 0 and x.dtype is _F16 and qweight.dtype is _I32
            and scales.dtype is _F16 and zeros.dtype is _F16 and qs[0] * 8 == xs[1]
            and group_size > 0 and xs[1] % group_size == 0 and group_size % _BLOCK_K_RULE == 0
            and scales.shape == (xs[1] // group_size, qs[1]) and zeros.shape == scales.shape
            and qweight.get_device() == d and scales.get_device() == d and zeros.get_device() == d
            and x.is_contiguous() and qweight.is_contiguous() and scales.is_contiguous()
            and zeros.is_contiguous()):
        _check_inputs(x, qweight, scales, zeros, group_size)
    M, K = xs
    N = qs[1]
    if bias is not None:
        assert bias.get_device() == d, "bias must be on the inputs' CUDA device"
        assert bias.dtype is _F16 and bias.shape == (N,) and bias.is_contiguous(), (
            f"bias must be a contiguous fp16 [{N}] tensor"
        )

    if out is None:
        y = torch.empty((M, N), device=d, dtype=_F16)
    else:
        assert out.shape == (M, N) and out.dtype is _F16 and out.is_contiguous()
        assert out.get_device() == d, "out must be on the inputs' CUDA device"
        y = out

    _launch(x, qweight, scales, zeros, bias, y, M, N, K, group_size, N,
            _lib.FLAG_KERNEL_ORDER if kernel_order else 0)
    return y


def _check_inputs(x: Tensor, qweight: Tensor, scales: Tensor, zeros: Tensor, group_size: int) -> None:
    """The reference's assertions (triton_kernel.py:153-182) and this library's device
    rule, one by one, so a bad call fails with the specific message."""
    assert x.is_cuda, "x must be on CUDA (a B200 / sm_100 device)"
    assert qweight.is_cuda and scales.is_cuda and zeros.is_cuda, "all inputs must be on CUDA"
    assert x.dtype == torch.float16, f"x must be fp16, got {x.dtype}"
    assert qweight.dtype == torch.int32, f"qweight must be int32, got {qweight.dtype}"
    assert scales.dtype == torch.float16, f"scales must be fp16, got {scales.dtype}"
    assert zeros.dtype == torch.float16, f"zeros must be fp16, got {zeros.dtype}"
    assert x.dim() == 2 and qweight.dim() == 2, "x and qweight must be 2D"

    M, K = x.shape
    Kp, N = qweight.shape
    assert Kp * 8 == K, f"qweight rows (K//8)={Kp} incompatible with x K={K}"
    assert K % 8 == 0, f"K={K} must be divisible by 8"
    assert K % group_size == 0, f"K={K} must be divisible by group_size={group_size}"
    num_groups = K // group_size
    assert scales.shape == (num_groups, N), f"scales shape {tuple(scales.shape)} != {(num_groups, N)}"
    assert zeros.shape == (num_groups, N), f"zeros shape {tuple(zeros.shape)} != {(num_groups, N)}"

    assert x.is_contiguous(), "x must be contiguous"
    assert qweight.is_contiguous(), "qweight must be contiguous"
    assert scales.is_contiguous(), "scales must be contiguous"
    assert zeros.is_contiguous(), "zeros must be contiguous"

    assert group_size % _BLOCK_K_RULE == 0, (
        f"group_size={group_size} must be a multiple of {_BLOCK_K_RULE} (every K tile of the "
        f"kernels must lie inside one quantisation group)"
    )
    dev = x.device
    assert qweight.device == dev and scales.device == dev and zeros.device == dev, (
        "all inputs must be on the same CUDA device"
    )


def _launch(x, qweight, scales, zeros, bias, y, M, N, K, G, ldy, flags=0) -> None:
    d = x.get_device()
    if d != _current_device():
        with torch.cuda.device(d):
            return _launch(x, qweight, scales, zeros, bias, y, M, N, K, G, ldy, flags)
    stream = _raw_stream(d)
    ws_ptr, ws_bytes = _lib.workspace_for(M, N, K, G, d, stream)
    if flags:
        if y.dtype is torch.float32:
            flags |= _lib.FLAG_F32_OUT
        st = _lib.lib().w4a16_gemm_ex(
            x.data_ptr(), qweight.data_ptr(), scales.data_ptr(), zeros.data_ptr(),
            None if bias is None else bias.data_ptr(), y.data_ptr(), M, N, K, G, ldy, flags,
            ws_ptr, ws_bytes, stream)
        if st:
            _lib.check(st, "w4a16_gemm_ex")
        return
    if y.dtype is torch.float32:
        assert bias is None
        st = _lib.lib().w4a16_gemm_f32(
            x.data_ptr(), qweight.data_ptr(), scales.data_ptr(), zeros.data_ptr(),
            y.data_ptr(), M, N, K, G, ldy, ws_ptr, ws_bytes, stream)
    else:
        st = _lib.lib().w4a16_gemm(
            x.data_ptr(), qweight.data_ptr(), scales.data_ptr(), zeros.data_ptr(),
            None if bias is None else bias.data_ptr(), y.data_ptr(), M, N, K, G, ldy,
            ws_ptr, ws_bytes, stream)
    if st:
        _lib.check(st, "w4a16_gemm")


def w4a16_matmul_f32(x: Tensor, qweight: Tensor, scales: Tensor, zeros: Tensor, group_size: int,
                     out: Tensor | None = None, *, kernel_order: bool = False) -> Tensor:
    """``X @ dequant(qweight)`` as unrounded fp32 sums (no bias): the partial
    result of a K-sharded layer, to be summed across ranks before rounding.
    Same argument checks as :func:`w4a16_matmul`."""
    w4a16_matmul(x[:0], qweight, scales, zeros, group_size)   # argument validation only
    M, K = x.shape
    N = qweight.shape[1]
    if out is None:
        out = torch.empty((M, N), device=x.device, dtype=torch.float32)
    else:
        assert out.shape == (M, N) and out.dtype == torch.float32 and out.is_contiguous()
    _launch(x, qweight, scales, zeros, None, out, M, N, K, group_size, N,
            _lib.FLAG_KERNEL_ORDER if kernel_order else 0)
    return out


def to_fp16(x: Tensor, out: Tensor | None = None) -> Tensor:
    """``x`` (bf16, fp32 or fp16, on CUDA) rounded to fp16 by the library's conversion
    kernel. bf16 -> fp16 is exact for |x| in [2^-14, 65504] (and 0)."""
    assert x.is_cuda and x.dtype in _lib.DTYPE_CODES and x.is_contiguous()
    if out is None:
        out = torch.empty(x.shape, dtype=torch.float16, device=x.device)
    assert out.shape == x.shape and out.dtype == torch.float16 and out.is_contiguous()
    with torch.cuda.device(x.device):
        st = _lib.lib().w4a16_convert(x.data_ptr(), _lib.DTYPE_CODES[x.dtype], out.data_ptr(),
                                      _lib.DTYPE_CODES[torch.float16], x.numel(), _lib.stream_of(x.device))
    _lib.check(st, "w4a16_convert")
    return out


def w4a16_matmul_bf16(x: Tensor, qweight: Tensor, scales: Tensor, zeros: Tensor, group_size: int,
                      out: Tensor | None = None, *, bias: Tensor | None = None,
                      kernel_order: bool = False) -> Tensor:
    """The fused GEMM for bf16 activations (an extension: the reference takes fp16 only).

    ``x`` bf16 [M, K] is converted to fp16 by the library (exact for |x| in fp16's
    normal range, which holds for activations), the same fp16 GEMM runs, and its
    epilogue rounds the fp32 sums to bf16 (then adds the optional bf16 ``bias``,
    rounded again). Returns bf16 [M, N]. Weights are the usual fp16-scaled format."""
    assert x.is_cuda and x.dtype == torch.bfloat16, f"x must be bf16 on CUDA, got {x.dtype}"
    assert x.dim() == 2 and x.is_contiguous(), "x must be a contiguous 2D tensor"
    xh = to_fp16(x)
    w4a16_matmul(xh[:0], qweight, scales, zeros, group_size)   # the GEMM's argument checks
    M, K = x.shape
    N = qweight.shape[1]
    d = x.get_device()
    if bias is not None:
        assert bias.get_device() == d and bias.dtype == torch.bfloat16 and bias.shape == (N,) and \
            bias.is_contiguous(), f"bias must be a contiguous bf16 [{N}] tensor on the inputs' device"
    if out is None:
        out = torch.empty((M, N), device=d, dtype=torch.bfloat16)
    else:
        assert out.shape == (M, N) and out.dtype == torch.bfloat16 and out.is_contiguous()
        assert out.get_device() == d, "out must be on the inputs' CUDA device"
    _launch(xh, qweight, scales, zeros, bias, out, M, N, K, group_size, N,
            _lib.FLAG_BF16_OUT | (_lib.FLAG_KERNEL_ORDER if kernel_order else 0))
    return out


def repack_qweight(qweight: Tensor, to_kernel_order: bool = True, out: Tensor | None = None) -> Tensor:
    """``qweight`` [K/8, N] with its nibbles moved between the reference order (row
    8i+j in nibble j) and the kernel order (rows k0, k2, k4, k6, k1, k3, k5, k7 in
    nibbles 0..7) that the GEMMs read with ``kernel_order=True``. ``out`` may be
    ``qweight`` itself (in place). No reference counterpart: a load-time layout."""
    assert qweight.is_cuda and qweight.dtype == torch.int32 and qweight.dim() == 2
    assert qweight.is_contiguous(), "qweight must be contiguous"
    if out is None:
        out = torch.empty_like(qweight)
    assert out.shape == qweight.shape and out.dtype == torch.int32 and out.is_contiguous()
    Kp, N = qweight.shape
    with torch.cuda.device(qweight.device):
        st = _lib.lib().w4a16_repack(qweight.data_ptr(), out.data_ptr(), Kp * 8, N,
                                     1 if to_kernel_order else 0, _lib.stream_of(qweight.device))
    _lib.check(st, "w4a16_repack")
    return out


def swiglu(gate_up: Tensor, out: Tensor | None = None) -> Tensor:
    """``silu(g) * u`` for ``gate_up = [g | u]`` of shape [M, 2H] (fp16) -> [M, H]."""
    assert gate_up.is_cuda and gate_up.dtype == torch.float16 and gate_up.dim() == 2
    assert gate_up.is_contiguous() and gate_up.shape[1] % 2 == 0
    M, H2 = gate_up.shape
    H = H2 // 2
    if out is None:
        out = torch.empty((M, H), device=gate_up.device, dtype=torch.float16)
    dev = gate_up.device
    with torch.cuda.device(dev):
        st = _lib.lib().w4a16_swiglu(gate_up.data_ptr(), out.data_ptr(), M, H, H2, H,
                                     _lib.stream_of(dev))
    _lib.check(st, "w4a16_swiglu")
    return out


SWIGLU_BLOCK = 16


def interleave_gate_up(gate: Tensor, up: Tensor, block: int = SWIGLU_BLOCK) -> Tensor:
    """``[R, H]`` gate and up column blocks side by side in blocks of ``block``
    columns (gate block b, then up block b, ...): the ``[R, 2H]`` layout
    :func:`w4a16_matmul_swiglu` reads. Applies to qweight, scales and zeros alike."""
    assert gate.shape == up.shape and gate.dim() == 2 and gate.shape[1] % block == 0
    R, H = gate.shape
    return torch.stack([gate.reshape(R, H // block, block), up.reshape(R, H // block, block)],
                       dim=2).reshape(R, 2 * H).contiguous()


def w4a16_matmul_swiglu(x: Tensor, qweight: Tensor, scales: Tensor, zeros: Tensor, group_size: int,
                        out: Tensor | None = None, *, kernel_order: bool = False) -> Tensor:
    """``silu(x @ W_gate) * (x @ W_up)`` in one GEMM whose epilogue applies SwiGLU.

    ``qweight`` / ``scales`` / ``zeros`` hold the gate and up projections interleaved
    by :func:`interleave_gate_up` (``[K/8, 2H]`` etc.). Returns fp16 ``[M, H]``, the
    same values as :func:`swiglu` of the fp16 gate/up GEMM output (no extension of the
    reference: it fuses the MLP block's activation into the projection)."""
    w4a16_matmul(x[:0], qweight, scales, zeros, group_size)   # the GEMM's argument checks
    M, K = x.shape
    N = qweight.shape[1]
    assert N % (2 * SWIGLU_BLOCK) == 0, f"fused gate/up columns N={N} must be a multiple of {2 * SWIGLU_BLOCK}"
    assert all(t.data_ptr() % 16 == 0 for t in (x, qweight, scales, zeros)), "inputs must be 16-byte aligned"
    if out is None:
        out = torch.empty((M, N // 2), device=x.device, dtype=torch.float16)
    else:
        assert out.shape == (M, N // 2) and out.dtype == torch.float16 and out.is_contiguous()
        assert out.device == x.device, "out must be on the inputs' CUDA device"
    dev = x.device
    if dev.index != torch.cuda.current_device():
        with torch.cuda.device(dev):
            return w4a16_matmul_swiglu(x, qweight, scales, zeros, group_size, out)
    if M == 0:
        return out
    stream = _lib.stream_of(dev)
    ws = _lib.gemm_workspace(_lib.gemm_workspace_bytes(M, N, K, group_size, dev), dev, stream)
    flags = _lib.FLAG_SWIGLU | (_lib.FLAG_KERNEL_ORDER if kernel_order else 0)
    st = _lib.lib().w4a16_gemm_ex(x.data_ptr(), qweight.data_ptr(), scales.data_ptr(), zeros.data_ptr(), None,
                                  out.data_ptr(), M, N, K, group_size, N // 2, flags, _lib.ptr(ws),
                                  0 if ws is None else ws.numel(), stream)
    _lib.check(st, "w4a16_gemm_swiglu")
    return out


def stage_copy(dst: Tensor, src: Tensor, src_ready: bool = False) -> Tensor:
    """``dst.copy_(src)`` as a kernel that chains with the GEMMs around it.

    For loops captured in a CUDA graph: a step's input copied in (or its output
    copied out) by ``Tensor.copy_`` becomes a memory-copy node, and a GEMM after
    such a node waits for its predecessor to finish instead of overlapping its
    tail (programmatic dependent launch). ``dst`` and ``src`` are contiguous
    tensors of the same size in bytes (a multiple of 16), on the current CUDA
    device or in pinned host memory. ``src_ready=True`` promises that no earlier
    kernel on the stream writes ``src`` (e.g. a pinned host buffer the host
    filled): the copy then reads it while the previous kernel still runs. ``dst``
    is written after the previous kernel completes. No reference counterpart.
    """
    assert dst.is_contiguous() and src.is_contiguous(), "stage_copy needs contiguous tensors"
    nbytes = src.numel() * src.element_size()
    assert dst.numel() * dst.element_size() == nbytes, "stage_copy needs equal sizes"
    dev = dst.device if dst.is_cuda else src.device
    assert dev.type == "cuda", "stage_copy needs a CUDA tensor on one side"
    with torch.cuda.device(dev):
        st = _lib.lib().w4a16_stage(src.data_ptr(), dst.data_ptr(), nbytes, 1 if src_ready else 0,
                                    _lib.stream_of(dev))
    _lib.check(st, "w4a16_stage")
    return dst


_host_scratch: dict[int, tuple] = {}


def _device_scratch(d: int, xbytes: int, ybytes: int) -> tuple[int, int]:
    """Grow-only per-device staging buffers of :func:`w4a16_matmul_host` (256-byte
    aligned allocations; the next call on the stream may reuse them)."""
    ent = _host_scratch.get(d)
    if ent is None or ent[0] < xbytes or ent[1] < ybytes:
        xb = max(xbytes, 0 if ent is None else ent[0])
        yb = max(ybytes, 0 if ent is None else ent[1])
        bufs = (torch.empty(xb, dtype=torch.uint8, device=d), torch.empty(yb, dtype=torch.uint8, device=d))
        ent = (xb, yb, bufs[0].data_ptr(), bufs[1].data_ptr(), bufs)
        _host_scratch[d] = ent
    return ent[2], ent[3]


def w4a16_matmul_host(x: Tensor, qweight: Tensor, scales: Tensor, zeros: Tensor, group_size: int,
                      out: Tensor | None = None, *, bias: Tensor | None = None,
                      kernel_order: bool = False) -> Tensor:
    """The fused GEMM on host-resident activations: ``x`` is a pinned CPU fp16
    [M, K] tensor, the weights live on a CUDA device, and the fp16 [M, N] result is
    written into the pinned CPU tensor ``out`` (allocated pinned when omitted, which
    is slow: pass ``out`` in a loop). One C call stages x in, runs the GEMM and stages
    y out as three kernels chained under programmatic dependent launch on the
    weights' device's current stream; ``out`` holds the result once that stream has
    completed (e.g. ``torch.cuda.current_stream(dev).synchronize()``). Host memory
    that is not pinned raises :class:`W4A16Error`. No reference counterpart: an eager
    serving loop on host buffers without copy-engine round trips.
    """
    d = qweight.get_device()
    xs, qs = x.shape, qweight.shape
    # the common case in one expression; anything else gets the specific assertion
    if not (d >= 0 and not x.is_cuda and len(xs) == 2 and len(qs) == 2 and x.dtype is _F16
            and qweight.dtype is _I32 and scales.dtype is _F16 and zeros.dtype is _F16
            and qs[0] * 8 == xs[1] and group_size > 0 and xs[1] % group_size == 0
            and group_size % _BLOCK_K_RULE == 0 and scales.shape == (xs[1] // group_size, qs[1])
            and zeros.shape == scales.shape and scales.get_device() == d and zeros.get_device() == d
            and x.is_contiguous() and qweight.is_contiguous() and scales.is_contiguous()
            and zeros.is_contiguous()):
        assert d >= 0, "qweight must be on a CUDA device"
        assert not x.is_cuda, "x must be a pinned CPU tensor"
        assert x.dim() == 2 and x.dtype is _F16 and x.is_contiguous(), "x must be a contiguous fp16 [M, K] tensor"
        w4a16_matmul(torch.empty((0, xs[1]), device=d, dtype=_F16), qweight, scales, zeros, group_size)
    M, K = xs
    N = qs[1]
    if out is None:
        out = torch.empty((M, N), dtype=_F16, pin_memory=True)
    else:
        assert not out.is_cuda and out.shape == (M, N) and out.dtype is _F16 and out.is_contiguous(), (
            f"out must be a contiguous pinned CPU fp16 [{M}, {N}] tensor")
    if bias is not None:
        assert bias.get_device() == d and bias.dtype is _F16 and bias.shape == (N,) and bias.is_contiguous()
    if M == 0 or N == 0:
        return out
    if d != _current_device():
        with torch.cuda.device(d):
            return w4a16_matmul_host(x, qweight, scales, zeros, group_size, out, bias=bias, kernel_order=kernel_order)
    stream = _raw_stream(d)
    ws_ptr, ws_bytes = _lib.workspace_for(M, N, K, group_size, d, stream)
    x_dev, y_dev = _device_scratch(d, M * K * 2, M * N * 2)
    st = _lib.lib().w4a16_gemm_host(
        x.data_ptr(), qweight.data_ptr(), scales.data_ptr(), zeros.data_ptr(),
        None if bias is None else bias.data_ptr(), out.data_ptr(), M, N, K, group_size,
        _lib.FLAG_KERNEL_ORDER if kernel_order else 0, x_dev, y_dev, ws_ptr, ws_bytes, stream)
    if st:
        _lib.check(st, "w4a16_gemm_host")
    return out


def w4a16_matmul_into(x: Tensor, qweight: Tensor, scales: Tensor, zeros: Tensor, group_size: int,
                      y: Tensor, ldy: int, bias: Tensor | None = None) -> None:
    """Low-level variant: write ``Y`` into rows of pitch ``ldy`` starting at
    ``y``'s first element (e.g. one column shard of a wider output buffer).

    No shape assertions beyond what the C ABI checks; used by the sharded
    layers in :mod:`w4a16.parallel`.
    """
    M, K = x.shape
    N = qweight.shape[1]
    _launch(x, qweight, scales, zeros, bias, y, M, N, K, group_size, ldy)
