"""Both prefill kernels (M > 32), each forced through w4a16_set_prefill_kernel:
the one whose dequantised weights are the shared-memory B operand of tcgen05.mma
and the one whose dequantised weights are the tensor-memory A operand. Each must
meet the GEMM tolerance against the oracle on its own, for every output form
(fp16 + bias, fp32 partials, bf16, fused SwiGLU, kernel nibble order, row pitch
without TMA stores), and the two must agree with each other.

Tolerance (tests/tolerance.py): |out - ref| <= 1e-2 + 1e-3*|ref| elementwise.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import w4a16
from helpers import gpu_case, np_, torch_reference
from tolerance import assert_gemm_close
from w4a16 import _lib, quantize_weight, w4a16_matmul

pytestmark = pytest.mark.gpu
KERNELS = {"smem_b": _lib.PREFILL_SMEM_B, "tmem_a": _lib.PREFILL_TMEM_A}


@pytest.fixture(params=sorted(KERNELS))
def kernel(request):
    _lib.set_prefill_kernel(KERNELS[request.param])
    try:
        yield request.param
    finally:
        _lib.set_prefill_kernel(_lib.PREFILL_AUTO)


def _build(M, K, N, G, sigma=1.0, seed=0):
    X, W = gpu_case(M, K, N, G, sigma=sigma, seed=seed)
    qw, s, z = quantize_weight(W, G)
    return X, qw, s, z


@pytest.mark.parametrize("M", [33, 64, 129, 200, 300, 777])
@pytest.mark.parametrize("K,N,G", [(64, 8, 64), (320, 264, 64), (1024, 520, 128), (768, 256, 256), (2048, 1000, 128)])
def test_prefill_kernel_matches_oracle(kernel, M, K, N, G):
    X, qw, s, z = _build(M, K, N, G, seed=M * 13 + N)
    y = w4a16_matmul(X, qw, s, z, G)
    assert _lib.check_device_errors() == 0
    assert_gemm_close(np_(y), oracle.reference_w4a16(np_(X), np_(qw), np_(s), np_(z), G), f"{kernel} M={M} N={N}")


@pytest.mark.parametrize("M", [100, 512])
def test_prefill_kernel_output_forms(kernel, M):
    """fp16 + bias (rounded as W4A16Linear's separate add), fp32 partials (the sums
    the fp16 output rounds), bf16 output of bf16 activations."""
    K, N, G = 1024, 776, 128
    X, qw, s, z = _build(M, K, N, G, sigma=0.05, seed=M)
    bias = (torch.randn(N, device="cuda") * 0.5).half()
    y = w4a16_matmul(X, qw, s, z, G)
    f32 = w4a16.w4a16_matmul_f32(X, qw, s, z, G)
    assert torch.equal(y, f32.half())
    yb = w4a16_matmul(X, qw, s, z, G, bias=bias)
    assert torch.equal(yb, (y.float() + bias.float()).half())
    xb = X.bfloat16()
    yh = w4a16.w4a16_matmul_bf16(xb, qw, s, z, G)
    assert torch.equal(yh, w4a16.w4a16_matmul_f32(w4a16.to_fp16(xb), qw, s, z, G).bfloat16())
    assert_gemm_close(np_(y), np_(torch_reference(X, qw, s, z, G)), f"{kernel} forms")


@pytest.mark.parametrize("M", [64, 300])
def test_prefill_kernel_order_and_swiglu(kernel, M):
    """Kernel nibble order gives the same bits as the reference order through the same
    kernel; the fused SwiGLU epilogue gives the same bits as the GEMM followed by the
    SwiGLU kernel."""
    K, H, G = 1024, 512, 128
    X, qw, s, z = _build(M, K, 2 * H, G, sigma=0.05, seed=M + 5)
    qk = w4a16.repack_qweight(qw)
    y = w4a16_matmul(X, qw, s, z, G)
    assert torch.equal(w4a16_matmul(X, qk, s, z, G, kernel_order=True), y)
    h = w4a16.w4a16_matmul_swiglu(X, qw, s, z, G)
    v = y.view(M, H // 16, 2, 16)
    plain = torch.cat([v[:, :, 0, :].reshape(M, H), v[:, :, 1, :].reshape(M, H)], dim=1).contiguous()
    assert torch.equal(h, w4a16.swiglu(plain))
    assert torch.equal(w4a16.w4a16_matmul_swiglu(X, qk, s, z, G, kernel_order=True), h)


@pytest.mark.parametrize("pad", [0, 3])
def test_prefill_kernel_row_pitch(kernel, pad):
    """Two column shards written into one wider buffer (pad 3: no TMA stores); nothing
    lands outside the shards."""
    from w4a16.gemm import w4a16_matmul_into
    M, K, N, G = 200, 1024, 264, 128
    X, qw, s, z = _build(M, K, 2 * N, G, sigma=0.05, seed=3)
    full = w4a16_matmul(X, qw, s, z, G)
    ldy = 2 * N + pad
    buf = torch.full((M, ldy), 7.0, device="cuda", dtype=torch.float16)
    for r in range(2):
        sl = slice(r * N, (r + 1) * N)
        w4a16_matmul_into(X, qw[:, sl].contiguous(), s[:, sl].contiguous(), z[:, sl].contiguous(), G,
                          buf[:, sl], ldy)
    torch.cuda.synchronize()
    assert_gemm_close(np_(buf[:, :2 * N]), np_(full).astype(np.float32), f"{kernel} row pitch")
    if pad:
        assert torch.all(buf[:, 2 * N:] == 7.0)


def test_prefill_kernels_agree_at_size():
    """The two kernels on one large shape (both within the tolerance of the torch fp32
    reference of the oracle math, and of each other)."""
    X, qw, s, z = _build(1536, 4096, 4096, 128, sigma=0.02, seed=9)
    out = {}
    try:
        for name, which in KERNELS.items():
            _lib.set_prefill_kernel(which)
            out[name] = w4a16_matmul(X, qw, s, z, 128)
    finally:
        _lib.set_prefill_kernel(_lib.PREFILL_AUTO)
    ref = np_(torch_reference(X, qw, s, z, 128))
    for name, y in out.items():
        assert_gemm_close(np_(y), ref, name)
    assert_gemm_close(np_(out["tmem_a"]), np_(out["smem_b"]).astype(np.float32), "kernels agree")
    assert _lib.check_device_errors() == 0


@pytest.mark.parametrize("M,N", [(4096, 14336), (4160, 14144), (4128, 4160)])
def test_prefill_partial_last_tiles_at_size(kernel, M, N):
    """Token and column counts that leave the last tiles partly empty (M = 4096 leaves 64
    of a 192-token tile; 4160 leaves 64 rows of a 256-row tile; N = 14144 and 4160 leave
    part of the last column tile), at a size that keeps every SM busy, so that the
    epilogue's TMA stores are still reading their staging buffers when the chunks past M
    or N come up: those chunks must leave the buffers alone. Repeated launches, checked
    on the device against the fp32 torch reference with the GEMM tolerance."""
    from tolerance import ATOL, RTOL
    K, G = 4096, 128
    X, qw, s, z = _build(M, K, N, G, sigma=0.02, seed=M + N)
    ref = torch_reference(X, qw, s, z, G).float()
    y = torch.empty(M, N, device="cuda", dtype=torch.float16)
    for rep in range(3):
        y.fill_(float("nan"))
        w4a16_matmul(X, qw, s, z, G, out=y)
        bad = ~((y.float() - ref).abs() <= ATOL + RTOL * ref.abs())
        if bool(bad.any()):
            rows, cols = torch.nonzero(bad, as_tuple=True)
            raise AssertionError(f"{kernel} M={M} N={N} launch {rep}: {int(bad.sum())} elements outside the "
                                 f"tolerance, rows {int(rows.min())}..{int(rows.max())}, "
                                 f"columns {int(cols.min())}..{int(cols.max())}")
    assert _lib.check_device_errors() == 0


def test_prefill_kernel_selection_rejects_unknown():
    with pytest.raises(RuntimeError):
        _lib.set_prefill_kernel(7)


def test_prefill_choice_query():
    """The per-shape choice: decode sizes report AUTO; a forced kernel is what the
    query reports; the automatic choice is one of the two kernels."""
    assert _lib.prefill_choice(32, 4096, 4096) == _lib.PREFILL_AUTO
    for M in (33, 512, 4096):
        assert _lib.prefill_choice(M, 14336, 4096) in (_lib.PREFILL_SMEM_B, _lib.PREFILL_TMEM_A)
    try:
        for which in KERNELS.values():
            _lib.set_prefill_kernel(which)
            assert _lib.prefill_choice(4096, 14336, 4096) == which
    finally:
        _lib.set_prefill_kernel(_lib.PREFILL_AUTO)


# ----------------------------------------------------------------- K split across CTAs
# Few tiles (one row of 256-column tiles) and a long K: the TMEM-operand kernel splits K
# over several CTAs per tile; the last split to arrive sums the fp32 partials in split order.
SPLIT_SHAPES = [(40, 4096, 1024, 128), (100, 8192, 2048, 128), (64, 2048, 512, 64), (200, 4096, 768, 128)]


def _check_split_case(M, K, N, G, seed):
    """The TMEM-operand kernel forced, on a shape it runs with K splits: identical bits on
    repeated calls, the fp32 sums, bias, SwiGLU and kernel-order forms agree with the plain
    output; returns (X, qw, s, z, y)."""
    X, qw, s, z = _build(M, K, N, G, sigma=0.05, seed=seed)
    _lib.set_prefill_kernel(_lib.PREFILL_TMEM_A)
    try:
        y1 = w4a16_matmul(X, qw, s, z, G)
        y2 = w4a16_matmul(X, qw, s, z, G)
        bias = (torch.randn(N, device="cuda") * 0.5).half()
        yb = w4a16_matmul(X, qw, s, z, G, bias=bias)
        f32 = w4a16.w4a16_matmul_f32(X, qw, s, z, G)
        h = w4a16.w4a16_matmul_swiglu(X, qw, s, z, G)
        yk = w4a16_matmul(X, w4a16.repack_qweight(qw), s, z, G, kernel_order=True)
    finally:
        _lib.set_prefill_kernel(_lib.PREFILL_AUTO)
    assert _lib.check_device_errors() == 0
    assert torch.equal(y1, y2), "split-K sums must not depend on which split arrives last"
    assert torch.equal(y1, f32.half())
    assert torch.equal(yb, (y1.float() + bias.float()).half())
    assert torch.equal(yk, y1)
    v = y1.view(M, N // 32, 2, 16)
    plain = torch.cat([v[:, :, 0, :].reshape(M, N // 2), v[:, :, 1, :].reshape(M, N // 2)], dim=1).contiguous()
    assert torch.equal(h, w4a16.swiglu(plain))
    return X, qw, s, z, y1


@pytest.mark.parametrize("M,K,N,G", SPLIT_SHAPES)
def test_split_k_matches_oracle_and_repeats(M, K, N, G):
    X, qw, s, z, y = _check_split_case(M, K, N, G, seed=M + K)
    assert_gemm_close(np_(y), oracle.reference_w4a16(np_(X), np_(qw), np_(s), np_(z), G), f"split M={M} K={K}")


# More tiles than CTAs with the last wave partly filled (tiles mod 148 = 2, 44, 64 at 128, 160
# and 192 tokens per tile): the tiles of the full waves run whole, the last wave's tiles are
# split into 2-3 parts whose partials the last split to arrive sums.
TAIL_SHAPES = [(200, 4096, 19200, 128), (300, 4096, 24576, 128), (500, 4096, 30720, 128)]


@pytest.mark.parametrize("M,K,N,G", TAIL_SHAPES)
def test_tail_split_matches_reference_and_repeats(M, K, N, G):
    import ctypes
    need = ctypes.c_int64(0)
    _lib.set_prefill_kernel(_lib.PREFILL_TMEM_A)
    try:
        assert _lib.lib().w4a16_gemm_workspace_size(M, N, K, G, ctypes.byref(need)) == 0
    finally:
        _lib.set_prefill_kernel(_lib.PREFILL_AUTO)
    assert need.value > 5 * 1024 * 1024, "this shape is expected to split the last wave's tiles"
    X, qw, s, z, y = _check_split_case(M, K, N, G, seed=M + N)
    assert_gemm_close(np_(y), np_(torch_reference(X, qw, s, z, G)), f"tail split M={M} N={N}")


def test_split_k_without_room_runs_unsplit():
    """A call given no (or too little) workspace, and the allocation-free entry point
    (whose static array leaves no room past the decode region), run without splitting K
    and still meet the tolerance."""
    import ctypes
    M, K, N, G = 40, 4096, 1024, 128
    X, qw, s, z = _build(M, K, N, G, sigma=0.05, seed=5)
    ref = oracle.reference_w4a16(np_(X), np_(qw), np_(s), np_(z), G)
    lib = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    _lib.set_prefill_kernel(_lib.PREFILL_TMEM_A)
    try:
        need = ctypes.c_int64(0)
        assert lib.w4a16_gemm_workspace_size(M, N, K, G, ctypes.byref(need)) == 0
        assert need.value > 5 * 1024 * 1024, "this shape is expected to split K"
        y = torch.empty(M, N, device="cuda", dtype=torch.float16)
        ptrs = (X.data_ptr(), qw.data_ptr(), s.data_ptr(), z.data_ptr())
        assert lib.w4a16_gemm(*ptrs, None, y.data_ptr(), M, N, K, G, N, None, 0, stream) == 0
        torch.cuda.synchronize()
        assert_gemm_close(np_(y), ref, "no workspace")
        small = torch.zeros(need.value // 2, dtype=torch.uint8, device="cuda")
        assert lib.w4a16_gemm(*ptrs, None, y.data_ptr(), M, N, K, G, N, small.data_ptr(), small.numel(),
                              stream) == 0
        torch.cuda.synchronize()
        assert_gemm_close(np_(y), ref, "small workspace")
        assert lib.w4a16_gemm_noalloc(*ptrs, None, y.data_ptr(), M, N, K, G, N, stream) == 0
        torch.cuda.synchronize()
        assert_gemm_close(np_(y), ref, "allocation-free")
    finally:
        _lib.set_prefill_kernel(_lib.PREFILL_AUTO)
    assert _lib.check_device_errors() == 0
