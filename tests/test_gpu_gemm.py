"""Fused GEMM (decode, prefill and fallback routes) vs the oracle.

Tolerance (tests/tolerance.py): |out - ref| <= 1e-2 + 1e-3*|ref| elementwise
on the fp16 output, against the reference's fp32-accumulated oracle on the
same quantised tensors. Ports the reference's test_correctness.py grid and
error checks, then covers every kernel route and its edges.
"""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

import oracle
import synth
import w4a16
from helpers import gpu_case, np_, torch_reference
from tolerance import assert_gemm_close
from w4a16 import W4A16Linear, quantize_weight, w4a16_matmul

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _oracle_y(X, qw, s, z, G):
    return oracle.reference_w4a16(np_(X), np_(qw), np_(s), np_(z), G)


def _build(M, K, N, G, sigma=1.0, seed=0):
    X, W = gpu_case(M, K, N, G, sigma=sigma, seed=seed)
    qw, s, z = quantize_weight(W, G)
    return X, qw, s, z


# ---------------------------- golden vectors from the reference --------------------
def test_golden_cases_match_reference_outputs():
    g = np.load(os.path.join(GOLDEN, "golden_small.npz"))
    names = sorted({k.split("/")[0] for k in g.files if not k.startswith("pack_")})
    for name in names:
        M, K, N, G = (int(v) for v in g[f"{name}/meta"])
        if G % 64:
            continue
        t = lambda k: torch.from_numpy(g[f"{name}/{k}"]).cuda()  # noqa: E731
        y = w4a16_matmul(t("X"), t("qweight"), t("scales"), t("zeros"), G)
        assert_gemm_close(np_(y), g[f"{name}/y_ref"], name)


def test_oracle_configuration_output():
    """16x4096x4096, G=128: the GPU result vs the reference's stored output."""
    ref = np.load(os.path.join(GOLDEN, "golden_oracle_cfg.npz"))
    X, W = synth.oracle_cfg_inputs()
    qw, s, z = quantize_weight(torch.from_numpy(W).cuda(), 128)
    y = w4a16_matmul(torch.from_numpy(X).cuda(), qw, s, z, 128)
    assert_gemm_close(np_(y), ref["y_ref"], "oracle configuration")


# ---------------------------- the reference's grid (test_correctness.py:35-46) ------
@pytest.mark.parametrize("M", [1, 16, 64, 256])
@pytest.mark.parametrize("K,N", [(4096, 4096), (4096, 11008), (11008, 4096)])
@pytest.mark.parametrize("group_size", [64, 128])
def test_matches_reference_grid(M, K, N, group_size):
    X, qw, s, z = _build(M, K, N, group_size)
    y = w4a16_matmul(X, qw, s, z, group_size)
    assert y.shape == (M, N) and y.dtype == torch.float16
    ref = _oracle_y(X, qw, s, z, group_size)
    assert_gemm_close(np_(y), ref, f"M={M} K={K} N={N} G={group_size}")
    torch.testing.assert_close(y, torch.from_numpy(ref).cuda(), rtol=1e-2, atol=1e-2)


# ---------------------------- every route and its edges ----------------------------
@pytest.mark.parametrize("M", [1, 2, 7, 8, 9, 15, 16, 17, 24, 25, 31, 32])
@pytest.mark.parametrize("K,N,G", [(256, 128, 64), (320, 72, 64), (1024, 264, 256), (576, 1000, 192),
                                   (1536, 136, 512), (3072, 128, 1024)])
def test_decode_route(M, K, N, G):
    X, qw, s, z = _build(M, K, N, G, seed=M * 31 + K)
    assert_gemm_close(np_(w4a16_matmul(X, qw, s, z, G)), _oracle_y(X, qw, s, z, G), f"decode M={M}")


@pytest.mark.parametrize("M", [33, 100, 127, 128, 129, 255, 300])
@pytest.mark.parametrize("K,N,G", [(64, 8, 64), (320, 264, 64), (1024, 520, 128), (768, 256, 256)])
def test_prefill_route(M, K, N, G):
    X, qw, s, z = _build(M, K, N, G, seed=M * 17 + N)
    assert_gemm_close(np_(w4a16_matmul(X, qw, s, z, G)), _oracle_y(X, qw, s, z, G), f"prefill M={M}")


@pytest.mark.parametrize("M", [1, 5, 33, 70])
@pytest.mark.parametrize("N", [1, 13, 100, 254])
def test_fallback_route_odd_n(M, N):
    """N not a multiple of 8 cannot use TMA: the plain-load kernel takes it."""
    X, qw, s, z = _build(M, 256, N, 64, seed=N)
    assert_gemm_close(np_(w4a16_matmul(X, qw, s, z, 64)), _oracle_y(X, qw, s, z, 64), f"fallback N={N}")


def test_unaligned_views_use_fallback():
    X, qw, s, z = _build(3, 256, 64, 64)
    big = torch.zeros(3 * 256 + 8, dtype=torch.float16, device="cuda")
    Xv = big[4:4 + 3 * 256].view(3, 256)      # 8-byte aligned, not 16
    Xv.copy_(X)
    assert Xv.data_ptr() % 16 != 0
    assert_gemm_close(np_(w4a16_matmul(Xv, qw, s, z, 64)), _oracle_y(X, qw, s, z, 64), "unaligned")


def test_empty_and_out_argument():
    X, qw, s, z = _build(4, 256, 64, 64)
    y0 = w4a16_matmul(X[:0], qw, s, z, 64)
    assert y0.shape == (0, 64)
    out = torch.full((4, 64), 7.0, dtype=torch.float16, device="cuda")
    y = w4a16_matmul(X, qw, s, z, 64, out=out)
    assert y.data_ptr() == out.data_ptr()
    assert_gemm_close(np_(out), _oracle_y(X, qw, s, z, 64), "out=")


@pytest.mark.parametrize("M", [1, 20, 200])
def test_fused_bias_rounds_like_separate_add(M):
    """Epilogue bias == the reference's separate fp16 ``y + bias`` bit for bit."""
    X, qw, s, z = _build(M, 512, 264, 128, seed=M)
    bias = torch.randn(264, device="cuda").half()
    y = w4a16_matmul(X, qw, s, z, 128)
    yb = w4a16_matmul(X, qw, s, z, 128, bias=bias)
    assert torch.equal(yb, y + bias)


def test_deterministic():
    for M in (1, 16, 300):
        X, qw, s, z = _build(M, 1024, 512, 128, seed=M)
        a = w4a16_matmul(X, qw, s, z, 128)
        b = w4a16_matmul(X, qw, s, z, 128)
        assert torch.equal(a, b)


def test_cuda_graph_capture_replays_identically():
    X, qw, s, z = _build(8, 1024, 512, 128)
    y = torch.empty(8, 512, dtype=torch.float16, device="cuda")
    w4a16_matmul(X, qw, s, z, 128, out=y)       # warm-up outside capture
    torch.cuda.synchronize()
    ref = y.clone()
    y.zero_()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        w4a16_matmul(X, qw, s, z, 128, out=y)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, ref)


def test_non_default_stream():
    X, qw, s, z = _build(16, 512, 256, 128)
    ref = w4a16_matmul(X, qw, s, z, 128)
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        y = w4a16_matmul(X, qw, s, z, 128)
    st.synchronize()
    assert torch.equal(y, ref)


# ---------------------------- error behaviour (test_correctness.py:49-70) -----------
def test_kernel_asserts_contiguity():
    X, qw, s, z = _build(8, 128, 64, 64)
    X_bad = torch.randn(128, 8, dtype=torch.float16, device="cuda").t()
    assert not X_bad.is_contiguous()
    with pytest.raises(AssertionError):
        w4a16_matmul(X_bad, qw, s, z, 64)


def test_kernel_rejects_bad_group_size():
    X, W = gpu_case(8, 64, 64, 8)
    qw, s, z = quantize_weight(W, 8)
    with pytest.raises(AssertionError):
        w4a16_matmul(X, qw, s, z, 8)


def test_kernel_rejects_bad_dtypes_and_shapes():
    X, qw, s, z = _build(2, 128, 64, 64)
    with pytest.raises(AssertionError):
        w4a16_matmul(X.float(), qw, s, z, 64)
    with pytest.raises(AssertionError):
        w4a16_matmul(X, qw, s[:1], z, 64)
    with pytest.raises(AssertionError):
        w4a16_matmul(X[:, :120], qw, s, z, 64)


# ---------------------------- module (test_correctness.py:73-89) --------------------
def test_w4a16_linear_end_to_end():
    torch.manual_seed(2)
    K, N, M = 4096, 4096, 16
    lin = torch.nn.Linear(K, N, bias=True).cuda().half()
    qlin = W4A16Linear.from_linear(lin, group_size=128)
    x = torch.randn(M, K, dtype=torch.float16, device="cuda")
    y = qlin(x)
    ref = oracle.reference_w4a16(np_(x), np_(qlin.qweight), np_(qlin.scales), np_(qlin.zeros), 128)
    ref_b = (torch.from_numpy(ref).cuda() + qlin.bias)
    assert y.shape == (M, N)
    torch.testing.assert_close(y, ref_b, rtol=1e-2, atol=1e-2)
    # the module's weights are the reference quantiser's, bit for bit
    want = oracle.quantize_weight(np_(lin.weight.detach().t().contiguous()), 128)
    assert np.array_equal(np_(qlin.qweight), want[0])


def test_w4a16_linear_3d_input_and_no_bias():
    lin = torch.nn.Linear(512, 264, bias=False).cuda().half()
    qlin = W4A16Linear.from_linear(lin, group_size=64)
    x = torch.randn(2, 3, 512, dtype=torch.float16, device="cuda")
    y = qlin(x)
    assert y.shape == (2, 3, 264)
    ref = _oracle_y(x.reshape(6, 512), qlin.qweight, qlin.scales, qlin.zeros, 64)
    assert_gemm_close(np_(y.reshape(6, 264)), ref, "3d")


def test_w4a16_linear_from_cpu_linear():
    lin = torch.nn.Linear(256, 64, bias=True).half()
    qlin = W4A16Linear.from_linear(lin, group_size=128)
    assert not qlin.qweight.is_cuda
    qlin = qlin.cuda()
    x = torch.randn(5, 256, dtype=torch.float16, device="cuda")
    y = qlin(x)
    ref = torch.from_numpy(_oracle_y(x, qlin.qweight, qlin.scales, qlin.zeros, 128)).cuda() + qlin.bias
    assert_gemm_close(np_(y), np_(ref), "cpu-built module")


# ---------------------------- cross-route consistency -------------------------------
def test_decode_and_prefill_routes_agree():
    """The same rows through the decode route (M <= 32 slices) and the prefill
    route (all rows at once) agree within the tolerance -- a size-independent
    property that does not need the oracle."""
    X, qw, s, z = _build(96, 2048, 768, 128, sigma=0.02)
    full = w4a16_matmul(X, qw, s, z, 128)
    parts = torch.cat([w4a16_matmul(X[i:i + 32].contiguous(), qw, s, z, 128) for i in range(0, 96, 32)])
    assert_gemm_close(np_(parts), np_(full), "decode vs prefill")
    assert_gemm_close(np_(full), np_(torch_reference(X, qw, s, z, 128)), "vs torch fp32")


@pytest.mark.parametrize("M", [5, 300])
@pytest.mark.parametrize("pad", [0, 8, 3])
def test_column_slices_of_a_wider_output(M, pad):
    """Two column shards written into one [M, 2N + pad] buffer through the row-pitch
    argument (decode and prefill routes; pitches that allow TMA stores and one that
    does not). Every element outside the shards keeps its sentinel value."""
    from w4a16.gemm import w4a16_matmul_into
    K, N, G = 1024, 264, 128
    X, W = gpu_case(M, K, 2 * N, G, sigma=0.05, seed=7 + M)
    qw, s, z = quantize_weight(W, G)
    full = w4a16_matmul(X, qw, s, z, G)
    ldy = 2 * N + pad
    buf = torch.full((M, ldy), 7.0, device="cuda", dtype=torch.float16)
    for r in range(2):
        sl = slice(r * N, (r + 1) * N)
        w4a16_matmul_into(X, qw[:, sl].contiguous(), s[:, sl].contiguous(), z[:, sl].contiguous(), G,
                          buf[:, sl], ldy)
    torch.cuda.synchronize()
    # (stream-K split points depend on N, so the fp32 summation order may differ)
    assert_gemm_close(np_(buf[:, :2 * N]), np_(full).astype(np.float32), "column slices")
    if pad:
        assert torch.all(buf[:, 2 * N:] == 7.0), "a store landed outside the shards"


# ---------------------------- host-resident activations (w4a16.w4a16_matmul_host) --
@pytest.mark.parametrize("M,K,N,G", [(1, 4096, 11008, 128), (5, 1024, 264, 64), (32, 2048, 512, 128),
                                     (300, 1024, 520, 128)])
def test_matmul_host_matches_device_path(M, K, N, G):
    """Pinned x in, pinned y out through one call (stage in, GEMM, stage out): the same
    bits as the device GEMM on the same inputs, with and without bias and in the
    kernel nibble order; repeated calls reuse the staging buffers."""
    X, qw, s, z = _build(M, K, N, G, sigma=0.05, seed=M + N)
    bias = torch.randn(N, device="cuda").half()
    xh = X.cpu().pin_memory()
    yh = torch.empty(M, N, dtype=torch.float16).pin_memory()
    for b in (None, bias):
        want = w4a16_matmul(X, qw, s, z, G, bias=b)
        for _ in range(2):
            yh.fill_(0)
            w4a16.w4a16_matmul_host(xh, qw, s, z, G, out=yh, bias=b)
            torch.cuda.current_stream().synchronize()
            assert torch.equal(yh.cuda(), want)
    qk = w4a16.repack_qweight(qw)
    got = w4a16.w4a16_matmul_host(xh, qk, s, z, G, kernel_order=True)
    torch.cuda.current_stream().synchronize()
    assert torch.equal(got.cuda(), w4a16_matmul(X, qk, s, z, G, kernel_order=True))


def test_matmul_host_rejects_unpinned_and_device_inputs():
    X, qw, s, z = _build(4, 256, 64, 64)
    with pytest.raises(AssertionError):
        w4a16.w4a16_matmul_host(X, qw, s, z, 64)               # x on the device
    with pytest.raises(w4a16.W4A16Error):
        w4a16.w4a16_matmul_host(X.cpu(), qw, s, z, 64)         # x not pinned: the C ABI refuses it


# ---------------------------- staging copies (w4a16.stage_copy) --------------------
def test_stage_copy_host_device_and_back():
    from w4a16 import stage_copy
    g = torch.Generator().manual_seed(11)
    src = torch.randint(-2**31, 2**31 - 1, (4096 + 48,), generator=g, dtype=torch.int32).pin_memory()
    for ready in (True, False):
        d = torch.empty(src.shape, dtype=torch.int32, device="cuda")
        stage_copy(d, src, src_ready=ready)
        torch.cuda.synchronize()
        assert torch.equal(d.cpu(), src)
    back = torch.empty_like(src).pin_memory()
    stage_copy(back, d)
    d2 = torch.empty_like(d)
    stage_copy(d2, d)
    torch.cuda.synchronize()
    assert torch.equal(back, src) and torch.equal(d2, d)


def test_stage_copy_rejects_what_the_device_cannot_reach():
    from w4a16 import W4A16Error, stage_copy
    pageable = torch.zeros(64, dtype=torch.int32)   # not pinned: refused before any launch
    with pytest.raises(W4A16Error):
        stage_copy(torch.empty(64, dtype=torch.int32, device="cuda"), pageable)
    with pytest.raises(W4A16Error):   # 8 bytes: not a multiple of 16
        stage_copy(torch.empty(2, dtype=torch.int32, device="cuda"),
                   torch.zeros(2, dtype=torch.int32, device="cuda"))


def test_stage_copy_then_gemm_replayed_from_a_graph():
    """x staged in from pinned memory by a kernel, then the decode GEMM, step after
    step in one CUDA graph: the same bits as the eager GEMM."""
    from w4a16 import stage_copy
    X, qw, s, z = _build(1, 4096, 1024, 128, seed=3)
    Xh = X.cpu().pin_memory()
    Xd = [torch.empty_like(X) for _ in range(2)]
    Y = [torch.empty(1, 1024, device="cuda", dtype=torch.float16) for _ in range(6)]
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        stage_copy(Xd[0], Xh, src_ready=True)
        w4a16_matmul(Xd[0], qw, s, z, 128, out=Y[0])
    torch.cuda.synchronize()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.stream(st):
        with torch.cuda.graph(gr, stream=st):
            for i in range(6):
                stage_copy(Xd[i % 2], Xh, src_ready=True)
                w4a16_matmul(Xd[i % 2], qw, s, z, 128, out=Y[i])
        gr.replay()
    torch.cuda.synchronize()
    ref = w4a16_matmul(X, qw, s, z, 128)
    for i in range(6):
        assert torch.equal(Y[i], ref), f"step {i}"


# ----------------------------------------------------------------------------- kernel nibble order
def _np_repack(qw: np.ndarray) -> np.ndarray:
    """Reference nibble j -> kernel nibble {0,4,1,5,2,6,3,7}[j], restated in numpy."""
    w = qw.view(np.uint32)
    out = np.zeros_like(w)
    for j in range(8):
        pos = (j >> 1) | ((j & 1) << 2)
        out |= ((w >> np.uint32(4 * j)) & np.uint32(0xF)) << np.uint32(4 * pos)
    return out.view(np.int32)


def test_repack_layout_and_round_trip():
    qw = torch.randint(-2**31, 2**31 - 1, (96, 264), dtype=torch.int64).to(torch.int32).cuda()
    k = w4a16.repack_qweight(qw)
    assert np.array_equal(np_(k), _np_repack(np_(qw)))
    assert torch.equal(w4a16.repack_qweight(k, False), qw)
    inplace = qw.clone()
    w4a16.repack_qweight(inplace, True, out=inplace)
    assert torch.equal(inplace, k)


@pytest.mark.parametrize("M,K,N,G", [(1, 4096, 11008, 128), (7, 1024, 264, 64), (32, 2048, 512, 128),
                                     (33, 512, 256, 128), (300, 1024, 264, 128)])
def test_kernel_order_gemm_matches_oracle(M, K, N, G):
    X, W = gpu_case(M, K, N, G, sigma=0.05, seed=M + 5)
    qw, s, z = quantize_weight(W, G)
    ref = oracle.reference_w4a16(np_(X), np_(qw), np_(s), np_(z), G)
    bias = torch.randn(N, device="cuda").half()
    y = w4a16_matmul(X, w4a16.repack_qweight(qw), s, z, G, kernel_order=True)
    assert_gemm_close(np_(y), ref, f"kernel order M={M}")
    yb = w4a16_matmul(X, w4a16.repack_qweight(qw), s, z, G, bias=bias, kernel_order=True)
    assert_gemm_close(np_(yb), (ref + np_(bias)).astype(np.float16), f"kernel order + bias M={M}")


def test_linear_repack_keeps_reference_state_dict():
    lin = torch.nn.Linear(512, 264, bias=True).cuda().half()
    a = w4a16.W4A16Linear.from_linear(lin, group_size=128)
    b = w4a16.W4A16Linear.from_linear(lin, group_size=128).repack_()
    x = torch.randn(5, 512, device="cuda").half()
    assert_gemm_close(np_(b(x)), np_(a(x)), "repacked module")
    sa, sb = a.state_dict(), b.state_dict()
    assert sa.keys() == sb.keys() and all(torch.equal(sa[k], sb[k]) for k in sa)
    c = w4a16.W4A16Linear(512, 264, group_size=128, device="cuda").repack_()
    c.load_state_dict(sa)
    assert torch.equal(c.qweight, b.qweight) and torch.equal(c(x), b(x))


# ----------------------------------------------------------------------------- bf16 activations
@pytest.mark.parametrize("M,K,N,G", [(1, 4096, 11008, 128), (9, 1024, 264, 64), (40, 512, 256, 128),
                                     (300, 1024, 512, 128), (3, 256, 60, 64)])
@pytest.mark.parametrize("kernel_order", [False, True])
def test_bf16_activations(M, K, N, G, kernel_order):
    if kernel_order and N % 8:
        pytest.skip("the kernel nibble order needs the TMA route (N % 8 == 0)")
    X, W = gpu_case(M, K, N, G, sigma=0.05, seed=M + 11)
    xb = X.bfloat16()
    qw, s, z = quantize_weight(W, G)
    qk = w4a16.repack_qweight(qw) if kernel_order else qw
    bias = torch.randn(N, device="cuda").bfloat16()
    y = w4a16.w4a16_matmul_bf16(xb, qk, s, z, G, kernel_order=kernel_order)
    assert y.dtype == torch.bfloat16 and y.shape == (M, N)
    # the same fp32 sums as the fp16 GEMM of the converted x, rounded once to bf16
    xh = w4a16.to_fp16(xb)
    assert torch.equal(xh.float(), xb.float())            # |x| in fp16's normal range: exact
    f32 = w4a16.w4a16_matmul_f32(xh, qk, s, z, G, kernel_order=kernel_order)
    assert torch.equal(y, f32.bfloat16())
    ref = torch_reference(xh, qw, s, z, G).float()       # fp32 oracle math on the GPU
    assert float((y.float() - ref).abs().max()) <= 1e-2 + 8e-3 * float(ref.abs().max())
    yb = w4a16.w4a16_matmul_bf16(xb, qk, s, z, G, bias=bias, kernel_order=kernel_order)
    assert torch.equal(yb, (y.float() + bias.float()).bfloat16())
