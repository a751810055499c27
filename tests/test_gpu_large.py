"""The benchmark configurations at full size.

The numpy oracle cannot finish these in seconds, so the checks are (a) a
plain-PyTorch fp32 reference on the GPU that restates the oracle's arithmetic
(tests/helpers.py), (b) the oracle itself on a few rows, and (c) properties
that hold at any size: column shards of the weight give the matching column
slice of the output, and row slices the matching rows (bit for bit unless a call
splits K across CTAs).
"""
from __future__ import annotations

import pytest
import torch

import oracle
from helpers import gpu_case, np_, torch_reference
from tolerance import assert_gemm_close
from w4a16 import quantize_weight, w4a16_matmul

pytestmark = pytest.mark.gpu


def _check(X, qw, s, z, G, what, oracle_rows=2):
    y = w4a16_matmul(X, qw, s, z, G)
    assert_gemm_close(np_(y), np_(torch_reference(X, qw, s, z, G)), what)
    r = min(oracle_rows, X.shape[0])
    if r:
        ref = oracle.reference_w4a16(np_(X[:r]), np_(qw), np_(s), np_(z), G)
        assert_gemm_close(np_(y[:r]), ref, what + " (oracle rows)")
    return y


def test_decode_configuration():
    """M=1, K=4096, N=11008, G=128, W ~ N(0, 0.02)."""
    X, W = gpu_case(1, 4096, 11008, 128, sigma=0.02, seed=2)
    qw, s, z = quantize_weight(W, 128)
    _check(X, qw, s, z, 128, "decode")


@pytest.mark.parametrize("M", [1, 4, 8, 16, 32])
def test_batched_decode_sweep_and_column_shards(M):
    """M in {1,4,8,16,32}, K=8192, N=28672, G=128, W ~ N(0, 0.015) with 0.1%
    outliers; plus the column shards each of 2/4/8 GPUs would own."""
    X, W = gpu_case(M, 8192, 28672, 128, sigma=0.015, seed=3, outlier_frac=0.001)
    qw, s, z = quantize_weight(W, 128)
    del W
    y = _check(X, qw, s, z, 128, f"sweep M={M}", oracle_rows=1 if M == 1 else 0)
    for p in (2, 8):
        n = 28672 // p
        for r in (0, p - 1):
            c = slice(r * n, (r + 1) * n)
            ys = w4a16_matmul(X, qw[:, c].contiguous(), s[:, c].contiguous(), z[:, c].contiguous(), 128)
            assert_gemm_close(np_(ys), np_(y[:, c]), f"shard {r}/{p}")


@pytest.mark.parametrize("M", [512, 2048, 4096, 8192])
def test_prefill_configuration(M):
    """M in {512,2048,4096,8192}, K=4096, N=14336, G=128 on the tcgen05 kernel."""
    X, W = gpu_case(M, 4096, 14336, 128, sigma=0.02, seed=4)
    qw, s, z = quantize_weight(W, 128)
    y = _check(X, qw, s, z, 128, f"prefill M={M}")
    # row slices are the matching rows: bit for bit when neither call splits K across
    # CTAs (the same summation order per output), within the GEMM tolerance otherwise
    rows = slice(M // 2, M // 2 + 256)
    ys = w4a16_matmul(X[rows].contiguous(), qw, s, z, 128)
    if _splits_k(M, 14336, 4096) or _splits_k(256, 14336, 4096):
        assert_gemm_close(np_(ys), np_(y[rows]).astype("float32"), f"row slice of M={M}")
    else:
        assert torch.equal(ys, y[rows])


def _splits_k(M, N, K, G=128):
    """True when the shape's prefill GEMM splits K across CTAs: the workspace it asks
    for reaches past the decode region."""
    import ctypes
    from w4a16 import _lib
    need = ctypes.c_int64(0)
    assert _lib.lib().w4a16_gemm_workspace_size(M, N, K, G, ctypes.byref(need)) == 0
    return need.value > 5 * 1024 * 1024


@pytest.mark.parametrize("M", [1, 2048])
def test_mlp_projection_shapes(M):
    """The MLP block's projections: gate/up 8192->28672 and down 28672->8192."""
    for K, N in ((8192, 28672), (28672, 8192)):
        X, W = gpu_case(M, K, N, 128, sigma=0.02, seed=K)
        qw, s, z = quantize_weight(W, 128)
        del W
        _check(X, qw, s, z, 128, f"mlp {K}->{N} M={M}", oracle_rows=0)
