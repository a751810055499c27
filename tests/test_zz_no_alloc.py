"""w4a16_gemm_noalloc: the workspace-free C entry point, called through the C
ABI, must give what the workspace entry point (w4a16_gemm via w4a16_matmul)
gives, on two calls in a row (the second reuses the static scratch the first
left behind). Named so it is collected last: it must pass both alone in a
fresh process and after every other test has used the library."""
from __future__ import annotations

import ctypes

import pytest
import torch

from helpers import gpu_case, np_
from tolerance import assert_gemm_close
from w4a16 import _lib, quantize_weight, w4a16_matmul

pytestmark = pytest.mark.gpu


def _noalloc(X, qw, s, z, G, bias=None):
    M, K = X.shape
    N = qw.shape[1]
    y = torch.empty((M, N), device=X.device, dtype=torch.float16)
    stream = torch.cuda.current_stream(X.device).cuda_stream
    st = _lib.lib().w4a16_gemm_noalloc(
        X.data_ptr(), qw.data_ptr(), s.data_ptr(), z.data_ptr(),
        bias.data_ptr() if bias is not None else None, y.data_ptr(), M, N, K, G, N, stream)
    assert st == 0, _lib.strerror(st)
    return y


@pytest.mark.parametrize("M,K,N,G", [
    (1, 4096, 11008, 128),   # decode: strips shared between CTAs (scratch used)
    (7, 1024, 264, 64),      # decode: ragged last strip
    (32, 2048, 4096, 128),   # decode: largest token count (most scratch)
    (130, 512, 256, 128),    # prefill route: no scratch
])
def test_noalloc_matches_workspace_entry_point_twice(M, K, N, G):
    X, W = gpu_case(M, K, N, G, sigma=0.05, seed=M + N)
    qw, s, z = quantize_weight(W, G)
    ref = np_(w4a16_matmul(X, qw, s, z, G))
    for call in range(2):
        y = _noalloc(X, qw, s, z, G)
        torch.cuda.synchronize()
        assert_gemm_close(np_(y), ref, f"noalloc call {call} M={M} K={K} N={N}")
    assert _lib.check_device_errors(X.device) == 0


def test_noalloc_with_bias_and_bad_arguments():
    M, K, N, G = 3, 1024, 512, 128
    X, W = gpu_case(M, K, N, G, sigma=0.05, seed=9)
    qw, s, z = quantize_weight(W, G)
    bias = torch.randn(N, device="cuda").half()
    ref = np_(w4a16_matmul(X, qw, s, z, G, bias=bias))
    for call in range(2):
        assert_gemm_close(np_(_noalloc(X, qw, s, z, G, bias)), ref, f"noalloc bias call {call}")
    y = torch.empty((M, N), device="cuda", dtype=torch.float16)
    # group size that is not a multiple of 64: rejected before any device work
    st = _lib.lib().w4a16_gemm_noalloc(X.data_ptr(), qw.data_ptr(), s.data_ptr(), z.data_ptr(),
                                       None, y.data_ptr(), M, N, K, 96, N,
                                       torch.cuda.current_stream().cuda_stream)
    assert st == -1   # W4A16_ERR_INVALID


def test_scratch_limit_status_has_text():
    text = _lib.strerror(-7)
    assert "static buffer" in text and "w4a16_gemm" in text
    out = ctypes.c_int64(0)
    # every decode shape on this device fits the static scratch
    assert _lib.lib().w4a16_gemm_workspace_size(32, 1 << 20, 8192, 128, ctypes.byref(out)) == 0
    assert 0 < out.value <= 5 * 1024 * 1024
