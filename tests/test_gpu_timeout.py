"""The bounded-wait failure path on one GPU, without faulting it.

A fused row-parallel call (``w4a16_gemm_allreduce``) runs as rank 0 of a
two-rank group whose "peer buffers" are two local buffers: rank 0 writes its
words into both, but nothing ever writes rank 1's slot, so the call's finishing
CTAs wait for words that never come. With a 20 ms wait budget they give up,
set the sticky device flag and return; the host reads ``W4A16_ERR_TIMEOUT``.
The library must then be usable again: the flag is clear after the read, the
scratch is re-zeroed, and the next GEMMs (workspace and allocation-free entry
points) match the oracle. The context stays healthy throughout: no trap, no
fault, no endless wait."""
from __future__ import annotations

import ctypes
import time

import pytest
import torch

import oracle
from helpers import gpu_case, np_
from tolerance import assert_gemm_close
from w4a16 import _lib, quantize_weight, w4a16_matmul

pytestmark = pytest.mark.gpu


def test_allreduce_wait_runs_out_reports_timeout_and_recovers():
    lib = _lib.lib()
    dev = torch.device("cuda", torch.cuda.current_device())
    M, K, N, G = 2, 1024, 512, 128
    X, W = gpu_case(M, K, N, G, sigma=0.05, seed=5)
    qw, s, z = quantize_weight(W, G)
    ref = oracle.reference_w4a16(np_(X), np_(qw), np_(s), np_(z), G)
    assert _lib.check_device_errors(dev) == 0   # start from a clear flag

    slot = (M * N + 1) // 2 * 2
    nbytes = ctypes.c_int64(0)
    assert lib.w4a16_p2p_buffer_bytes(2, slot, ctypes.byref(nbytes)) == 0
    bufs = [torch.zeros(nbytes.value, dtype=torch.uint8, device=dev) for _ in range(2)]
    peers = (ctypes.c_ulonglong * 2)(bufs[0].data_ptr(), bufs[1].data_ptr())
    ctl = torch.zeros(4, dtype=torch.int32, device=dev)
    y = torch.empty((M, N), dtype=torch.float16, device=dev)
    stream = _lib.stream_of(dev)
    ws = _lib.gemm_workspace(_lib.gemm_workspace_bytes(M, N, K, G, dev), dev, stream)

    _lib.set_wait_budget_ns(20_000_000)   # 20 ms
    try:
        st = lib.w4a16_gemm_allreduce(
            X.data_ptr(), qw.data_ptr(), s.data_ptr(), z.data_ptr(), None, y.data_ptr(),
            M, N, K, G, N, _lib.ptr(ws), 0 if ws is None else ws.numel(), peers, 2, 0,
            ctl.data_ptr(), slot, stream)
        assert st == 0, _lib.strerror(st)
        t0 = time.perf_counter()
        flags = ctypes.c_uint32(0)
        st = lib.w4a16_check_device_errors(stream, ctypes.byref(flags))
        waited = time.perf_counter() - t0
    finally:
        _lib.set_wait_budget_ns(0)
    assert st == _lib.W4A16_ERR_TIMEOUT, _lib.strerror(st)
    assert flags.value & 1
    assert waited < 3.0, f"the 20 ms budget did not bound the wait ({waited:.2f} s)"
    # the read cleared the flag; every launch since then is clean again
    assert _lib.check_device_errors(dev) == 0

    # recovery: zero the scratch the abandoned call may have left, then compute again
    _lib.reset_workspaces()
    for _ in range(2):
        assert_gemm_close(np_(w4a16_matmul(X, qw, s, z, G)), ref, "GEMM after a timeout")
        y2 = torch.empty((M, N), dtype=torch.float16, device=dev)
        st = lib.w4a16_gemm_noalloc(X.data_ptr(), qw.data_ptr(), s.data_ptr(), z.data_ptr(), None,
                                    y2.data_ptr(), M, N, K, G, N, stream)
        assert st == 0, _lib.strerror(st)
        assert_gemm_close(np_(y2), ref, "allocation-free GEMM after a timeout")
    assert _lib.check_device_errors(dev) == 0

