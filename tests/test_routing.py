"""The prefill routing (which kernel, how many tokens per tile, how many K splits) as
the C library's cost model computes it on the host (w4a16_prefill_plan: no GPU needed),
for a 148-SM B200. It pins the choices the GPU tests and the benchmark rely on (the
shapes the K-split tests expect to split, the benchmark's prefill shapes) and the
plan's invariants over a grid of shapes.
"""
from __future__ import annotations

import itertools

import pytest

from w4a16 import _lib

SMS = 148
AUTO, SMEM_B, TMEM_A = _lib.PREFILL_AUTO, _lib.PREFILL_SMEM_B, _lib.PREFILL_TMEM_A


@pytest.fixture
def forced():
    """Force a prefill kernel for one test; back to the per-shape choice afterwards."""
    def force(which):
        _lib.set_prefill_kernel(which)
    yield force
    _lib.set_prefill_kernel(AUTO)


def test_decode_sizes_have_no_prefill_plan():
    for M in (1, 8, 32):
        assert _lib.prefill_plan(M, 14336, 4096, SMS) == (AUTO, 0, 1)


@pytest.mark.parametrize("M,N,K,sms", [(64, 4096, 4100, SMS), (64, 4096, 4096, 0), (0, 4096, 4096, SMS),
                                       (64, 0, 4096, SMS), (64, 4096, 0, SMS)])
def test_plan_rejects_bad_arguments(M, N, K, sms):
    with pytest.raises(RuntimeError):
        _lib.prefill_plan(M, N, K, sms)


def test_benchmark_prefill_shapes():
    """K=4096, N=14336: the tensor-memory-operand kernel at 2048-8192 tokens in 192-token
    tiles with the last, partly filled wave's tiles split in two; the shared-memory-operand
    kernel at 512 tokens (one wave of its 256-row tiles)."""
    for M in (2048, 4096, 8192):
        assert _lib.prefill_plan(M, 14336, 4096, SMS) == (TMEM_A, 192, 2), M
    assert _lib.prefill_plan(512, 14336, 4096, SMS)[0] == SMEM_B


def test_shapes_the_gpu_split_tests_expect_to_split(forced):
    """The K-split GPU tests force the tensor-memory-operand kernel and assert (through
    the workspace size) that these shapes split K: every tile when the tiles do not fill
    a wave, the last wave's tiles otherwise."""
    forced(TMEM_A)
    for M, K, N in [(40, 4096, 1024), (100, 8192, 2048), (200, 4096, 768),       # every tile
                    (200, 4096, 19200), (300, 4096, 24576), (500, 4096, 30720)]:  # last wave
        which, mt, sp = _lib.prefill_plan(M, N, K, SMS)
        assert which == TMEM_A and sp > 1, (M, K, N, mt, sp)


def test_plan_invariants(forced):
    """Over a grid of shapes: a legal tile height, 1-8 splits of at least 8 steps of 64 K
    each, the forced kernel reported as forced."""
    shapes = list(itertools.product([33, 64, 100, 128, 200, 512, 777, 2048, 4096, 8192],
                                    [8, 264, 1024, 4096, 14336, 28672, 57344],
                                    [64, 512, 2048, 4096, 8192, 28672]))
    for M, N, K in shapes:
        which, mt, sp = _lib.prefill_plan(M, N, K, SMS)
        assert which in (SMEM_B, TMEM_A)
        if which == TMEM_A:
            assert mt in (64, 96, 128, 160, 192) and 1 <= sp <= 8, (M, N, K, mt, sp)
            assert sp == 1 or (K // 64) // sp >= 8, (M, N, K, sp)
        else:
            assert (mt, sp) == (0, 1)
    forced(TMEM_A)
    assert all(_lib.prefill_plan(M, N, K, SMS)[0] == TMEM_A for M, N, K in shapes[::7])
    forced(SMEM_B)
    assert all(_lib.prefill_plan(M, N, K, SMS) == (SMEM_B, 0, 1) for M, N, K in shapes[::7])


def test_plan_follows_the_sm_count():
    """The plan is computed for the SM count passed in (waves of that many CTAs); every
    count gives a legal plan."""
    for sms in (1, 74, 132, 148, 160):
        which, mt, sp = _lib.prefill_plan(4096, 14336, 4096, sms)
        assert which in (SMEM_B, TMEM_A) and 1 <= sp <= 8
