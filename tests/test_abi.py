"""The C-ABI library: it loads without a GPU, exports every symbol the header
declares, and rejects invalid arguments before touching a device."""
from __future__ import annotations

import ctypes
import os
import re

import pytest

from w4a16 import _lib

HEADER = os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "include", "w4a16_b200.h")


def _declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\**(w4a16_\w+)\s*\(", text, flags=re.M)))


def test_library_builds_and_loads():
    lib = _lib.lib()
    assert os.path.exists(_lib.LIB_PATH)
    assert lib.w4a16_version() >= 10000


def test_every_declared_symbol_is_exported():
    declared = _declared_functions()
    assert len(declared) >= 8, declared
    lib = _lib.lib()
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in the header but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_workspace_size_query_without_a_device():
    out = ctypes.c_int64(-1)
    lib = _lib.lib()
    assert lib.w4a16_gemm_workspace_size(1, 64, 100, 64, ctypes.byref(out)) == -1
    # the plain-load route (N % 8 != 0) needs no workspace and answers without a device;
    # the decode and prefill routes size theirs from the device's SM count
    assert lib.w4a16_gemm_workspace_size(4, 13, 256, 64, ctypes.byref(out)) == 0 and out.value == 0
    assert lib.w4a16_gemm_workspace_size(64, 13, 256, 64, ctypes.byref(out)) == 0 and out.value == 0
    assert lib.w4a16_gemm_workspace_size(64, 256, 256, 64, ctypes.byref(out)) == -4   # W4A16_ERR_DEVICE


def test_strerror_covers_every_status():
    for code in (0, -1, -2, -3, -4, -5, -6):
        s = _lib.strerror(code)
        assert s and s != "unknown w4a16 status"
    assert _lib.strerror(-99) == "unknown w4a16 status"


@pytest.mark.parametrize("M,N,K,G,ldy", [
    (1, 64, 100, 64, 64),      # K % 8
    (1, 64, 128, 96, 64),      # K % G
    (1, 64, 128, 32, 64),      # G % 64 (the reference's BLOCK_K rule)
    (1, 64, 128, 64, 32),      # ldy < N
    (-1, 64, 128, 64, 64),     # negative M
])
def test_gemm_rejects_bad_arguments_without_a_device(M, N, K, G, ldy):
    lib = _lib.lib()
    st = lib.w4a16_gemm(None, None, None, None, None, None, M, N, K, G, ldy, None, 0, None)
    assert st == -1


def test_gemm_empty_is_noop():
    assert _lib.lib().w4a16_gemm(None, None, None, None, None, None, 0, 64, 128, 64, 64, None, 0, None) == 0


def test_quantize_rejects_bad_arguments_without_a_device():
    lib = _lib.lib()
    assert lib.w4a16_quantize(None, 0, None, None, None, 100, 8, 4, None) == -1
    assert lib.w4a16_quantize(None, 0, None, None, None, 96, 8, 64, None) == -1
    assert lib.w4a16_pack_int4(None, None, 7, 4, None) == -1
    assert lib.w4a16_unpack_int4(None, None, 9, 4, None) == -1
    assert lib.w4a16_dequantize(None, None, None, None, 128, 8, 96, None) == -1


def test_check_device_errors_signature():
    fn = _lib.lib().w4a16_check_device_errors
    assert fn.argtypes[1] == ctypes.POINTER(ctypes.c_uint32)


@pytest.mark.parametrize("fn", ["w4a16_gemm_allreduce", "w4a16_gemm_allgather"])
@pytest.mark.parametrize("M,N,ldy,world,rank", [
    (33, 64, 128, 2, 0),            # more than 32 tokens
    (1, 60, 128, 2, 0),             # N % 8
    (1, 64, 128, 1, 0),             # one rank
    (1, 64, 128, 9, 0),             # more ranks than the buffers hold
    (1, 64, 128, 2, 2),             # rank outside the group
    (32, 1 << 28, 1 << 29, 2, 0),   # output beyond the finishing CTAs' 32-bit indices
])
def test_fused_collectives_reject_bad_arguments_without_a_device(fn, M, N, ldy, world, rank):
    lib = _lib.lib()
    peers = (ctypes.c_ulonglong * 8)()
    st = getattr(lib, fn)(None, None, None, None, None, None, M, N, 128, 64, ldy, None, 0,
                          peers, world, rank, None, M * N, None)
    assert st == -1   # W4A16_ERR_INVALID, before any device work


def test_allgather_needs_room_for_every_rank():
    lib = _lib.lib()
    peers = (ctypes.c_ulonglong * 8)()
    # y rows of 64 columns cannot hold 2 ranks x 64 columns
    assert lib.w4a16_gemm_allgather(None, None, None, None, None, None, 1, 64, 128, 64, 64, None, 0,
                                    peers, 2, 0, None, 64, None) == -1


@pytest.mark.parametrize("nbytes,src,dst", [
    (24, 16, 16),     # not a multiple of 16 bytes
    (-16, 16, 16),    # negative size
    (32, None, 16),   # no source
    (32, 16, None),   # no destination
])
def test_stage_rejects_bad_arguments_without_a_device(nbytes, src, dst):
    st = _lib.lib().w4a16_stage(src, dst, nbytes, 1, None)
    assert st == -1   # W4A16_ERR_INVALID, before any device work


def test_stage_rejects_misaligned_pointers_without_a_device():
    assert _lib.lib().w4a16_stage(8, 16, 32, 0, None) == -2   # W4A16_ERR_ALIGNMENT
    assert _lib.lib().w4a16_stage(16, 0, 0, 0, None) == 0      # nothing to copy


def test_wait_budget_setter_validates_without_a_device():
    lib = _lib.lib()
    assert lib.w4a16_set_wait_budget_ns(-1) == -1
    assert lib.w4a16_set_wait_budget_ns(999_999) == -1           # below 1 ms
    assert lib.w4a16_set_wait_budget_ns(601 * 10**9) == -1       # above 600 s
    assert lib.w4a16_set_wait_budget_ns(20_000_000) == 0
    assert lib.w4a16_set_wait_budget_ns(0) == 0                  # back to the default


def test_reset_scratch_rejects_bad_arguments_without_a_device():
    lib = _lib.lib()
    assert lib.w4a16_reset_scratch(None, 16, None) == -1
    assert lib.w4a16_reset_scratch(None, -1, None) == -1


@pytest.mark.parametrize("N,ldh", [(48, 24), (64, 31)])   # N % 32, ldh < N/2
def test_gemm_swiglu_rejects_bad_arguments_without_a_device(N, ldh):
    assert _lib.lib().w4a16_gemm_swiglu(None, None, None, None, None, 1, N, 128, 64, ldh, None, 0,
                                        None) == -1


def test_quantize_ex_rejects_unknown_bits_without_a_device():
    assert _lib.lib().w4a16_quantize_ex(None, 0, None, None, None, 64, 8, 64, 2, None) == -1
