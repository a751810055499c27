"""ctypes binding of the sm_100a C-ABI library (``include/w4a16_b200.h``).

The shared library is built in-tree by ``build.py`` (or ``__graft_entry__.build()``)
next to this file. Loading it needs no GPU; calling into it needs a B200
(sm_100). There is no CPU fallback: if the library is missing, every GEMM /
quantisation entry point raises ``RuntimeError`` naming the missing file.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libw4a16_b200.so")

W4A16_OK = 0
FLAG_KERNEL_ORDER = 1
FLAG_SWIGLU = 2
FLAG_F32_OUT = 4
FLAG_BF16_OUT = 8
PREFILL_AUTO, PREFILL_SMEM_B, PREFILL_TMEM_A = 0, 1, 2
W4A16_ERR_TIMEOUT = -5
W4A16_ERR_WORKSPACE = -6
DTYPE_CODES = {torch.float16: 0, torch.float32: 1, torch.bfloat16: 2}

# Every symbol the header declares, with its ctypes signature.
_c_i64 = ctypes.c_int64
_vp = ctypes.c_void_p
SIGNATURES = {
    "w4a16_version": ([], ctypes.c_int),
    "w4a16_strerror": ([ctypes.c_int], ctypes.c_char_p),
    "w4a16_gemm": ([_vp, _vp, _vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _vp,
                    _c_i64, _vp], ctypes.c_int),
    "w4a16_gemm_f32": ([_vp, _vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _vp,
                        _c_i64, _vp], ctypes.c_int),
    "w4a16_swiglu": ([_vp, _vp, _c_i64, _c_i64, _c_i64, _c_i64, _vp], ctypes.c_int),
    "w4a16_gemm_ex": ([_vp, _vp, _vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_uint32,
                       _vp, _c_i64, _vp], ctypes.c_int),
    "w4a16_repack": ([_vp, _vp, _c_i64, _c_i64, ctypes.c_int, _vp], ctypes.c_int),
    "w4a16_convert": ([_vp, ctypes.c_int, _vp, ctypes.c_int, _c_i64, _vp], ctypes.c_int),
    "w4a16_gemm_swiglu": ([_vp, _vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _vp, _c_i64,
                           _vp], ctypes.c_int),
    "w4a16_stage": ([_vp, _vp, _c_i64, ctypes.c_int, _vp], ctypes.c_int),
    "w4a16_gemm_host": ([_vp] * 6 + [_c_i64] * 4 + [ctypes.c_uint32] + [_vp] * 3 + [_c_i64, _vp], ctypes.c_int),
    "w4a16_gemm_workspace_size": ([_c_i64, _c_i64, _c_i64, _c_i64, ctypes.POINTER(_c_i64)],
                                  ctypes.c_int),
    "w4a16_quantize": ([_vp, ctypes.c_int, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _vp], ctypes.c_int),
    "w4a16_quantize_ex": ([_vp, ctypes.c_int, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, ctypes.c_uint32, _vp],
                          ctypes.c_int),
    "w4a16_pack_int4": ([_vp, _vp, _c_i64, _c_i64, _vp], ctypes.c_int),
    "w4a16_unpack_int4": ([_vp, _vp, _c_i64, _c_i64, _vp], ctypes.c_int),
    "w4a16_dequantize": ([_vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _vp], ctypes.c_int),
    "w4a16_check_device_errors": ([_vp, ctypes.POINTER(ctypes.c_uint32)], ctypes.c_int),
    "w4a16_set_wait_budget_ns": ([_c_i64], ctypes.c_int),
    "w4a16_set_prefill_kernel": ([ctypes.c_int], ctypes.c_int),
    "w4a16_prefill_choice": ([_c_i64, _c_i64, _c_i64, ctypes.POINTER(ctypes.c_int)], ctypes.c_int),
    "w4a16_prefill_plan": ([_c_i64, _c_i64, _c_i64, ctypes.c_int, ctypes.POINTER(ctypes.c_int),
                            ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)], ctypes.c_int),
    "w4a16_reset_scratch": ([_vp, _c_i64, _vp], ctypes.c_int),
    "w4a16_gemm_noalloc": ([_vp, _vp, _vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
                            _vp], ctypes.c_int),
    "w4a16_gemm_allreduce": ([_vp, _vp, _vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
                              _vp, _c_i64, _vp, ctypes.c_int, ctypes.c_int, _vp, _c_i64, _vp],
                             ctypes.c_int),
    "w4a16_gemm_allgather": ([_vp, _vp, _vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
                              _vp, _c_i64, _vp, ctypes.c_int, ctypes.c_int, _vp, _c_i64, _vp],
                             ctypes.c_int),
    "w4a16_p2p_buffer_bytes": ([ctypes.c_int, _c_i64, ctypes.POINTER(_c_i64)], ctypes.c_int),
    "w4a16_p2p_alloc": ([_c_i64, ctypes.POINTER(_vp), _vp], ctypes.c_int),
    "w4a16_p2p_open": ([_vp, ctypes.POINTER(_vp)], ctypes.c_int),
    "w4a16_p2p_close": ([_vp], ctypes.c_int),
    "w4a16_p2p_free": ([_vp], ctypes.c_int),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class W4A16Error(RuntimeError):
    """A non-zero status returned by the C ABI."""

    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what} failed: {strerror(status)} (status {status})")


def lib() -> ctypes.CDLL:
    """Load (once) and return the C-ABI library; raise loudly if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"W4A16 sm_100a library not built: {LIB_PATH} is missing. Build it with "
                    "`python w4a16-dequant-fused-matmul-kernel_b200/build.py` (there is no CPU "
                    "or PyTorch fallback for the W4A16 kernels).")
            handle = ctypes.CDLL(LIB_PATH)
            for name, (argtypes, restype) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.argtypes = argtypes
                fn.restype = restype
            _lib = handle
    return _lib


def strerror(status: int) -> str:
    return lib().w4a16_strerror(int(status)).decode()


def check(status: int, what: str) -> None:
    if status != W4A16_OK:
        raise W4A16Error(status, what)


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_of(device: torch.device) -> int:
    """Raw cudaStream_t of torch's current stream on ``device``."""
    if _raw_stream is not None:
        return _raw_stream(device.index)
    return torch.cuda.current_stream(device).cuda_stream


def stream_of_index(index: int) -> int:
    """Raw cudaStream_t of torch's current stream on CUDA device ``index``."""
    if _raw_stream is not None:
        return _raw_stream(index)
    return torch.cuda.current_stream(index).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def check_device_errors(device: torch.device | int | None = None) -> int:
    """Read and clear the device's sticky kernel error flags (synchronises).

    Raises :class:`W4A16Error` if a GEMM kernel's bounded wait expired since
    the last check; returns 0 otherwise.
    """
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(
        "cuda", device) if isinstance(device, int) else device
    flags = ctypes.c_uint32(0)
    with torch.cuda.device(dev):
        st = lib().w4a16_check_device_errors(stream_of(dev), ctypes.byref(flags))
    check(st, "w4a16_check_device_errors")
    return int(flags.value)


# ---------------------------------------------------------------------------
# GEMM workspace: one zeroed buffer per (device, stream), grown on demand. The
# decode kernel leaves it zero after every launch, so the buffer is
# reused without clearing. Superseded buffers are kept alive because a CUDA
# graph captured earlier may still refer to them.
# ---------------------------------------------------------------------------
_ws_lock = threading.Lock()
_ws_cache: dict[tuple[int, int], torch.Tensor] = {}
_ws_retired: list[torch.Tensor] = []


_ws_size_cache: dict[tuple[int, int, int, int, int], int] = {}


def gemm_workspace_bytes(M: int, N: int, K: int, G: int, device: torch.device) -> int:
    """Workspace bytes for this shape on ``device`` (memoised: it depends only on
    the shape and the device's SM count)."""
    key = (M, N, K, G, device.index)
    n = _ws_size_cache.get(key)
    if n is None:
        out = ctypes.c_int64(0)
        with torch.cuda.device(device):
            st = lib().w4a16_gemm_workspace_size(M, N, K, G, ctypes.byref(out))
        check(st, "w4a16_gemm_workspace_size")
        n = _ws_size_cache[key] = int(out.value)
    return n


def gemm_workspace(nbytes: int, device: torch.device, stream: int) -> torch.Tensor | None:
    """A zeroed, 256-byte-aligned scratch buffer of >= nbytes for this stream."""
    if nbytes <= 0:
        return None
    key = (device.index, stream)
    with _ws_lock:
        ws = _ws_cache.get(key)
        if ws is None or ws.numel() < nbytes:
            if ws is not None:
                _ws_retired.append(ws)
            size = max(nbytes, 1 << 20)
            ws = torch.zeros(size, dtype=torch.uint8, device=device)
            _ws_cache[key] = ws
        return ws


_ws_for: dict[tuple[int, int, int, int, int, int], tuple[int | None, int]] = {}


def workspace_for(M: int, N: int, K: int, G: int, device_index: int, stream: int) -> tuple[int | None, int]:
    """(pointer, bytes) of the zeroed workspace a GEMM of this shape uses on ``stream``
    of device ``device_index``; (None, 0) when the shape needs none. Memoised: a hit
    is one dictionary lookup (the buffer it names is kept alive by the cache below)."""
    key = (M, N, K, G, device_index, stream)
    hit = _ws_for.get(key)
    if hit is not None:
        return hit
    dev = torch.device("cuda", device_index)
    nbytes = gemm_workspace_bytes(M, N, K, G, dev) if M > 0 and N > 0 else 0
    ws = gemm_workspace(nbytes, dev, stream)
    val = (None, 0) if ws is None else (ws.data_ptr(), ws.numel())
    with _ws_lock:
        # a later, larger request can replace the stream's buffer: drop memoised entries
        # that name a retired buffer
        live = {t.data_ptr() for t in _ws_cache.values()}
        for k in [k for k, v in _ws_for.items() if v[0] is not None and v[0] not in live]:
            del _ws_for[k]
        _ws_for[key] = val
    return val


def reset_workspaces() -> None:
    """Zero every cached workspace and each device's allocation-free scratch array
    (after a kernel reported W4A16_ERR_TIMEOUT), on the stream each workspace serves;
    then synchronise those devices."""
    with _ws_lock:
        items = list(_ws_cache.items())
    devices = set()
    for (dev_index, stream), ws in items:
        with torch.cuda.device(dev_index):
            check(lib().w4a16_reset_scratch(ws.data_ptr(), ws.numel(), stream), "w4a16_reset_scratch")
        devices.add(dev_index)
    for dev_index in devices:
        torch.cuda.synchronize(dev_index)


def set_wait_budget_ns(ns: int) -> None:
    """Time budget of every bounded wait in kernels launched from now on (0: the
    default 4 s). Launches already queued or captured keep their budget."""
    check(lib().w4a16_set_wait_budget_ns(int(ns)), "w4a16_set_wait_budget_ns")


def set_prefill_kernel(which: int) -> None:
    """Prefill (M > 32) kernel for launches from now on: PREFILL_AUTO (per-shape
    choice), PREFILL_SMEM_B (dequantised weights as the shared-memory MMA operand) or
    PREFILL_TMEM_A (dequantised weights in tensor memory). For tests and tuning."""
    check(lib().w4a16_set_prefill_kernel(int(which)), "w4a16_set_prefill_kernel")


def prefill_choice(M: int, N: int, K: int) -> int:
    """The prefill kernel the current selection gives an M x N x K GEMM on the current
    device (PREFILL_SMEM_B or PREFILL_TMEM_A; PREFILL_AUTO when M <= 32)."""
    which = ctypes.c_int(0)
    check(lib().w4a16_prefill_choice(int(M), int(N), int(K), ctypes.byref(which)), "w4a16_prefill_choice")
    return which.value


def prefill_plan(M: int, N: int, K: int, num_sms: int) -> tuple[int, int, int]:
    """(kernel, tokens per tile, K splits) the cost model picks for an M x N x K GEMM on a
    GPU with ``num_sms`` SMs under the current selection, computed on the host (no device
    needed): as :func:`prefill_choice` for the kernel; tokens per tile and splits describe
    the tensor-memory-operand kernel (0 and 1 for the other kernel and for M <= 32)."""
    which, mt, sp = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0)
    check(lib().w4a16_prefill_plan(int(M), int(N), int(K), int(num_sms), ctypes.byref(which), ctypes.byref(mt),
                                   ctypes.byref(sp)), "w4a16_prefill_plan")
    return which.value, mt.value, sp.value
