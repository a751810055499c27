"""Peer-to-peer channel for tensor-parallel decode GEMMs fused with their collective.

``PeerAllReduce`` owns, on every rank of a process group, one CUDA IPC buffer
mapped on every other rank (plain peer memory over NVLink / NVSwitch; no
multicast object), the list of those mappings and two device control words.
``gemm`` runs ``w4a16_gemm_allreduce`` (row-parallel: one kernel per rank
computes its partial GEMM and writes each finished fp32 element, tagged with the
call's epoch, into every rank's buffer; its last CTAs wait for every rank's
tagged elements of their share and sum them in rank order -- the same result as
an fp32 all-reduce followed by one fp16 rounding). ``gemm_allgather`` runs
``w4a16_gemm_allgather`` (column-parallel: the finished fp16 elements are
exchanged the same way and placed, so every rank receives the whole output --
the same bits as the GEMM followed by an all-gather).

Creating a channel is collective (every rank of the group, same order, same
arguments); so is every call. Calls on one channel must be issued on one
stream at a time. ``close()`` is collective as well.

Failure handling: a call whose C entry point refuses it, or a ``check()`` that
finds a kernel's bounded wait expired (a peer that never wrote its words), marks
the channel broken -- its epochs may be out of step with the peers' -- and every
later call raises until the ranks run the collective ``reset()``.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib

__all__ = ["PeerAllReduce", "MAX_RANKS"]

MAX_RANKS = 8
MAX_TOKENS = 32


class PeerAllReduce:
    """Peer buffers for fused GEMM + all-reduce of outputs up to ``max_tokens x n``."""

    def __init__(self, n: int, group=None, max_tokens: int = MAX_TOKENS,
                 device: torch.device | None = None) -> None:
        if not (dist.is_available() and dist.is_initialized()):
            raise RuntimeError("PeerAllReduce needs an initialised process group")
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if not 2 <= self.world <= MAX_RANKS:
            raise ValueError(f"PeerAllReduce supports 2..{MAX_RANKS} ranks, got {self.world}")
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.n = n
        self.max_tokens = max_tokens
        self.slot = (max_tokens * n + 1) // 2 * 2   # even: the kernel reads word pairs
        lib = _lib.lib()
        nbytes = ctypes.c_int64(0)
        _lib.check(lib.w4a16_p2p_buffer_bytes(self.world, self.slot, ctypes.byref(nbytes)),
                   "w4a16_p2p_buffer_bytes")
        own = ctypes.c_void_p(0)
        handle = (ctypes.c_ubyte * 64)()
        with torch.cuda.device(self.device):
            _lib.check(lib.w4a16_p2p_alloc(nbytes.value, ctypes.byref(own), handle), "w4a16_p2p_alloc")
        self._own = own.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        ptrs, self._opened = [], []
        with torch.cuda.device(self.device):
            for q, h in enumerate(handles):
                if q == self.rank:
                    ptrs.append(self._own)
                    continue
                hb = (ctypes.c_ubyte * 64).from_buffer_copy(h)
                p = ctypes.c_void_p(0)
                _lib.check(lib.w4a16_p2p_open(hb, ctypes.byref(p)), "w4a16_p2p_open")
                ptrs.append(p.value)
                self._opened.append(p.value)
        self.peers = (ctypes.c_ulonglong * self.world)(*ptrs)   # host array, copied into each launch
        self.ctl = torch.zeros(4, dtype=torch.int32, device=self.device)
        self._nbytes = nbytes.value
        self.broken: str | None = None
        torch.cuda.synchronize(self.device)
        dist.barrier(group=group)   # every buffer is mapped and zero before the first call

    def _usable(self) -> None:
        if self.broken is not None:
            raise RuntimeError(f"peer channel is broken ({self.broken}); every rank must call reset()")

    def _launched(self, st: int, what: str) -> None:
        if st != _lib.W4A16_OK:
            self.broken = f"{what} returned status {st}"
            _lib.check(st, what)

    def check(self) -> None:
        """Synchronise this device and raise ``W4A16Error`` if any kernel's bounded
        wait expired since the last check (the channel is then marked broken)."""
        try:
            _lib.check_device_errors(self.device)
        except _lib.W4A16Error:
            self.broken = "a bounded wait expired"
            raise

    def reset(self) -> None:
        """Collective: zero this rank's control words and buffer after a failure,
        so every rank starts again from epoch 0."""
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)   # no rank still writes into a buffer
        with torch.cuda.device(self.device):
            self.ctl.zero_()
            # the peer buffer is raw memory from w4a16_p2p_alloc: zeroed like a workspace
            _lib.check(_lib.lib().w4a16_reset_scratch(self._own, self._nbytes, _lib.stream_of(self.device)),
                       "w4a16_reset_scratch")
        torch.cuda.synchronize(self.device)
        _lib.reset_workspaces()
        dist.barrier(group=self.group)   # every buffer is zero before the next call
        self.broken = None

    def gemm(self, x: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor,
             group_size: int, bias: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
        """fp16 ``sum over ranks of x_r @ dequant(W_r)`` [+ bias] for this rank's K-slice."""
        self._usable()
        M, K = x.shape
        N = qweight.shape[1]
        assert M <= self.max_tokens and N == self.n, "shape outside this channel"
        assert x.is_contiguous() and x.dtype == torch.float16 and x.device == self.device
        y = out if out is not None else torch.empty((M, N), device=x.device, dtype=torch.float16)
        assert y.is_contiguous() and y.shape == (M, N) and y.dtype == torch.float16 and y.device == x.device
        dev = x.device
        stream = _lib.stream_of(dev)
        nb = _lib.gemm_workspace_bytes(M, N, K, group_size, dev)
        ws = _lib.gemm_workspace(nb, dev, stream)
        st = _lib.lib().w4a16_gemm_allreduce(
            x.data_ptr(), qweight.data_ptr(), scales.data_ptr(), zeros.data_ptr(), _lib.ptr(bias),
            y.data_ptr(), M, N, K, group_size, N, _lib.ptr(ws), 0 if ws is None else ws.numel(),
            self.peers, self.world, self.rank, self.ctl.data_ptr(), self.slot, stream)
        self._launched(st, "w4a16_gemm_allreduce")
        return y

    def gemm_allgather(self, x: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor,
                       zeros: torch.Tensor, group_size: int, bias: torch.Tensor | None = None,
                       out: torch.Tensor | None = None) -> torch.Tensor:
        """fp16 ``[x @ dequant(W_0) | ... | x @ dequant(W_{p-1})]`` (each shard's bias
        added) for this rank's column shard ``W_r``: the whole output on every rank."""
        self._usable()
        M, K = x.shape
        N = qweight.shape[1]
        assert M <= self.max_tokens and N == self.n, "shape outside this channel"
        assert x.is_contiguous() and x.dtype == torch.float16 and x.device == self.device
        y = out if out is not None else torch.empty((M, self.world * N), device=x.device, dtype=torch.float16)
        assert y.is_contiguous() and y.shape == (M, self.world * N) and y.dtype == torch.float16
        assert y.device == x.device
        dev = x.device
        stream = _lib.stream_of(dev)
        nb = _lib.gemm_workspace_bytes(M, N, K, group_size, dev)
        ws = _lib.gemm_workspace(nb, dev, stream)
        st = _lib.lib().w4a16_gemm_allgather(
            x.data_ptr(), qweight.data_ptr(), scales.data_ptr(), zeros.data_ptr(), _lib.ptr(bias),
            y.data_ptr(), M, N, K, group_size, self.world * N, _lib.ptr(ws), 0 if ws is None else ws.numel(),
            self.peers, self.world, self.rank, self.ctl.data_ptr(), self.slot, stream)
        self._launched(st, "w4a16_gemm_allgather")
        return y

    def close(self) -> None:
        """Collective: unmap the peers' buffers and free this rank's."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)   # no rank still writes into a buffer
        lib = _lib.lib()
        with torch.cuda.device(self.device):
            for p in self._opened:
                lib.w4a16_p2p_close(ctypes.c_void_p(p))
            dist.barrier(group=self.group)   # every mapping of this rank's buffer is gone
            lib.w4a16_p2p_free(ctypes.c_void_p(self._own))
        self._opened, self._own = [], None
