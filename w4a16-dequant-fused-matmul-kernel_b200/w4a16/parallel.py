"""Tensor-parallel W4A16 layers: one process per GPU, torch.distributed (NCCL
over NVLink / NVSwitch) for the exchanges.

The reference has no multi-GPU path; these layers add the two sharding
schemes the benchmark configurations name:

* column-parallel (``ColumnParallelW4A16Linear``): rank r owns the column
  slice ``[r*N/p, (r+1)*N/p)`` of qweight / scales / zeros (all N-minor, so
  each shard is a contiguous copy of whole rows). x is replicated; every rank
  computes its slice of y with no communication. Only a caller that needs the
  full y pays an all-gather (``gather=True``): up to 32 tokens the GEMM and the
  all-gather run as one kernel per rank over NVLink peer memory, larger inputs
  use NCCL's all-gather.
* row-parallel (``RowParallelW4A16Linear``): rank r owns the K rows
  ``[r*K/p, (r+1)*K/p)`` (K/p must stay a multiple of the group size) and a
  K-slice of x. Each rank computes unrounded fp32 partial sums, they are
  all-reduced (sum) in fp32 and rounded to fp16 once, so the sharded layer
  matches the unsharded one within the parity tolerance. Up to 32 tokens the
  GEMM and the all-reduce run as one kernel per rank over NVLink peer memory
  (``w4a16.p2p.PeerAllReduce``); larger inputs use NCCL.
* ``W4A16MLP``: the decoder MLP block -- gate and up projections fused into
  one column-parallel GEMM (the shards' columns interleaved in blocks of 16)
  whose epilogue applies SwiGLU, then the row-parallel down projection and its
  all-reduce.

Without an initialised process group (or with one rank) the layers run
unsharded and communicate nothing.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
from torch import Tensor, nn

from .gemm import interleave_gate_up, repack_qweight, w4a16_matmul, w4a16_matmul_f32, w4a16_matmul_swiglu
from .quant import quantize_weight

__all__ = [
    "close_peer_channels",
    "shard_columns",
    "shard_rows",
    "gather_columns",
    "all_reduce_sum",
    "ColumnParallelW4A16Linear",
    "RowParallelW4A16Linear",
    "W4A16MLP",
]


_peer_channels: dict = {}


def _peer_channel(group, device: torch.device, n: int):
    """The fused GEMM + all-reduce / all-gather channel for (group, device, n) (n: the
    columns one rank's GEMM computes); created on first use (collectively: every rank's
    first eligible forward reaches here in the same order)."""
    from .p2p import PeerAllReduce
    key = (id(group), device.index, n)
    ch = _peer_channels.get(key)
    if ch is None:
        ch = _peer_channels[key] = PeerAllReduce(n, group=group, device=device)
    return ch


def close_peer_channels() -> None:
    """Collective: release every peer channel (call before destroying the process group)."""
    for key in sorted(_peer_channels, key=lambda k: (k[1], k[2])):
        _peer_channels[key].close()
    _peer_channels.clear()


def _fused_route(world: int, enabled: bool, x: Tensor, n: int) -> bool:
    """Whether a call takes the fused GEMM + collective kernel. The decision uses only
    facts every rank shares (world size, the layer's switch, the token count and the
    column count), so all ranks of a collective call choose the same route; facts that
    could differ between ranks (contiguity, alignment) are fixed up by ``_aligned``
    instead of changing the route."""
    from .p2p import MAX_TOKENS
    return (world > 1 and enabled and x.is_cuda and x.dim() == 2 and x.dtype == torch.float16
            and x.shape[0] <= MAX_TOKENS and n % 8 == 0)


def _aligned(x: Tensor) -> Tensor:
    """``x`` contiguous with a 16-byte-aligned base (a fresh copy when it is not)."""
    if x.is_contiguous() and x.data_ptr() % 16 == 0:
        return x
    return x.clone(memory_format=torch.contiguous_format)


def _world(group=None) -> tuple[int, int]:
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(group), dist.get_world_size(group)
    return 0, 1


def shard_columns(qweight: Tensor, scales: Tensor, zeros: Tensor, rank: int, world: int,
                  bias: Tensor | None = None):
    """Rank ``rank``'s contiguous column shard of a quantised ``[K, N]`` weight."""
    N = qweight.shape[1]
    assert N % world == 0, f"N={N} must divide evenly over {world} ranks"
    n = N // world
    sl = slice(rank * n, (rank + 1) * n)
    out = (qweight[:, sl].contiguous(), scales[:, sl].contiguous(), zeros[:, sl].contiguous())
    return out + ((bias[sl].contiguous() if bias is not None else None),)


def shard_rows(qweight: Tensor, scales: Tensor, zeros: Tensor, group_size: int, rank: int,
               world: int):
    """Rank ``rank``'s K-row shard; K/world must be a multiple of 8 and of the group size."""
    K = qweight.shape[0] * 8
    assert K % world == 0, f"K={K} must divide evenly over {world} ranks"
    k = K // world
    assert k % 8 == 0 and k % group_size == 0, (
        f"each rank's K={k} must be a multiple of 8 and of group_size={group_size}")
    return (qweight[rank * k // 8:(rank + 1) * k // 8].contiguous(),
            scales[rank * k // group_size:(rank + 1) * k // group_size].contiguous(),
            zeros[rank * k // group_size:(rank + 1) * k // group_size].contiguous())


def gather_columns(y_local: Tensor, group=None) -> Tensor:
    """All-gather the column shards ``[M, N/p]`` of every rank into ``[M, N]``."""
    rank, world = _world(group)
    if world == 1:
        return y_local
    M, n = y_local.shape
    buf = torch.empty((world * M, n), dtype=y_local.dtype, device=y_local.device)
    dist.all_gather_into_tensor(buf, y_local.contiguous(), group=group)   # rank-major
    if M == 1:
        return buf.view(1, world * n)
    return buf.view(world, M, n).permute(1, 0, 2).reshape(M, world * n)


def all_reduce_sum(t: Tensor, group=None) -> Tensor:
    """In-place sum across ranks (no-op without a process group)."""
    rank, world = _world(group)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return t


class ColumnParallelW4A16Linear(nn.Module):
    """W4A16 linear layer whose output columns are split across ranks."""

    def __init__(self, in_features: int, out_features: int, group_size: int = 128,
                 bias: bool = True, device=None, group=None, fused_gather: bool = True) -> None:
        super().__init__()
        self.group = group
        self.rank, self.world = _world(group)
        self.fused_gather = fused_gather
        if in_features % 8 != 0 or in_features % group_size != 0:
            raise ValueError(f"in_features={in_features} must be divisible by 8 and group_size={group_size}")
        if out_features % self.world != 0:
            raise ValueError(f"out_features={out_features} must divide over {self.world} ranks")
        self.in_features, self.out_features, self.group_size = in_features, out_features, group_size
        n = out_features // self.world
        K = in_features
        self.register_buffer("qweight", torch.zeros((K // 8, n), dtype=torch.int32, device=device))
        self.register_buffer("scales", torch.zeros((K // group_size, n), dtype=torch.float16, device=device))
        self.register_buffer("zeros", torch.zeros((K // group_size, n), dtype=torch.float16, device=device))
        self.register_buffer("bias", torch.zeros(n, dtype=torch.float16, device=device) if bias else None)

    @classmethod
    def from_quantized(cls, qweight: Tensor, scales: Tensor, zeros: Tensor, group_size: int,
                       bias: Tensor | None = None, group=None) -> "ColumnParallelW4A16Linear":
        """Build this rank's shard from a full quantised weight (the same on every rank)."""
        K, N = qweight.shape[0] * 8, qweight.shape[1]
        mod = cls(K, N, group_size, bias is not None, device=qweight.device, group=group)
        q, s, z, b = shard_columns(qweight, scales, zeros, mod.rank, mod.world, bias)
        mod.qweight.copy_(q)
        mod.scales.copy_(s)
        mod.zeros.copy_(z)
        if b is not None:
            mod.bias.copy_(b)
        return mod

    def forward(self, x: Tensor, gather: bool = False) -> Tensor:
        n = self.out_features // self.world
        if gather and _fused_route(self.world, self.fused_gather, x, n):
            ch = _peer_channel(self.group, x.device, n)
            return ch.gemm_allgather(_aligned(x), self.qweight, self.scales, self.zeros, self.group_size,
                                     bias=self.bias)
        y = w4a16_matmul(x, self.qweight, self.scales, self.zeros, self.group_size, bias=self.bias)
        return gather_columns(y, self.group) if gather else y


class RowParallelW4A16Linear(nn.Module):
    """W4A16 linear layer whose K rows (and input features) are split across ranks."""

    def __init__(self, in_features: int, out_features: int, group_size: int = 128,
                 bias: bool = True, device=None, group=None, fused_allreduce: bool = True) -> None:
        super().__init__()
        self.group = group
        self.rank, self.world = _world(group)
        self.fused_allreduce = fused_allreduce
        if in_features % self.world != 0:
            raise ValueError(f"in_features={in_features} must divide over {self.world} ranks")
        k = in_features // self.world
        if k % 8 != 0 or k % group_size != 0:
            raise ValueError(f"per-rank in_features={k} must be divisible by 8 and group_size={group_size}")
        self.in_features, self.out_features, self.group_size = in_features, out_features, group_size
        N = out_features
        self.register_buffer("qweight", torch.zeros((k // 8, N), dtype=torch.int32, device=device))
        self.register_buffer("scales", torch.zeros((k // group_size, N), dtype=torch.float16, device=device))
        self.register_buffer("zeros", torch.zeros((k // group_size, N), dtype=torch.float16, device=device))
        self.register_buffer("bias", torch.zeros(N, dtype=torch.float16, device=device) if bias else None)

    @classmethod
    def from_quantized(cls, qweight: Tensor, scales: Tensor, zeros: Tensor, group_size: int,
                       bias: Tensor | None = None, group=None) -> "RowParallelW4A16Linear":
        K, N = qweight.shape[0] * 8, qweight.shape[1]
        mod = cls(K, N, group_size, bias is not None, device=qweight.device, group=group)
        q, s, z = shard_rows(qweight, scales, zeros, group_size, mod.rank, mod.world)
        mod.qweight.copy_(q)
        mod.scales.copy_(s)
        mod.zeros.copy_(z)
        if bias is not None:
            mod.bias.copy_(bias)
        return mod

    def forward(self, x_local: Tensor) -> Tensor:
        """``x_local`` is this rank's K-slice of the input, ``[M, K/p]``."""
        if _fused_route(self.world, self.fused_allreduce, x_local, self.out_features):
            ch = _peer_channel(self.group, x_local.device, self.out_features)
            return ch.gemm(_aligned(x_local), self.qweight, self.scales, self.zeros, self.group_size,
                           bias=self.bias)
        part = w4a16_matmul_f32(x_local, self.qweight, self.scales, self.zeros, self.group_size)
        y = all_reduce_sum(part, self.group).to(torch.float16)
        return y + self.bias if self.bias is not None else y


class _QuantizedWeight(nn.Module):
    """Buffers of one quantised ``[K, N]`` weight (no forward of its own)."""

    def __init__(self, K: int, N: int, group_size: int, device=None) -> None:
        super().__init__()
        self.register_buffer("qweight", torch.zeros((K // 8, N), dtype=torch.int32, device=device))
        self.register_buffer("scales", torch.zeros((K // group_size, N), dtype=torch.float16, device=device))
        self.register_buffer("zeros", torch.zeros((K // group_size, N), dtype=torch.float16, device=device))


class W4A16MLP(nn.Module):
    """Decoder MLP block ``down(silu(gate(x)) * up(x))`` with W4A16 weights,
    tensor-parallel over the process group: gate/up column-parallel, fused into
    one GEMM whose epilogue computes the SwiGLU (``gate_up`` holds this rank's
    gate and up shards interleaved in blocks of 16 columns), then down
    row-parallel with its all-reduce."""

    def __init__(self, hidden: int, intermediate: int, group_size: int = 128, device=None,
                 group=None) -> None:
        super().__init__()
        self.group = group
        self.rank, self.world = _world(group)
        if intermediate % self.world != 0:
            raise ValueError(f"intermediate={intermediate} must divide over {self.world} ranks")
        h = intermediate // self.world
        self.hidden, self.intermediate, self.group_size = hidden, intermediate, group_size
        # this rank's gate and up shards, columns interleaved in blocks of 16 and packed in
        # the kernel nibble order: one GEMM with N = 2h whose epilogue writes silu(gate) * up
        self.gate_up = _QuantizedWeight(hidden, 2 * h, group_size, device)
        self.gate_up_kernel_order = False
        self.down = RowParallelW4A16Linear(intermediate, hidden, group_size, bias=False,
                                           device=device, group=group)

    @classmethod
    def from_dense(cls, w_gate: Tensor, w_up: Tensor, w_down: Tensor, group_size: int = 128,
                   group=None) -> "W4A16MLP":
        """Quantise dense ``[hidden, intermediate]`` gate/up and ``[intermediate, hidden]``
        down weights (logical [K, N] layout) and keep this rank's shards."""
        hidden, inter = w_gate.shape
        mod = cls(hidden, inter, group_size, device=w_gate.device, group=group)
        gq, gs, gz = quantize_weight(w_gate, group_size)
        uq, us, uz = quantize_weight(w_up, group_size)
        dq, ds, dz = quantize_weight(w_down, group_size)
        return mod.load_quantized((gq, gs, gz), (uq, us, uz), (dq, ds, dz))

    def load_quantized(self, gate, up, down) -> "W4A16MLP":
        r, p = self.rank, self.world
        g = shard_columns(*gate, r, p)[:3]
        u = shard_columns(*up, r, p)[:3]
        for name, a, b in zip(("qweight", "scales", "zeros"), g, u):
            getattr(self.gate_up, name).copy_(interleave_gate_up(a, b))
        if self.gate_up.qweight.is_cuda:
            repack_qweight(self.gate_up.qweight, True, out=self.gate_up.qweight)
            self.gate_up_kernel_order = True
        d = shard_rows(*down, self.group_size, r, p)
        for name, t in zip(("qweight", "scales", "zeros"), d):
            getattr(self.down, name).copy_(t)
        return self

    def forward(self, x: Tensor) -> Tensor:
        h = w4a16_matmul_swiglu(x, self.gate_up.qweight, self.gate_up.scales, self.gate_up.zeros,
                                self.group_size, kernel_order=self.gate_up_kernel_order)
        return self.down(h)
