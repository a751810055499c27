"""``W4A16Linear`` -- drop-in for the reference module (w4a16-kernel/src/w4a16/linear.py:19-98).

Same constructor, buffers (names, dtypes, shapes: state_dicts interchange
with the reference), ``from_linear`` / ``quantize_from_dense`` / ``forward`` /
``extra_repr``. Differences, all internal:

* ``forward`` calls the sm_100a fused GEMM and fuses the bias add into its
  epilogue (rounding as the reference's separate ``y + bias``: the fp16 GEMM
  result plus the fp16 bias, rounded to fp16);
* quantisation runs in the bit-exact CUDA quantiser.
"""
from __future__ import annotations

import torch
from torch import Tensor, nn

from .gemm import repack_qweight, w4a16_matmul
from .quant import quantize_weight

__all__ = ["W4A16Linear"]


class W4A16Linear(nn.Module):
    """``y = x @ W + b`` where W is held as group-wise uint4 codes and x, y are fp16.

    The module stores the quantised weight exactly as ``quantize_weight`` returns
    it, so a state_dict moves between this package and the reference unchanged:
    ``qweight`` (int32, ``in_features/8`` rows of ``out_features`` packed words),
    ``scales`` and ``zeros`` (fp16, one row per group of ``group_size`` input
    features) and, when the layer has one, ``bias`` (fp16, ``out_features``).
    Inputs of any leading shape are flattened to rows for the GEMM and the
    result is reshaped back.
    """

    def __init__(
        self,
        in_features: int,
        out_features: int,
        group_size: int = 128,
        bias: bool = True,
        device: torch.device | str | None = None,
    ) -> None:
        super().__init__()
        if in_features % 8 != 0:
            raise ValueError(f"in_features={in_features} must be divisible by 8")
        if in_features % group_size != 0:
            raise ValueError(f"in_features={in_features} must be divisible by group_size={group_size}")
        self.in_features = in_features
        self.out_features = out_features
        self.group_size = group_size

        K, N = in_features, out_features
        self.register_buffer("qweight", torch.zeros((K // 8, N), dtype=torch.int32, device=device))
        self.register_buffer("scales", torch.zeros((K // group_size, N), dtype=torch.float16, device=device))
        self.register_buffer("zeros", torch.zeros((K // group_size, N), dtype=torch.float16, device=device))
        if bias:
            self.register_buffer("bias", torch.zeros(N, dtype=torch.float16, device=device))
        else:
            self.bias = None
        # False: ``qweight`` holds the reference nibble order; True after repack_()
        self.kernel_order = False

    def repack_(self) -> "W4A16Linear":
        """Keep ``qweight`` in the kernel nibble order from now on (an extension of
        the reference module): the GEMM extracts each word's row pairs with one shift
        and four masks. ``state_dict()`` still returns the reference order and
        ``load_state_dict()`` still takes it; the conversion happens at those two points.
        Needs a CUDA module whose columns allow the TMA kernels (out_features % 8 == 0)."""
        if not self.kernel_order:
            assert self.qweight.is_cuda and self.out_features % 8 == 0, (
                "the kernel nibble order needs a CUDA module with out_features % 8 == 0")
            repack_qweight(self.qweight, True, out=self.qweight)
            self.kernel_order = True
        return self

    def _save_to_state_dict(self, destination, prefix, keep_vars):
        super()._save_to_state_dict(destination, prefix, keep_vars)
        if self.kernel_order:
            destination[prefix + "qweight"] = repack_qweight(self.qweight.detach(), False)

    def _load_from_state_dict(self, state_dict, prefix, *args, **kwargs):
        super()._load_from_state_dict(state_dict, prefix, *args, **kwargs)
        if self.kernel_order and (prefix + "qweight") in state_dict:
            repack_qweight(self.qweight, True, out=self.qweight)

    @classmethod
    def from_linear(cls, linear: nn.Linear, group_size: int = 128) -> "W4A16Linear":
        """A new layer holding ``linear``'s weight quantised with this group size (torch
        keeps ``nn.Linear.weight`` as ``[out, in]``; it is transposed to the ``[in, out]``
        layout the GEMM reads) and its bias in fp16."""
        N, K = linear.weight.shape
        mod = cls(
            in_features=K,
            out_features=N,
            group_size=group_size,
            bias=linear.bias is not None,
            device=linear.weight.device,
        )
        W = linear.weight.detach().t().contiguous()  # [N, K] -> [K, N]
        mod.quantize_from_dense(W)
        if linear.bias is not None:
            mod.bias.copy_(linear.bias.detach().to(torch.float16))
        return mod

    def quantize_from_dense(self, W: Tensor) -> None:
        """Replace the stored weight by ``W`` (``[in_features, out_features]``, any float
        dtype) quantised on the GPU with the bit-exact quantiser."""
        assert W.shape == (self.in_features, self.out_features), (
            f"expected weight [K,N]={(self.in_features, self.out_features)}, got {tuple(W.shape)}"
        )
        qweight, scales, zeros = quantize_weight(W, self.group_size)
        self.qweight.copy_(qweight.to(self.qweight.device))
        if self.kernel_order:
            repack_qweight(self.qweight, True, out=self.qweight)
        self.scales.copy_(scales.to(self.scales.device))
        self.zeros.copy_(zeros.to(self.zeros.device))

    def forward(self, x: Tensor) -> Tensor:
        assert x.dtype == torch.float16, f"x must be fp16, got {x.dtype}"
        assert x.shape[-1] == self.in_features, (
            f"x last dim {x.shape[-1]} != in_features {self.in_features}"
        )
        orig_shape = x.shape
        x2d = x.reshape(-1, self.in_features).contiguous()
        y = w4a16_matmul(x2d, self.qweight, self.scales, self.zeros, self.group_size, bias=self.bias,
                         kernel_order=self.kernel_order)
        return y.reshape(*orig_shape[:-1], self.out_features)

    def extra_repr(self) -> str:
        return (
            f"in_features={self.in_features}, out_features={self.out_features}, "
            f"group_size={self.group_size}, bias={self.bias is not None}"
        )
