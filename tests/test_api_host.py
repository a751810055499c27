"""Host-side behaviour of the drop-in API that needs no GPU: the reference's
error conventions (w4a16-kernel/tests/test_quant.py:103-109,
test_correctness.py:49-70; quant.py:116-119; linear.py:38-41;
triton_kernel.py:153-182) and the module's buffers/state_dict layout."""
from __future__ import annotations

import pytest
import torch

import w4a16
from w4a16 import W4A16Linear, pack_int4, quantize_weight, w4a16_matmul


def test_public_api_matches_reference_names():
    for name in ["quantize_weight", "dequantize_weight", "pack_int4", "unpack_int4",
                 "reference_w4a16", "dequant_then_matmul", "fp16_matmul", "w4a16_matmul",
                 "W4A16Linear"]:
        assert hasattr(w4a16, name), name
    from w4a16.cuda_kernel import load_cuda_module, w4a16_matmul_cuda  # noqa: F401
    from w4a16.triton_kernel import w4a16_matmul as wm
    assert wm is w4a16_matmul


def test_quantize_divisibility_errors_are_value_errors():
    with pytest.raises(ValueError):
        quantize_weight(torch.randn(100, 16, dtype=torch.float16), group_size=64)
    with pytest.raises(ValueError):
        quantize_weight(torch.randn(96, 16, dtype=torch.float16), group_size=64)


def test_pack_requires_k_div_8():
    with pytest.raises(AssertionError):
        pack_int4(torch.zeros((7, 4), dtype=torch.int32))


def test_matmul_rejects_cpu_tensors():
    x = torch.zeros(2, 128, dtype=torch.float16)
    qw = torch.zeros(16, 64, dtype=torch.int32)
    s = torch.zeros(2, 64, dtype=torch.float16)
    with pytest.raises(AssertionError):
        w4a16_matmul(x, qw, s, s, 64)


def test_linear_ctor_errors():
    with pytest.raises(ValueError):
        W4A16Linear(100, 16)
    with pytest.raises(ValueError):
        W4A16Linear(192, 16, group_size=128)


def test_linear_buffers_and_state_dict_layout():
    """Same buffer names, dtypes and shapes as the reference (linear.py:47-53),
    so reference state_dicts load unchanged."""
    m = W4A16Linear(256, 48, group_size=64, bias=True)
    sd = m.state_dict()
    assert sd["qweight"].shape == (32, 48) and sd["qweight"].dtype == torch.int32
    assert sd["scales"].shape == (4, 48) and sd["scales"].dtype == torch.float16
    assert sd["zeros"].shape == (4, 48) and sd["zeros"].dtype == torch.float16
    assert sd["bias"].shape == (48,) and sd["bias"].dtype == torch.float16
    m2 = W4A16Linear(256, 48, group_size=64, bias=True)
    sd["qweight"].random_(0, 1 << 30)
    m2.load_state_dict(sd)
    assert torch.equal(m2.qweight, sd["qweight"])
    nb = W4A16Linear(256, 48, group_size=64, bias=False)
    assert nb.bias is None and "bias" not in nb.state_dict()
    assert "group_size=64" in repr(m)


def test_interleave_gate_up_layout():
    """Blocks of 16 columns alternate gate, up: output column j of the fused SwiGLU
    GEMM reads fused columns 32*(j//16) + j%16 (gate) and that + 16 (up)."""
    R, H = 3, 48
    g = torch.arange(R * H, dtype=torch.int32).reshape(R, H)
    u = -g - 1
    f = w4a16.interleave_gate_up(g, u)
    assert f.shape == (R, 2 * H) and f.is_contiguous()
    for j in range(H):
        cg = 32 * (j // 16) + j % 16
        assert torch.equal(f[:, cg], g[:, j]) and torch.equal(f[:, cg + 16], u[:, j])
    with pytest.raises(AssertionError):
        w4a16.interleave_gate_up(g[:, :40], u[:, :40])   # not a multiple of 16
