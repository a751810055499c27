"""Quantise / pack / unpack / dequantise kernels vs the oracle: bit-exact.

Ports of the reference's test_quant.py (run on the GPU kernels) plus golden
vectors from the reference and the benchmark configurations' weight shapes.
"""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

import oracle
import synth
from helpers import bits16, np_
from tolerance import assert_gemm_close
from w4a16 import dequantize_weight, pack_int4, quantize_weight, unpack_int4, w4a16_matmul

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def golden():
    return np.load(os.path.join(GOLDEN, "golden_small.npz"))


def _cases(g):
    return sorted({k.split("/")[0] for k in g.files if not k.startswith("pack_")})


def _assert_quant_equal(got, want, what):
    qw, s, z = got
    wq, ws, wz = want
    assert np.array_equal(np_(qw), wq), f"{what}: qweight differs"
    assert np.array_equal(bits16(s), bits16(ws)), f"{what}: scales differ"
    assert np.array_equal(bits16(z), bits16(wz)), f"{what}: zeros differ"


def test_golden_quantise_bit_exact(golden):
    for name in _cases(golden):
        G = int(golden[f"{name}/meta"][3])
        W = torch.from_numpy(golden[f"{name}/W"]).cuda()
        got = quantize_weight(W, G)
        assert got[0].is_cuda
        _assert_quant_equal(got, (golden[f"{name}/qweight"], golden[f"{name}/scales"],
                                  golden[f"{name}/zeros"]), name)


def test_golden_quantise_from_cpu_tensor(golden):
    """CPU input: computed on the GPU, returned on the CPU (like the reference's device rule)."""
    name = "g64_n72"
    got = quantize_weight(torch.from_numpy(golden[f"{name}/W"]), 64)
    assert not got[0].is_cuda
    _assert_quant_equal(got, (golden[f"{name}/qweight"], golden[f"{name}/scales"],
                              golden[f"{name}/zeros"]), name)


def test_golden_dequantise_and_pack(golden):
    for name in _cases(golden):
        G = int(golden[f"{name}/meta"][3])
        qw = torch.from_numpy(golden[f"{name}/qweight"]).cuda()
        s = torch.from_numpy(golden[f"{name}/scales"]).cuda()
        z = torch.from_numpy(golden[f"{name}/zeros"]).cuda()
        w = dequantize_weight(qw, s, z, G)
        assert np.array_equal(bits16(w), bits16(golden[f"{name}/w_dq"])), name
    for key in [k for k in golden.files if k.startswith("pack_") and k.endswith("/q")]:
        base = key[:-2]
        p = pack_int4(torch.from_numpy(golden[key]).cuda())
        assert np.array_equal(np_(p), golden[base + "/packed"]), base
        assert np.array_equal(np_(unpack_int4(p)), golden[key]), base


def test_spec_examples_on_gpu():
    """W4A16_SPEC.md:84-105 (G=4: a word straddles groups) and :146-171."""
    W = torch.tensor([0.1, -0.3, 0.5, -0.1, 0.1, -0.3, 0.5, -0.1], dtype=torch.float16).view(8, 1).cuda()
    qw, s, z = quantize_weight(W, 4)
    assert unpack_int4(qw)[:4, 0].tolist() == [8, 0, 15, 4]
    assert float(z[0, 0]) == 6.0 and float(s[0, 0]) == 0.0533447265625
    q = torch.tensor([8, 0, 15, 4, 1, 7, 2, 12], dtype=torch.int32).view(8, 1).cuda()
    assert int(pack_int4(q)[0, 0]) & 0xFFFFFFFF == 0xC2714F08


@pytest.mark.parametrize("K", [8, 64, 128, 4096])
@pytest.mark.parametrize("N", [1, 16, 4096])
def test_pack_unpack_roundtrip(K, N):
    """test_quant.py:21-31 on the GPU kernels."""
    x = torch.randint(0, 16, (K, N), dtype=torch.int32, device="cuda")
    packed = pack_int4(x)
    assert packed.shape == (K // 8, N) and packed.dtype == torch.int32
    assert torch.equal(unpack_int4(packed, K), x)
    assert np.array_equal(np_(packed), oracle.pack_int4(np_(x)))


def test_pack_extremes_and_nibble_position():
    for val in (0, 15):
        x = torch.full((16, 8), val, dtype=torch.int32, device="cuda")
        assert torch.equal(unpack_int4(pack_int4(x)), x)
    x = torch.zeros((8, 1), dtype=torch.int32, device="cuda")
    x[3, 0] = 0xA
    assert int(pack_int4(x)[0, 0]) == (0xA << 12)
    with pytest.raises(AssertionError):
        pack_int4(torch.full((8, 2), 16, dtype=torch.int32, device="cuda"))


@pytest.mark.parametrize("group_size", [64, 128])
def test_quant_dequant_roundtrip_error(group_size):
    """test_quant.py:71-90."""
    torch.manual_seed(1)
    W = torch.randn(4096, 1024, dtype=torch.float16, device="cuda")
    qw, s, z = quantize_weight(W, group_size)
    Wdq = dequantize_weight(qw, s, z, group_size)
    rel = ((Wdq.float() - W.float()).abs().mean() / W.float().abs().mean()).item()
    assert rel < 0.15
    assert torch.all(z >= 0) and torch.all(z <= 15) and torch.all(z == torch.round(z.float()))


def test_constant_group_and_nonfinite():
    W = torch.zeros((128, 8), dtype=torch.float16, device="cuda")
    W[:, 0] = 3.0
    qw, s, z = quantize_weight(W, 64)
    assert torch.allclose(dequantize_weight(qw, s, z, 64).float(), W.float(), atol=1e-3)
    W[5, 3] = float("nan")
    with pytest.raises(AssertionError):
        quantize_weight(W, 64)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_other_input_dtypes_match_oracle(dtype):
    W = (torch.randn(256, 40, device="cuda") * 0.05).to(dtype)
    got = quantize_weight(W, 64)
    want = oracle.quantize_weight(np_(W.float()), 64)
    _assert_quant_equal(got, want, str(dtype))


def test_oracle_configuration_digest():
    """The 16x4096x4096 oracle configuration, quantised on the GPU, hashes to
    the reference's own output."""
    import hashlib
    ref = np.load(os.path.join(GOLDEN, "golden_oracle_cfg.npz"))
    _, W = synth.oracle_cfg_inputs()
    qw, s, z = quantize_weight(torch.from_numpy(W).cuda(), 128)
    sha = lambda t: hashlib.sha256(np.ascontiguousarray(np_(t)).tobytes()).hexdigest()  # noqa: E731
    assert sha(qw) == str(ref["qweight_sha256"])
    assert sha(s) == str(ref["scales_sha256"])
    assert sha(z) == str(ref["zeros_sha256"])
    assert sha(dequantize_weight(qw, s, z, 128)) == str(ref["w_dq_sha256"])


@pytest.mark.parametrize("K,N,sigma,outliers,full", [
    (4096, 11008, 0.02, 0.0, True),      # decode configuration
    (4096, 14336, 0.02, 0.0, True),      # prefill configuration
    (8192, 28672, 0.015, 0.001, False),  # batched-decode sweep (outliers)
    (28672, 8192, 0.02, 0.0, False),     # MLP down projection
])
def test_benchmark_weight_shapes_bit_exact(K, N, sigma, outliers, full):
    """Full-size weights of the benchmark configurations. Quantisation is
    column-independent, so the largest two are checked on a spread of column
    slices (first, middle, last); the others in full."""
    gen = torch.Generator(device="cuda").manual_seed(K + N)
    W = torch.randn(K, N, generator=gen, device="cuda") * sigma
    if outliers:
        mask = torch.rand(K, N, generator=gen, device="cuda") < outliers
        W = torch.where(mask, torch.randn(K, N, generator=gen, device="cuda") * 0.2, W)
    W = W.half()
    qw, s, z = quantize_weight(W, 128)
    cols = [slice(0, N)] if full else [slice(0, 96), slice(N // 2 - 40, N // 2 + 56), slice(N - 96, N)]
    for c in cols:
        want = oracle.quantize_weight(np_(W[:, c]), 128)
        _assert_quant_equal((qw[:, c], s[:, c], z[:, c]), want, f"{K}x{N}[{c}]")
    # size-independent properties over the whole matrix
    assert torch.all((z >= 0) & (z <= 15))
    # |W - dequant(W)| <= one quantisation step (half a step from rounding, up
    # to half more where the rounded zero-point makes an extreme clamp), plus
    # the fp16 rounding of the scale and of the dequantised value.
    Wdq = dequantize_weight(qw, s, z, 128).float()
    step = s.float().repeat_interleave(128, 0)
    assert torch.all((Wdq - W.float()).abs() <= 1.05 * step + 1e-6)


# ----------------------------------------------------------------------------- symmetric codes
def _np_quantize_symmetric(W: np.ndarray, G: int):
    """Symmetric group quantisation restated in numpy (fp32, IEEE division, half-even):
    zero = 8, scale = 2 * max|w| / 15 (1 when not > 0), q = clamp(rint(w / scale) + 8, 0, 15)."""
    K, N = W.shape
    Wf = W.astype(np.float32).reshape(K // G, G, N)
    amax = np.max(np.abs(Wf), axis=1)
    scale = (np.float32(2.0) * amax) / np.float32(15.0)
    scale = np.where(scale > 0, scale, np.float32(1.0)).astype(np.float32)
    q = np.clip(np.rint(Wf / scale[:, None, :]) + np.float32(8.0), 0, 15).astype(np.int32).reshape(K, N)
    return oracle.pack_int4(q), scale.astype(np.float16), np.full((K // G, N), 8.0, dtype=np.float16)


@pytest.mark.parametrize("K,N,G", [(256, 264, 64), (1024, 512, 128), (384, 96, 192)])
def test_symmetric_quantisation_and_gemm(K, N, G):
    W = (torch.randn(K, N, generator=torch.Generator().manual_seed(K + N)) * 0.05).half()
    W[:, 0] = 0.0
    W[:G, 1] = torch.abs(W[:G, 1])   # an all-positive group
    qw, s, z = quantize_weight(W.cuda(), G, symmetric=True)
    eq, es, ez = _np_quantize_symmetric(W.numpy(), G)
    assert np.array_equal(np_(qw), eq)
    assert np.array_equal(bits16(s), bits16(es)) and np.array_equal(bits16(z), bits16(ez))
    X = torch.randn(5, K, device="cuda").half()
    y = w4a16_matmul(X, qw, s, z, G)
    assert_gemm_close(np_(y), oracle.reference_w4a16(np_(X), np_(qw), np_(s), np_(z), G), "symmetric GEMM")
