"""Pin the CPU oracle (oracle/w4a16_oracle.py) before trusting it.

Three sources of truth, none of them the oracle itself:

* the worked examples of the format spec (W4A16_SPEC.md:84-105 quantise,
  :146-171 packing);
* the known answers of the reference's own unit tests
  (w4a16-kernel/tests/test_quant.py);
* golden vectors produced by running the reference's ``quant.py`` and
  ``reference.py`` (tests/golden/make_golden.py), including the 16x4096x4096
  oracle configuration (as SHA-256 digests plus the full output).
"""
from __future__ import annotations

import hashlib
import os

import numpy as np
import pytest

import oracle
import synth
from tolerance import assert_gemm_close

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def golden():
    return np.load(os.path.join(GOLDEN, "golden_small.npz"))


def _cases(g):
    return sorted({k.split("/")[0] for k in g.files if not k.startswith("pack_")})


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint16 if a.dtype == np.float16 else a.dtype)


# ----------------------------- spec worked examples -----------------------------
def test_spec_quantise_example():
    """W4A16_SPEC.md:84-105: G=4, W=[0.1,-0.3,0.5,-0.1] -> q=[8,0,15,4], zero=6."""
    W = np.array([[0.1], [-0.3], [0.5], [-0.1], [0.1], [-0.3], [0.5], [-0.1]], dtype=np.float16)
    qw, s, z = oracle.quantize_weight(W, 4)
    q = oracle.unpack_int4(qw)
    assert q[:4, 0].tolist() == [8, 0, 15, 4]
    assert float(z[0, 0]) == 6.0
    assert float(s[0, 0]) == 0.0533447265625   # fp16(0.8/15)


def test_spec_packing_example():
    """W4A16_SPEC.md:146-171: q=[8,0,15,4,1,7,2,12] -> 0xC2714F08."""
    q = np.array([8, 0, 15, 4, 1, 7, 2, 12], dtype=np.int32).reshape(8, 1)
    packed = oracle.pack_int4(q)
    assert packed.view(np.uint32)[0, 0] == 0xC2714F08
    assert oracle.unpack_int4(packed)[:, 0].tolist() == [8, 0, 15, 4, 1, 7, 2, 12]


# ----------------------------- reference unit-test known answers -----------------
@pytest.mark.parametrize("K", [8, 64, 128, 4096])
@pytest.mark.parametrize("N", [1, 16, 4096])
def test_pack_unpack_roundtrip(K, N):
    """test_quant.py:21-31."""
    x = np.random.default_rng(K * 7 + N).integers(0, 16, size=(K, N), dtype=np.int32)
    packed = oracle.pack_int4(x)
    assert packed.shape == (K // 8, N) and packed.dtype == np.int32
    assert np.array_equal(oracle.unpack_int4(packed, K), x)


def test_pack_unpack_extremes():
    """test_quant.py:34-38: all-0 and all-15 (sign bit set) round-trip."""
    for val in (0, 15):
        x = np.full((16, 8), val, dtype=np.int32)
        assert np.array_equal(oracle.unpack_int4(oracle.pack_int4(x)), x)


def test_pack_nibble_position():
    """test_quant.py:41-47: x[3,0]=0xA lands at bits [12:16]."""
    x = np.zeros((8, 1), dtype=np.int32)
    x[3, 0] = 0xA
    assert int(oracle.pack_int4(x)[0, 0]) == (0xA << 12)


def test_pack_requires_k_div_8():
    with pytest.raises(AssertionError):
        oracle.pack_int4(np.zeros((7, 4), dtype=np.int32))


def test_pack_rejects_out_of_range():
    with pytest.raises(AssertionError):
        oracle.pack_int4(np.full((8, 2), 16, dtype=np.int32))


@pytest.mark.parametrize("group_size", [64, 128])
@pytest.mark.parametrize("K,N", [(128, 256), (4096, 512)])
def test_quant_shapes_dtypes(K, N, group_size):
    """test_quant.py:58-68."""
    W = synth.make_w(K, N, 1.0, seed=K + N)
    qw, s, z = oracle.quantize_weight(W, group_size)
    assert qw.shape == (K // 8, N) and qw.dtype == np.int32
    assert s.shape == (K // group_size, N) and s.dtype == np.float16
    assert z.shape == (K // group_size, N) and z.dtype == np.float16
    assert np.all(z >= 0) and np.all(z <= 15) and np.all(z == np.round(z))


@pytest.mark.parametrize("group_size", [64, 128])
def test_quant_dequant_roundtrip_error(group_size):
    """test_quant.py:71-90: mean relative error < 15% on N(0,1) weights."""
    W = synth.make_w(4096, 1024, 1.0, seed=1)
    qw, s, z = oracle.quantize_weight(W, group_size)
    Wdq = oracle.dequantize_weight(qw, s, z, group_size)
    rel = np.abs(Wdq.astype(np.float32) - W.astype(np.float32)).mean() / np.abs(W.astype(np.float32)).mean()
    assert rel < 0.15


def test_dequant_constant_group_is_exact():
    """test_quant.py:93-100."""
    W = np.zeros((128, 8), dtype=np.float16)
    W[:, 0] = 3.0
    qw, s, z = oracle.quantize_weight(W, 64)
    assert np.allclose(oracle.dequantize_weight(qw, s, z, 64).astype(np.float32), W.astype(np.float32), atol=1e-3)


def test_quant_divisibility_errors():
    """test_quant.py:103-109."""
    with pytest.raises(ValueError):
        oracle.quantize_weight(np.zeros((100, 16), np.float16), 64)
    with pytest.raises(ValueError):
        oracle.quantize_weight(np.zeros((96, 16), np.float16), 64)


# ----------------------------- golden vectors from the reference -----------------
def test_golden_quantise_bit_exact(golden):
    for name in _cases(golden):
        M, K, N, G = (int(v) for v in golden[f"{name}/meta"])
        qw, s, z = oracle.quantize_weight(golden[f"{name}/W"], G)
        assert np.array_equal(qw, golden[f"{name}/qweight"]), name
        assert np.array_equal(_bits(s), _bits(golden[f"{name}/scales"])), name
        assert np.array_equal(_bits(z), _bits(golden[f"{name}/zeros"])), name


def test_golden_dequantise_bit_exact(golden):
    for name in _cases(golden):
        G = int(golden[f"{name}/meta"][3])
        w = oracle.dequantize_weight(golden[f"{name}/qweight"], golden[f"{name}/scales"],
                                     golden[f"{name}/zeros"], G)
        assert np.array_equal(_bits(w), _bits(golden[f"{name}/w_dq"])), name


def test_golden_gemm(golden):
    for name in _cases(golden):
        G = int(golden[f"{name}/meta"][3])
        args = (golden[f"{name}/X"], golden[f"{name}/qweight"], golden[f"{name}/scales"],
                golden[f"{name}/zeros"], G)
        assert_gemm_close(oracle.reference_w4a16(*args), golden[f"{name}/y_ref"], name)
        assert_gemm_close(oracle.dequant_then_matmul(*args), golden[f"{name}/y_dtm"], name)


def test_golden_pack_vectors(golden):
    for key in [k for k in golden.files if k.startswith("pack_") and k.endswith("/q")]:
        base = key[:-2]
        assert np.array_equal(oracle.pack_int4(golden[key]), golden[base + "/packed"]), base


def test_golden_special_zero_points(golden):
    """All-zero group -> zero-point -0.0 (sign kept by the reference's clamp);
    all-positive group -> 0; all-negative group -> 15."""
    z = golden["g64_special/zeros"]
    assert np.all(_bits(z[:, 0]) == 0x8000)
    assert np.all(z[:, 2] == 0) and np.all(z[:, 3] == 15)
    qw, s, zz = oracle.quantize_weight(golden["g64_special/W"], 64)
    assert np.array_equal(_bits(zz), _bits(z))


def test_oracle_configuration_digests():
    """The 16x4096x4096, G=128 oracle configuration against the reference's outputs."""
    ref = np.load(os.path.join(GOLDEN, "golden_oracle_cfg.npz"))
    X, W = synth.oracle_cfg_inputs()
    sha = lambda a: hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()  # noqa: E731
    assert sha(X) == str(ref["x_sha256"]) and sha(W) == str(ref["w_sha256"])
    qw, s, z = oracle.quantize_weight(W, 128)
    assert sha(qw) == str(ref["qweight_sha256"])
    assert sha(s) == str(ref["scales_sha256"])
    assert sha(z) == str(ref["zeros_sha256"])
    assert sha(oracle.dequantize_weight(qw, s, z, 128)) == str(ref["w_dq_sha256"])
    assert_gemm_close(oracle.reference_w4a16(X, qw, s, z, 128), ref["y_ref"], "oracle cfg")
