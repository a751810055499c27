"""Generate the golden vectors in this folder by running the REFERENCE itself.

Run once, on a machine where the reference project is checked out:

    python tests/golden/make_golden.py --reference-src <path>/w4a16-kernel/src

It imports the reference's own ``w4a16.quant`` and ``w4a16.reference`` modules
(pure PyTorch, CPU) and records, for seeded inputs from ``synth.py``:

* ``quantize_weight`` outputs (qweight / scales / zeros, bit patterns),
* ``dequantize_weight`` output (fp16 bit patterns),
* ``reference_w4a16`` and ``dequant_then_matmul`` outputs (fp16),
* ``pack_int4`` / ``unpack_int4`` round trips on random codes.

Small cases are stored whole in ``golden_small.npz``; for the 16x4096x4096
oracle configuration the packed weights are stored as SHA-256 digests and the
[16, 4096] output whole, in ``golden_oracle_cfg.npz``. The GPU box never runs
this script; the tests only read the ``.npz`` files.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import synth  # noqa: E402

# (name, M, K, N, G, sigma, seed, kind)
SMALL_CASES = [
    ("g64_n72", 3, 256, 72, 64, 1.0, 11, "normal"),
    ("g128_n40", 5, 384, 40, 128, 0.02, 12, "normal"),
    ("g64_special", 4, 256, 16, 64, 1.0, 13, "special"),
    ("g128_special", 2, 256, 8, 128, 1.0, 14, "special"),
    ("g64_odd_n13", 2, 128, 13, 64, 1.0, 15, "normal"),
    ("g64_n1", 1, 128, 1, 64, 1.0, 16, "normal"),
    ("g64_fp32_in", 3, 128, 24, 64, 1.0, 17, "fp32"),
    ("g256_m37", 37, 512, 136, 256, 0.05, 18, "normal"),
    ("g128_outliers", 9, 256, 96, 128, 0.015, 19, "outliers"),
    ("g192_m33", 33, 384, 48, 192, 1.0, 20, "normal"),
]


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", required=True,
                    help="the reference's w4a16-kernel/src directory")
    args = ap.parse_args()
    sys.path.insert(0, args.reference_src)
    import torch
    from w4a16.quant import quantize_weight, dequantize_weight, pack_int4, unpack_int4
    from w4a16.reference import reference_w4a16, dequant_then_matmul

    torch.set_num_threads(1)  # one summation order for the stored fp32 GEMM outputs
    out = {}
    for name, M, K, N, G, sigma, seed, kind in SMALL_CASES:
        if kind == "special":
            W = synth.make_special_w(K, N, G, seed)
        elif kind == "fp32":
            W = synth.make_w(K, N, sigma, seed, dtype=np.float32)
        elif kind == "outliers":
            W = synth.make_w(K, N, sigma, seed, outlier_frac=0.001)
        else:
            W = synth.make_w(K, N, sigma, seed)
        X = synth.make_x(M, K, seed + 1000)
        qw, s, z = quantize_weight(torch.from_numpy(W), G)
        Wdq = dequantize_weight(qw, s, z, G)
        Xt = torch.from_numpy(X)
        Y = reference_w4a16(Xt, qw, s, z, G)
        Ydm = dequant_then_matmul(Xt, qw, s, z, G)
        out[f"{name}/W"] = W
        out[f"{name}/X"] = X
        out[f"{name}/qweight"] = qw.numpy()
        out[f"{name}/scales"] = s.numpy()
        out[f"{name}/zeros"] = z.numpy()
        out[f"{name}/w_dq"] = Wdq.numpy()
        out[f"{name}/y_ref"] = Y.numpy()
        out[f"{name}/y_dtm"] = Ydm.numpy()
        out[f"{name}/meta"] = np.array([M, K, N, G], dtype=np.int64)

    # pack / unpack known answers on random codes (test_quant.py:21-31 shapes)
    rng = np.random.default_rng(7)
    for K, N in [(8, 1), (64, 16), (128, 33)]:
        q = rng.integers(0, 16, size=(K, N), dtype=np.int32)
        p = pack_int4(torch.from_numpy(q))
        out[f"pack_{K}x{N}/q"] = q
        out[f"pack_{K}x{N}/packed"] = p.numpy()
        assert np.array_equal(unpack_int4(p, K).numpy(), q)
    np.savez_compressed(os.path.join(HERE, "golden_small.npz"), **out)

    # oracle configuration: digests of the packed weights, the output in full
    X, W = synth.oracle_cfg_inputs()
    G = synth.ORACLE_CFG["G"]
    qw, s, z = quantize_weight(torch.from_numpy(W), G)
    Wdq = dequantize_weight(qw, s, z, G)
    Y = reference_w4a16(torch.from_numpy(X), qw, s, z, G)
    np.savez_compressed(
        os.path.join(HERE, "golden_oracle_cfg.npz"),
        qweight_sha256=np.array(sha(qw.numpy())),
        scales_sha256=np.array(sha(s.numpy())),
        zeros_sha256=np.array(sha(z.numpy())),
        w_dq_sha256=np.array(sha(Wdq.numpy())),
        x_sha256=np.array(sha(X)),
        w_sha256=np.array(sha(W)),
        y_ref=Y.numpy(),
        scales_row0=s.numpy()[0],
        zeros_row0=z.numpy()[0],
        qweight_row0=qw.numpy()[0],
    )
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
