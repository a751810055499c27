"""Seeded synthetic inputs shared by the golden-vector generator and the tests.

The reference measures on no dataset; every input is synthetic. Values follow
the shapes and distributions the benchmark configurations name: activations
``X ~ N(0, 1)`` and weights ``W ~ N(0, sigma^2)``, both rounded to fp16, drawn
from ``numpy.random.default_rng(seed)`` so that the same arrays can be rebuilt
on any machine without the generator's output being stored.
"""
from __future__ import annotations

import numpy as np


def make_x(M: int, K: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.standard_normal((M, K), dtype=np.float32).astype(np.float16)


def make_w(K: int, N: int, sigma: float, seed: int, dtype=np.float16,
           outlier_frac: float = 0.0, outlier_sigma: float = 0.2) -> np.ndarray:
    """``sigma * N(0,1)`` weights; optionally a Bernoulli(outlier_frac) mask of
    elements is redrawn from ``N(0, outlier_sigma^2)`` (the sweep config's
    "0.1% outliers")."""
    rng = np.random.default_rng(seed)
    W = rng.standard_normal((K, N), dtype=np.float32) * np.float32(sigma)
    if outlier_frac > 0:
        mask = rng.random((K, N)) < outlier_frac
        W[mask] = rng.standard_normal(int(mask.sum()), dtype=np.float32) * np.float32(outlier_sigma)
    return W.astype(dtype)


def make_special_w(K: int, N: int, G: int, seed: int) -> np.ndarray:
    """Weights with the edge cases the quantiser must get right, one per column:

    col 0: an all-zero column (constant groups, zero-point ``-0.0``)
    col 1: a constant 3.0 column (test_quant.py:93-100)
    col 2: all-positive values (zero-point clamps to 0)
    col 3: all-negative values (zero-point clamps to 15)
    col 4: one large outlier per group
    col 5: values that sit exactly on rounding ties
    other columns: N(0, 1)
    """
    assert N >= 8
    rng = np.random.default_rng(seed)
    W = rng.standard_normal((K, N), dtype=np.float32)
    W[:, 0] = 0.0
    W[:, 1] = 3.0
    W[:, 2] = np.abs(W[:, 2]) + 0.5
    W[:, 3] = -np.abs(W[:, 3]) - 0.5
    W[::G, 4] = 40.0
    W[:, 5] = np.tile(np.arange(G, dtype=np.float32) / 2.0 - G / 4.0, K // G)
    return W.astype(np.float16)


# The CPU oracle configuration named first in the benchmark configs:
# X fp16 [16, 4096] ~ N(0,1), W fp16 [4096, 4096] ~ N(0, 0.02), seed 0, G = 128.
ORACLE_CFG = dict(M=16, K=4096, N=4096, G=128, sigma=0.02, seed=0)


def oracle_cfg_inputs():
    c = ORACLE_CFG
    X = make_x(c["M"], c["K"], c["seed"])
    W = make_w(c["K"], c["N"], c["sigma"], c["seed"] + 1)
    return X, W
