"""Shared pytest setup.

Puts the package source root and the repository root (for ``oracle``) on
``sys.path`` -- as the reference's conftest puts ``src/`` there -- registers
the ``gpu`` marker, and seeds torch per session.

``-m "not gpu"`` runs everything that needs no GPU: the oracle against the
reference's golden vectors, the C-ABI library's symbol table, and the host
logic. ``-m gpu`` runs the parity tests on a B200 through the C ABI.
"""
from __future__ import annotations

import os
import sys

import pytest
import torch

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
PKG_ROOT = os.path.join(ROOT, "w4a16-dequant-fused-matmul-kernel_b200")
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
for p in (PKG_ROOT, ROOT, GOLDEN):
    if p not in sys.path:
        sys.path.insert(0, p)

CUDA_AVAILABLE = torch.cuda.is_available()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")


def pytest_collection_modifyitems(config, items):
    if CUDA_AVAILABLE:
        return
    skip = pytest.mark.skip(reason="needs a CUDA GPU")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session", autouse=True)
def _seed() -> None:
    torch.manual_seed(0)
