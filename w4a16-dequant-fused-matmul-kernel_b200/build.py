"""Build the sm_100a C-ABI library ``w4a16/libw4a16_b200.so`` in-tree.

    python w4a16-dequant-fused-matmul-kernel_b200/build.py [--verbose]

The library is one CUDA translation unit (``csrc/w4a16_b200.cu``) compiled by
nvcc for ``sm_100a`` only, linked against the static CUDA runtime so that it
loads next to any torch build. No ``--use_fast_math``: the quantiser must use
IEEE division and round-half-even to stay bit-exact with the reference.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
OUT = os.path.join(HERE, "w4a16", "libw4a16_b200.so")
SOURCES = [os.path.join(CSRC, "w4a16_b200.cu")]
DEPENDS = SOURCES + [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cuh")] + [
    os.path.join(INCLUDE, "w4a16_b200.h")
]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the sm_100a library cannot be built")
    return cand


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    return all(os.path.getmtime(d) <= t for d in DEPENDS)


def build(verbose: bool = False, force: bool = False) -> str:
    if not force and up_to_date():
        return OUT
    cmd = [
        nvcc_path(),
        "-gencode", "arch=compute_100a,code=sm_100a",
        "-O3", "-lineinfo", "-std=c++17",
        "-Xcompiler", "-fPIC", "-shared",
        "-cudart", "static",
        "-I", INCLUDE, "-I", CSRC,
        "-o", OUT + ".tmp",
    ] + SOURCES
    if verbose:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed building the W4A16 library:\n" + r.stderr[-4000:])
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(verbose=a.verbose, force=a.force))
