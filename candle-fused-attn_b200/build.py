# SPDX-License-Identifier: MIT OR Apache-2.0
"""Builds libcfa.so in-tree: the sm_100a kernels and the C ABI of include/cfa.h.

    python candle-fused-attn_b200/build.py

nvcc cross-compiles without a GPU; the shared library lands beside the Python package
(candle_fused_attn/libcfa.so) and travels with the tree. SASS only (code=sm_100a), no PTX: no
driver JIT, so the arithmetic (FMA contraction included) is fixed at build time.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OUT = PKG / "candle_fused_attn" / "libcfa.so"
SOURCES = ["fwd_ffma.cu", "bwd_ffma.cu", "hd_ffma.cu", "cfa_abi.cu", "cfa_noalloc.cu"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "-Xptxas", "-v",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[Path]:
    return [CSRC / s for s in SOURCES]


def up_to_date() -> bool:
    if not OUT.exists():
        return False
    t = OUT.stat().st_mtime
    deps = sources() + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [ROOT / "include" / "cfa.h"]
    return all(p.stat().st_mtime <= t for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return OUT
    cmd = [nvcc(), *NVCC_FLAGS, "-I", str(ROOT / "include"), "-I", str(CSRC),
           "-o", str(OUT), *map(str, sources())]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode})")
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
