# SPDX-License-Identifier: MIT OR Apache-2.0
"""Builds libcfa.so in-tree: the sm_100a kernels and the C ABI of include/cfa.h; and
libcfa_host.so, the C++ host layer above it (host/: src/lib.rs's API for compiled callers).

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
SOURCES = ["fwd_ffma.cu", "fwd_tc.cu", "bwd_ffma.cu", "bwd_tc.cu", "hd_ffma.cu", "linear_tc.cu",
           "cfa_abi.cu", "cfa_noalloc.cu"]
HOST_DIR = PKG / "host"
HOST_OUT = PKG / "candle_fused_attn" / "libcfa_host.so"
HOST_SOURCES = ["tensor.cu", "candle_fused_attn.cpp"]

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


def build_host(force: bool = False, verbose: bool = False) -> Path:
    """libcfa_host.so: host/*.cu|cpp linked against libcfa.so (found beside it via $ORIGIN)."""
    lib = build(force=force, verbose=verbose)
    srcs = [HOST_DIR / x for x in HOST_SOURCES]
    deps = srcs + list(HOST_DIR.glob("*.hpp")) + [lib, ROOT / "include" / "cfa.h"]
    if not force and HOST_OUT.exists() and all(
            p.stat().st_mtime <= HOST_OUT.stat().st_mtime for p in deps):
        return HOST_OUT
    cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
           "-Xcompiler", "-fPIC,-Wall", "-shared", "-I", str(ROOT / "include"), "-I", str(HOST_DIR),
           "-o", str(HOST_OUT), *map(str, srcs), "-L", str(lib.parent), "-lcfa",
           "-Xlinker", "-rpath", "-Xlinker", "$ORIGIN"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on the host layer ({r.returncode})")
    return HOST_OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
    print(build_host(force="--force" in sys.argv, verbose=True))
