# SPDX-License-Identifier: MIT OR Apache-2.0
"""The C ABI from a plain C program (tests/c_abi/abi_smoke.c): no Python or torch between the caller
and libcfa.so. The program is compiled here (gcc against include/cfa.h, linked to libcfa.so and
cudart) and its outputs are checked against the CPU oracle; the no-allocation backward must give
the same bits as the workspace one."""

import shutil
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from candle_fused_attn import _abi
from oracle import oracle

ROOT = Path(__file__).resolve().parents[1]
SRC = ROOT / "tests" / "c_abi" / "abi_smoke.c"


def _cuda_home():
    for c in ("/usr/local/cuda",):
        if Path(c, "include", "cuda_runtime.h").is_file():
            return Path(c)
    nvcc = shutil.which("nvcc")
    return Path(nvcc).resolve().parents[1] if nvcc else None


def build(tmp: Path) -> Path:
    cuda = _cuda_home()
    if cuda is None or shutil.which("gcc") is None:
        pytest.skip("gcc / CUDA headers unavailable")
    exe = tmp / "abi_smoke"
    libdir = _abi.LIB_PATH.parent
    cmd = ["gcc", "-O2", "-std=c11", "-o", str(exe), str(SRC), "-I", str(ROOT / "include"),
           "-I", str(cuda / "include"), "-L", str(libdir), "-lcfa",
           f"-Wl,-rpath,{libdir}", "-L", str(cuda / "lib64"), "-lcudart",
           f"-Wl,-rpath,{cuda / 'lib64'}"]
    subprocess.run(cmd, check=True)
    return exe


def test_c_program_builds(tmp_path):
    """CPU: the ABI header and library link from C."""
    build(tmp_path)


@pytest.mark.gpu
@pytest.mark.parametrize("b,h,s,causal", [(3, 2, 150, 0), (2, 3, 257, 1)])
def test_c_program_matches_oracle(tmp_path, cuda, b, h, s, causal):
    exe = build(tmp_path)
    qkv, dout = oracle.seeded_inputs(b, h, s, 21)
    qkv.numpy().tofile(tmp_path / "qkv.bin")
    dout.numpy().tofile(tmp_path / "dout.bin")
    out = subprocess.run([str(exe), str(b), str(h), str(s), str(causal)] +
                         [str(tmp_path / n) for n in ("qkv.bin", "dout.bin", "o.bin", "dqkv.bin",
                                                      "dqkv_na.bin")],
                         capture_output=True, text=True, timeout=120)
    sys.stdout.write(out.stdout + out.stderr)
    assert out.returncode == 0
    o = torch.from_numpy(np.fromfile(tmp_path / "o.bin", dtype=np.float32)).view(b, s, -1)
    g = torch.from_numpy(np.fromfile(tmp_path / "dqkv.bin", dtype=np.float32)).view(b, s, -1)
    g2 = torch.from_numpy(np.fromfile(tmp_path / "dqkv_na.bin", dtype=np.float32)).view(b, s, -1)
    o_ref, _, g_ref = oracle.qkv_forward_backward(qkv, dout, h, 0.125, bool(causal))
    assert oracle.normwise(o, o_ref) < 1e-5 and (o - o_ref).abs().max() < 5e-6
    assert oracle.normwise(g, g_ref) < 1e-5 and (g - g_ref).abs().max() < 5e-6
    assert torch.equal(g.view(torch.int32), g2.view(torch.int32))
