# SPDX-License-Identifier: MIT OR Apache-2.0
"""The C++ host layer's parity test on the GPU: tests/parity.rs's CUDA tests in C++ (the
fused_attention / fused_attention_qkv paths against the CPU oracle within 5e-6, 8 bitwise
reruns, merge-heads readiness, two backwards over one forward, error messages, head dims 32 and
128), through libcfa_host.so -> libcfa.so."""

import subprocess

import pytest

from test_cpp_host import build_binary

pytestmark = pytest.mark.gpu


def test_cpp_parity(cuda):
    r = subprocess.run([str(build_binary())], capture_output=True, text=True, timeout=600)
    print(r.stdout, r.stderr)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "0 failures" in r.stdout
