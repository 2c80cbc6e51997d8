# SPDX-License-Identifier: MIT OR Apache-2.0
"""The C++ host layer (candle-fused-attn_b200/host, libcfa_host.so): builds, exports the API and
passes the parity test's device-free part (layout predicates, qkv geometry, error messages of
src/lib.rs). The device part runs in tests/test_cpp_host_gpu.py."""

import importlib.util
import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
BIN = ROOT / "tests" / "cpp" / "parity_host"


def build_binary() -> Path:
    spec = importlib.util.spec_from_file_location("cfa_build", ROOT / "candle-fused-attn_b200" / "build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.build_host()
    subprocess.run(["make", "-s", "-C", str(ROOT / "oracle")], check=True)
    subprocess.run(["make", "-s", "-C", str(ROOT / "tests" / "cpp")], check=True)
    return BIN


def test_host_layer_exports_the_api():
    build_binary()
    lib = ROOT / "candle-fused-attn_b200" / "candle_fused_attn" / "libcfa_host.so"
    out = subprocess.run(["nm", "-D", "-C", "--defined-only", str(lib)], capture_output=True,
                         text=True, check=True).stdout
    for name in ("candle_fused_attn::fused_attention_qkv(", "candle_fused_attn::fused_attention(",
                 "candle_fused_attn::float4_aligned(", "candle_fused_attn::qkv_geometry(",
                 "candle_fused_attn::check_shapes(", "candle_fused_attn::bhs_strides(",
                 "candle_fused_attn::aligned_grad(", "candle_fused_attn::FusedAttention::bwd(",
                 "candle_fused_attn::FusedAttentionQkv::bwd("):
        assert name in out, name


def test_host_only_checks():
    r = subprocess.run([str(build_binary()), "--host-only"], capture_output=True, text=True)
    print(r.stdout, r.stderr)
    assert r.returncode == 0
    assert "0 failures" in r.stdout
