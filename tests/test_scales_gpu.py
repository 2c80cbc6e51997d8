# SPDX-License-Identifier: MIT OR Apache-2.0
"""Parity at scales that are not powers of two.

With scale 1/8 (the reference tests' 1/sqrt(64)) the product S * scale is exact, so those tests
never exercise the rounding of the scale multiply. The public API takes any f32 scale (the
reference scales by 1/sqrt(d), src/lib.rs:248 multiplies q k^T by it before the softmax; its
tests/parity.rs:80 takes 1/sqrt(d), not dyadic at d = 8). These cases run the tensor-core pair at
0.1, 1/sqrt(48), 0.3 and 1.0 through both public functions, causal and not, against the fp32
composed path (max-abs 5e-6 with the fp64 tie-break of tests/test_parity_gpu.py, and 1e-5
normwise), on the reference tests' closed-form inputs and on canvas slices, and require bitwise
reruns of the backward.
"""

import pytest
import torch

import candle_fused_attn as cfa
from oracle import oracle

pytestmark = pytest.mark.gpu

BAND_MAXABS = 5e-6  # tests/parity.rs:218
BAND_NORMWISE = 1e-5
SCALES = [0.1, 48 ** -0.5, 0.3, 1.0]


def run(path, qkv, w, h, scale, causal, dev):
    b, s, _ = qkv.shape
    x = qkv.to(dev).requires_grad_(True)
    if path == "fused":
        q, k, v = oracle.qkv_views(x, h)
        out = cfa.fused_attention(q, k, v, scale, causal).transpose(1, 2).reshape(b, s, -1)
    else:
        out = cfa.fused_attention_qkv(x, h, scale, causal)
    (out * w.to(dev)).sum().backward()
    cfa.check_status()
    return out.detach().cpu(), x.grad.detach().cpu()


def check_band(got, r32, r64, name):
    """Max-abs against the fp32 composed path, an element beyond the band passing when it is no
    farther from the fp64 path than the fp32 one is; and the normwise band."""
    band = BAND_MAXABS * max(1.0, r32.abs().max().item())
    off = (got - r32).abs() >= band
    worse = (got.double() - r64).abs() > (r32.double() - r64).abs() + 1e-7
    bad = int((off & worse).sum())
    assert bad == 0, (f"{name}: {bad} elements beyond {band:.1e} of the fp32 path and farther "
                      f"from fp64 than it (max-abs {(got - r32).abs().max():.2e})")
    nw = oracle.normwise(got, r32)
    assert nw < BAND_NORMWISE, f"{name} normwise {nw:.2e}"


@pytest.mark.parametrize("scale", SCALES, ids=lambda x: f"scale{x:.4g}")
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("path", ["fused", "fused_qkv"])
def test_closed_form(cuda, path, causal, scale):
    b, s, h = 2, 97, 3
    qkv, w = oracle.closed_form_inputs(b, s, h, 64)
    o32, _, g32 = oracle.qkv_forward_backward(qkv, w, h, scale, causal)
    o64, _, g64 = oracle.qkv_forward_backward(qkv, w, h, scale, causal, dtype=torch.float64)
    o, g = run(path, qkv, w, h, scale, causal, cuda)
    check_band(o, o32, o64, "O")
    check_band(g, g32, g64, "dqkv")


@pytest.mark.parametrize("scale", SCALES, ids=lambda x: f"scale{x:.4g}")
@pytest.mark.parametrize("causal", [False, True])
def test_canvas_slice(cuda, causal, scale):
    """Four batches of the canvas config (s = 240, 6 heads, N(0,1) * 0.5), both public functions
    bit-identical to each other, and the backward rerun bit for bit."""
    b, s, h = 4, 240, 6
    qkv, w = oracle.seeded_inputs(b, h, s, 31, 0.5)
    o32, _, g32 = oracle.qkv_forward_backward(qkv, w, h, scale, causal)
    o64, _, g64 = oracle.qkv_forward_backward(qkv, w, h, scale, causal, dtype=torch.float64)
    o, g = run("fused_qkv", qkv, w, h, scale, causal, cuda)
    check_band(o, o32, o64, "O")
    check_band(g, g32, g64, "dqkv")
    o2, g2 = run("fused_qkv", qkv, w, h, scale, causal, cuda)
    o3, g3 = run("fused", qkv, w, h, scale, causal, cuda)
    assert torch.equal(o, o2) and torch.equal(g, g2)
    assert torch.equal(o, o3) and torch.equal(g, g3)
