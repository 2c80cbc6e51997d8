# SPDX-License-Identifier: MIT OR Apache-2.0
"""The BASELINE.json configs at full size, where the oracle cannot run every slice in seconds:
a sample of (batch, head) slices against the oracle, and size-independent properties (bitwise
reruns, batch-split invariance, finiteness)."""

import pytest
import torch

import candle_fused_attn as cfa
from oracle import oracle

pytestmark = pytest.mark.gpu


def fwd_bwd_qkv(x, dout, h, causal, scale=0.125):
    x = x.detach().requires_grad_(True)
    o = cfa.fused_attention_qkv(x, h, scale, causal)
    (o * dout).sum().backward()
    torch.cuda.synchronize()
    return o.detach(), x.grad.detach()


def slice_check(qkv, dout, h, causal, o, g, slices, scale=0.125):
    """Oracle on the given (batch, head) slices only; compare those slices."""
    b, s, three_hd = qkv.shape
    d = three_hd // (3 * h)
    q, k, v = oracle.qkv_views(qkv, h)
    gv = oracle.heads_view(dout, h)
    for bh in slices:
        rng = (bh, bh + 1)
        o_ref, lse_ref = oracle.forward(q, k, v, scale, causal, bh_range=rng)
        d_ref = oracle.backward(q, k, v, o_ref, lse_ref, gv, scale, causal, bh_range=rng)
        bi, hi = divmod(bh, h)
        oc = o.view(b, s, h, d)[bi, :, hi].cpu()
        gc = g.view(b, s, 3, h, d)[bi, :, :, hi].cpu()
        assert oracle.normwise(oc, o_ref[bi, :, hi]) < 1e-5
        assert oracle.normwise(gc, d_ref[bi, :, :, hi]) < 1e-5


def test_canvas(cuda):
    """qkv [64, 240, 1152] N(0,1)*0.5, 6 heads, non-causal, dO N(0, 1)."""
    qkv, dout = oracle.seeded_inputs(64, 6, 240, 0, 0.5)
    x, gd = qkv.to(cuda), dout.to(cuda)
    o, g = fwd_bwd_qkv(x, gd, 6, False)
    assert torch.isfinite(o).all() and torch.isfinite(g).all()
    slice_check(qkv, dout, 6, False, o, g, [0, 1, 191, 383])
    o2, g2 = fwd_bwd_qkv(x, gd, 6, False)
    assert torch.equal(o.view(torch.int32), o2.view(torch.int32))
    assert torch.equal(g.view(torch.int32), g2.view(torch.int32))
    # batch-split invariance: the shards of an 8-way split give the same bits
    for lo in range(0, 64, 8):
        os_, gs_ = fwd_bwd_qkv(x[lo:lo + 8], gd[lo:lo + 8], 6, False)
        assert torch.equal(os_.view(torch.int32), o[lo:lo + 8].view(torch.int32))
        assert torch.equal(gs_.view(torch.int32), g[lo:lo + 8].view(torch.int32))


def test_strided_causal(cuda):
    """x [16, 1024, 3, 12, 64], q/k/v permuted views, causal."""
    g = torch.Generator().manual_seed(0)
    x = torch.randn(16, 1024, 3, 12, 64, generator=g)
    do = torch.randn(16, 12, 1024, 64, generator=g)
    xd = x.to(cuda).requires_grad_(True)
    q, k, v = (xd[:, :, i].permute(0, 2, 1, 3) for i in range(3))
    o = cfa.fused_attention(q, k, v, 0.125, True)
    (o * do.to(cuda)).sum().backward()
    torch.cuda.synchronize()
    qc, kc, vc = (x[:, :, i].permute(0, 2, 1, 3) for i in range(3))
    for bh in (0, 100, 191):
        rng = (bh, bh + 1)
        o_ref, lse_ref = oracle.forward(qc, kc, vc, 0.125, True, bh_range=rng)
        d_ref = oracle.backward(qc, kc, vc, o_ref, lse_ref, do, 0.125, True, bh_range=rng)
        bi, hi = divmod(bh, 12)
        assert oracle.normwise(o.detach()[bi, hi].cpu(), o_ref[bi, :, hi]) < 1e-5
        assert oracle.normwise(xd.grad[bi, :, :, hi].cpu(), d_ref[bi, :, :, hi]) < 1e-5


def test_long_causal(cuda):
    """qkv [4, 8192, 3072] N(0,1)*0.5, 16 heads, causal: 128 key blocks chain
    their dQ turns; bitwise reruns and two slices against the oracle."""
    qkv, dout = oracle.seeded_inputs(4, 16, 8192, 0, 0.5)
    x, gd = qkv.to(cuda), dout.to(cuda)
    o, g = fwd_bwd_qkv(x, gd, 16, True)
    assert torch.isfinite(o).all() and torch.isfinite(g).all()
    slice_check(qkv, dout, 16, True, o, g, [0, 63])
    o2, g2 = fwd_bwd_qkv(x, gd, 16, True)
    assert torch.equal(g.view(torch.int32), g2.view(torch.int32))


@pytest.mark.parametrize("d", [32, 128])
def test_canvas_shaped_head_dims(cuda, d):
    """The canvas projection [64, 240, 1152] as 384 / d heads of d (csrc/hd_ffma.cu), non-causal:
    sampled slices against the oracle, bitwise reruns, an 8-way batch split bit for bit."""
    h, scale = 384 // d, d ** -0.5
    qkv, dout = oracle.seeded_inputs(64, h, 240, 0, 0.5, d=d)
    x, gd = qkv.to(cuda), dout.to(cuda)
    o, g = fwd_bwd_qkv(x, gd, h, False, scale)
    assert torch.isfinite(o).all() and torch.isfinite(g).all()
    slice_check(qkv, dout, h, False, o, g, [0, 1, 64 * h - 1], scale)
    o2, g2 = fwd_bwd_qkv(x, gd, h, False, scale)
    assert torch.equal(o.view(torch.int32), o2.view(torch.int32))
    assert torch.equal(g.view(torch.int32), g2.view(torch.int32))
    for lo in range(0, 64, 8):
        os_, gs_ = fwd_bwd_qkv(x[lo:lo + 8], gd[lo:lo + 8], h, False, scale)
        assert torch.equal(os_.view(torch.int32), o[lo:lo + 8].view(torch.int32))
        assert torch.equal(gs_.view(torch.int32), g[lo:lo + 8].view(torch.int32))


def test_long_causal_head_dim_128(cuda):
    """The long projection [4, 8192, 3072] as 8 heads of 128, causal (the suite's head-dim-128
    config): 128 key blocks chain their dQ turns in the 512-thread backward; two slices against
    the oracle and a bitwise rerun."""
    h, scale = 8, 128 ** -0.5
    qkv, dout = oracle.seeded_inputs(4, h, 8192, 0, 0.5, d=128)
    x, gd = qkv.to(cuda), dout.to(cuda)
    o, g = fwd_bwd_qkv(x, gd, h, True, scale)
    assert torch.isfinite(o).all() and torch.isfinite(g).all()
    slice_check(qkv, dout, h, True, o, g, [0, 31], scale)
    o2, g2 = fwd_bwd_qkv(x, gd, h, True, scale)
    assert torch.equal(g.view(torch.int32), g2.view(torch.int32))
