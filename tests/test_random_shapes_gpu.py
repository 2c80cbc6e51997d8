# SPDX-License-Identifier: MIT OR Apache-2.0
"""Randomised parity (hypothesis, derandomised): batch, heads, sequence length, causality, and the
operand layout -- separate q, k, v tensors with padded (batch, head, seq) strides, or views of one
fused projection -- drawn at random; forward and backward against the CPU oracle, and a rerun that
must give the same bits."""

import pytest
import torch
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

import candle_fused_attn as cfa
from oracle import oracle

pytestmark = pytest.mark.gpu


def close(got, ref):
    """The reference tests' max-abs band (tests/parity.rs:218) always; the normwise bound too
    unless the reference is itself rounding noise (e.g. dQ, dK at s = 1, where softmax is exactly
    1 and both gradients are mathematically zero)."""
    assert (got - ref).abs().max() < 5e-6
    if ref.norm() / max(1.0, ref.numel()) ** 0.5 > 1e-5:
        assert oracle.normwise(got, ref) < 1e-5


def padded(b, h, s, pad_s, pad_h, gen):
    """A [b, h, s, 64] view with row stride 64 + 4 pad_s and head stride s (64 + 4 pad_s) + 4 pad_h
    (all multiples of 4 floats: read in place)."""
    ss = 64 + 4 * pad_s
    sh = s * ss + 4 * pad_h
    base = torch.randn(b * h * sh + 64, generator=gen)
    return base.as_strided((b, h, s, 64), (h * sh, sh, ss, 1))


@settings(max_examples=30, deadline=None, derandomize=True,
          suppress_health_check=[HealthCheck.function_scoped_fixture])
@given(b=st.integers(1, 3), h=st.integers(1, 4), s=st.integers(1, 300), causal=st.booleans(),
       fused=st.booleans(), pad_s=st.integers(0, 3), pad_h=st.integers(0, 2),
       seed=st.integers(0, 2**31 - 1))
def test_random_shapes(cuda, b, h, s, causal, fused, pad_s, pad_h, seed):
    gen = torch.Generator().manual_seed(seed)
    if fused:
        qkv = torch.randn(b, s, 3 * h * 64, generator=gen)
        q, k, v = oracle.qkv_views(qkv, h)
    else:
        q, k, v = (padded(b, h, s, pad_s, pad_h, gen) for _ in range(3))
    do = torch.randn(b, h, s, 64, generator=gen)
    o_ref, lse_ref = oracle.forward(q, k, v, 0.125, causal)
    g_ref = oracle.backward(q, k, v, o_ref, lse_ref, do, 0.125, causal)

    def run():
        qd, kd, vd = (t.to(cuda) for t in (q, k, v))
        if not fused:  # keep the padded strides on the device
            qd, kd, vd = (torch.empty_strided(t.shape, t.stride(), device=cuda).copy_(t)
                          for t in (q, k, v))
        qd, kd, vd = (t.requires_grad_(True) for t in (qd, kd, vd))
        o = cfa.fused_attention(qd, kd, vd, 0.125, causal)
        o.backward(do.to(cuda))
        torch.cuda.synchronize()
        return (o.detach().cpu(), qd.grad.cpu(), kd.grad.cpu(), vd.grad.cpu())

    o, dq, dk, dv = run()
    close(o, o_ref.transpose(1, 2))
    for got, i in ((dq, 0), (dk, 1), (dv, 2)):
        close(got, g_ref[:, :, i].transpose(1, 2))
    again = run()
    for x, y in zip(again, (o, dq, dk, dv)):
        assert torch.equal(x.view(torch.int32), y.view(torch.int32))


def padded_d(b, h, s, d, pad_s, pad_h, gen):
    """padded() for head dim d: row stride d + 4 pad_s, head stride s (d + 4 pad_s) + 4 pad_h."""
    ss = d + 4 * pad_s
    sh = s * ss + 4 * pad_h
    base = torch.randn(b * h * sh + d, generator=gen)
    return base.as_strided((b, h, s, d), (h * sh, sh, ss, 1))


@settings(max_examples=24, deadline=None, derandomize=True,
          suppress_health_check=[HealthCheck.function_scoped_fixture])
@given(d=st.sampled_from([32, 128]), b=st.integers(1, 3), h=st.integers(1, 3),
       s=st.integers(1, 300), causal=st.booleans(), fused=st.booleans(),
       pad_s=st.integers(0, 3), pad_h=st.integers(0, 2), seed=st.integers(0, 2**31 - 1))
def test_random_shapes_head_dims(cuda, d, b, h, s, causal, fused, pad_s, pad_h, seed):
    """The same draws for the head dims 32 and 128 (csrc/hd_ffma.cu), scale 1/sqrt(d), the
    max-abs band scaled by the output magnitude."""
    gen = torch.Generator().manual_seed(seed)
    scale = d ** -0.5
    if fused:
        qkv = torch.randn(b, s, 3 * h * d, generator=gen)
        q, k, v = oracle.qkv_views(qkv, h)
    else:
        q, k, v = (padded_d(b, h, s, d, pad_s, pad_h, gen) for _ in range(3))
    do = torch.randn(b, h, s, d, generator=gen)
    o_ref, lse_ref = oracle.forward(q, k, v, scale, causal)
    g_ref = oracle.backward(q, k, v, o_ref, lse_ref, do, scale, causal)

    def run():
        qd, kd, vd = (t.to(cuda) for t in (q, k, v))
        if not fused:
            qd, kd, vd = (torch.empty_strided(t.shape, t.stride(), device=cuda).copy_(t)
                          for t in (q, k, v))
        qd, kd, vd = (t.requires_grad_(True) for t in (qd, kd, vd))
        o = cfa.fused_attention(qd, kd, vd, scale, causal)
        o.backward(do.to(cuda))
        torch.cuda.synchronize()
        return (o.detach().cpu(), qd.grad.cpu(), kd.grad.cpu(), vd.grad.cpu())

    def close_d(got, ref):
        assert (got - ref).abs().max() < 5e-6 * max(1.0, ref.abs().max().item())
        if ref.norm() / max(1.0, ref.numel()) ** 0.5 > 1e-5:
            assert oracle.normwise(got, ref) < 1e-5

    o, dq, dk, dv = run()
    close_d(o, o_ref.transpose(1, 2))
    for got, i in ((dq, 0), (dk, 1), (dv, 2)):
        close_d(got, g_ref[:, :, i].transpose(1, 2))
    again = run()
    for x, y in zip(again, (o, dq, dk, dv)):
        assert torch.equal(x.view(torch.int32), y.view(torch.int32))
