# SPDX-License-Identifier: MIT OR Apache-2.0
"""The host-side mirror of src/lib.rs on the CPU: geometry, the alignment gate, error behaviour.
No kernel runs here (CPU tensors are rejected before any launch: there is no CPU fallback)."""

import pytest
import torch

import candle_fused_attn as cfa


def test_qkv_geometry_canvas():
    # src/lib.rs:191-206 at the canvas shape: [64, 240, 1152], 6 heads
    t = torch.empty(64, 240, 1152)
    dims, strides, offs = cfa.qkv_geometry(tuple(t.shape), t.stride(), 6)
    assert dims == (64, 6, 240, 64)
    assert strides == (276480, 64, 1152)
    assert offs == (0, 384, 768)


def test_qkv_geometry_errors():
    with pytest.raises(cfa.FusedAttentionError, match="is not 3 x 5 heads"):
        cfa.qkv_geometry((2, 3, 1152), (3456, 1152, 1), 5)
    with pytest.raises(cfa.FusedAttentionError, match="is not 3 x 0 heads"):
        cfa.qkv_geometry((2, 3, 1152), (3456, 1152, 1), 0)
    with pytest.raises(cfa.FusedAttentionError, match="last dimension must be contiguous"):
        cfa.qkv_geometry((2, 3, 1152), (3456, 1, 3), 6)


def test_float4_aligned():
    x = torch.empty(16, 1024, 3, 12, 64)
    q = x[:, :, 0].permute(0, 2, 1, 3)
    assert q.stride() == (2359296, 64, 2304, 1)
    assert cfa.float4_aligned(q)
    assert cfa.float4_aligned(x[:, :, 1].permute(0, 2, 1, 3))
    y = torch.empty(2, 3, 5, 66)[..., 1:65]  # offset 1: misaligned
    assert not cfa.float4_aligned(y)
    z = torch.empty(2, 3, 64, 5).transpose(2, 3)  # d not contiguous
    assert not cfa.float4_aligned(z)


def test_rejects_cpu_tensors_and_dtypes():
    qkv = torch.randn(2, 7, 3 * 3 * 64)
    with pytest.raises(cfa.FusedAttentionError, match="CUDA tensors required"):
        cfa.fused_attention_qkv(qkv, 3, 0.125, False)
    with pytest.raises(cfa.FusedAttentionError, match="f32 only"):
        cfa.fused_attention_qkv(qkv.double(), 3, 0.125, False)
    q = torch.randn(2, 3, 7, 64)
    with pytest.raises(cfa.FusedAttentionError, match="CUDA tensors required"):
        cfa.fused_attention(q, q, q, 0.125, False)
    with pytest.raises(cfa.FusedAttentionError, match="share one"):
        cfa.fused_attention(q, q[:, :2], q, 0.125, False)
