# SPDX-License-Identifier: MIT OR Apache-2.0
"""HostPipeline (host buffers in and out, batch chunks over three streams) gives the same bits as
one whole-batch fused_attention_qkv forward + backward on device tensors, step after step."""

import pytest
import torch

import candle_fused_attn as cfa
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("b,chunks,slots,causal", [(20, 6, 3, False), (7, 7, 2, True),
                                                   (5, 1, 1, False)])
def test_host_pipeline_bitwise(cuda, b, chunks, slots, causal):
    h, s = 6, 240
    pipe = cfa.HostPipeline(b, h, s, 0.125, causal, cuda, chunks=chunks, slots=slots)
    o_h = torch.empty(b, s, h * 64).pin_memory()
    g_h = torch.empty(b, s, 3 * h * 64).pin_memory()
    for seed in (1, 2):
        qkv, dout = oracle.seeded_inputs(b, h, s, seed, 0.5)
        x = qkv.to(cuda).requires_grad_(True)
        o = cfa.fused_attention_qkv(x, h, 0.125, causal)
        o.backward(dout.to(cuda))
        pipe.step(qkv.pin_memory(), dout.pin_memory(), o_h, g_h)
        pipe.synchronize()
        assert torch.equal(o_h.view(torch.int32), o.detach().cpu().view(torch.int32))
        assert torch.equal(g_h.view(torch.int32), x.grad.cpu().view(torch.int32))
