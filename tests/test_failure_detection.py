# SPDX-License-Identifier: MIT OR Apache-2.0
"""Failure detection without a GPU fault. On the GPU: a wait that nothing can satisfy runs out
after its limit (the bounded routine of the backward's dQ chain), the other waiters bail out as
soon as one has flagged the error, the host reads CFA_ERR_TIMEOUT, and the context stays usable.
On the host: the argument checks turn bad calls into status codes before anything launches."""

import time

import pytest
import torch

from candle_fused_attn import _abi


def test_selftest_rejects_bad_arguments_on_host():
    assert _abi.selftest_bounded_wait(None, 1000, 1, None) == _abi.CFA_ERR_NULL
    assert _abi.selftest_bounded_wait(1 << 20, 0, 1, None) == _abi.CFA_ERR_SHAPE
    assert _abi.selftest_bounded_wait(1 << 20, 1000, 0, None) == _abi.CFA_ERR_SHAPE
    assert _abi.selftest_bounded_wait((1 << 20) + 16, 1000, 1, None) == _abi.CFA_ERR_WORKSPACE


@pytest.mark.gpu
def test_bounded_wait_expires_and_reports(cuda):
    ws = torch.zeros(256, dtype=torch.uint8, device=cuda)
    stream = torch.cuda.current_stream().cuda_stream
    timeout_ns = 50_000_000  # 50 ms; the other blocks' own limit would be 5 s
    t0 = time.perf_counter()
    assert _abi.selftest_bounded_wait(ws.data_ptr(), timeout_ns, 8, stream) == _abi.CFA_OK
    assert _abi.bwd_status(ws.data_ptr(), stream) == _abi.CFA_ERR_TIMEOUT
    elapsed = time.perf_counter() - t0
    assert 0.04 < elapsed < 2.0, elapsed  # one expiry ended every waiter, nothing hung
    assert "expired" in _abi.strerror(_abi.CFA_ERR_TIMEOUT)
    # the expiry also reached the package's host flag if it is registered: consume it
    import candle_fused_attn as cfa
    try:
        cfa.check_status()
    except cfa.FusedAttentionError:
        pass
    # the context is still usable: a normal backward afterwards reports OK
    from oracle import oracle
    qkv, dout = oracle.seeded_inputs(2, 2, 100, 1)
    x = qkv.to(cuda).requires_grad_(True)
    o = cfa.fused_attention_qkv(x, 2, 0.125, False)
    o.backward(dout.to(cuda))
    torch.cuda.synchronize()
    assert torch.isfinite(x.grad).all()


@pytest.mark.gpu
def test_expiry_raises_through_the_public_api(cuda):
    """An expired bounded wait reaches the host flag the package registers (cfa_error_sink): the
    next public call raises FusedAttentionError without a synchronisation of its own, and so does
    check_status(); afterwards calls run normally again."""
    import candle_fused_attn as cfa
    from oracle import oracle
    qkv, dout = oracle.seeded_inputs(1, 2, 64, 3)
    x = qkv.to(cuda)
    cfa.fused_attention_qkv(x, 2, 0.125, False)  # registers the flag
    cfa.check_status()
    ws = torch.zeros(256, dtype=torch.uint8, device=cuda)
    stream = torch.cuda.current_stream().cuda_stream
    # a wait nothing can satisfy, in the same kernel routine the backward's dQ chain uses
    assert _abi.selftest_bounded_wait(ws.data_ptr(), 20_000_000, 2, stream) == _abi.CFA_OK
    torch.cuda.synchronize()  # the expiry has happened; the public call below does not sync
    with pytest.raises(cfa.FusedAttentionError, match="expired"):
        cfa.fused_attention_qkv(x, 2, 0.125, False)
    out = cfa.fused_attention_qkv(x, 2, 0.125, False)  # reported once, then clear
    assert _abi.selftest_bounded_wait(ws.data_ptr(), 20_000_000, 2, stream) == _abi.CFA_OK
    with pytest.raises(cfa.FusedAttentionError, match="expired"):
        cfa.check_status()
    cfa.check_status()
    assert torch.isfinite(out).all()
