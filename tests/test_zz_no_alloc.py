# SPDX-License-Identifier: MIT OR Apache-2.0
"""cfa_bwd_f32_d64_noalloc: the backward for callers that cannot call cudaMalloc.

Some callers cannot allocate device memory (under a host framework that owns every device byte, in
a real-time loop that cannot risk an allocation, behind an FFI that passes only given tensors), yet
they can hand over inputs and outputs. This entry point takes no workspace: its scratch is a static
device array in the library (4 MiB per GPU). These tests call it through the C ABI and compare it with the ordinary
backward (cfa_bwd_f32_d64 with a caller-allocated workspace): the same kernels on the same inputs,
so the results must agree bit for bit (well inside the 5e-6 band the other tests use), on two calls
in a row -- the second call reuses the array the first one left behind.

This file is collected last on purpose (pytest orders files by name), so a run that stops at the
first failure has run every other test before it."""

import pytest
import torch

from candle_fused_attn import _abi
from oracle import oracle

pytestmark = pytest.mark.gpu

BAND = 5e-6  # the max-abs band of the parity tests (tests/parity.rs:218)


def _setup(b, h, s, causal, seed, dev):
    qkv, dout = oracle.seeded_inputs(b, h, s, seed)
    x, g = qkv.to(dev), dout.to(dev)
    st = (x.stride(0), 64, x.stride(1))
    gst = (g.stride(0), 64, g.stride(1))
    base = x.data_ptr()
    ptrs = (base, base + 4 * h * 64, base + 8 * h * 64)
    o = torch.empty(b, s, h, 64, device=dev)
    lse = torch.empty(b, h, s, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    rc = _abi.fwd(ptrs[0], st, ptrs[1], st, ptrs[2], st, o.data_ptr(), lse.data_ptr(), b, h, s, 64,
                  0.125, causal, stream)
    assert rc == _abi.CFA_OK
    return x, g, st, gst, ptrs, o, lse, stream


def _reference_backward(b, h, s, causal, x, g, st, gst, ptrs, o, lse, stream, dev):
    # A workspace of the static scratch's size: the same kernel choice (the dQ partials, and with
    # them the tensor-core backward at s <= 1024, when they fit).
    nbytes = max(_abi.bwd_workspace_bytes(b, h, s), _abi.NOALLOC_SCRATCH_BYTES)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    dqkv = torch.empty(b, s, 3, h, 64, device=dev)
    rc = _abi.bwd(ptrs[0], st, ptrs[1], st, ptrs[2], st, o.data_ptr(), lse.data_ptr(),
                  g.data_ptr(), gst, dqkv.data_ptr(), ws.data_ptr(), nbytes, b, h, s, 64, 0.125,
                  causal, stream)
    assert rc == _abi.CFA_OK
    assert _abi.bwd_status(ws.data_ptr(), stream) == _abi.CFA_OK
    return dqkv


def _noalloc_backward(b, h, s, causal, g, st, gst, ptrs, o, lse, stream, dev):
    dqkv = torch.full((b, s, 3, h, 64), float("nan"), device=dev)
    rc = _abi.bwd_noalloc(ptrs[0], st, ptrs[1], st, ptrs[2], st, o.data_ptr(), lse.data_ptr(),
                          g.data_ptr(), gst, dqkv.data_ptr(), b, h, s, 64, 0.125, causal, stream)
    assert rc == _abi.CFA_OK, _abi.strerror(rc)
    torch.cuda.synchronize()
    return dqkv


# (3, 2, 150) and (2, 3, 257) fit their dQ partials into the static scratch (the no-wait dQ path);
# (64, 6, 240) and (32, 6, 240, causal) do not, and run the key-block turn chain through it.
@pytest.mark.parametrize("shape,causal", [((3, 2, 150), False), ((2, 3, 257), True),
                                          ((64, 6, 240), False), ((32, 6, 240), True)])
def test_noalloc_matches_workspace_backward_twice(cuda, shape, causal):
    b, h, s = shape
    x, g, st, gst, ptrs, o, lse, stream = _setup(b, h, s, causal, 5, cuda)
    want = _reference_backward(b, h, s, causal, x, g, st, gst, ptrs, o, lse, stream, cuda)
    for call in range(2):
        got = _noalloc_backward(b, h, s, causal, g, st, gst, ptrs, o, lse, stream, cuda)
        assert _abi.bwd_noalloc_status(stream) == _abi.CFA_OK, f"call {call}"
        assert torch.isfinite(got).all(), f"call {call}"
        assert (got - want).abs().max().item() < BAND, f"call {call}"
        assert torch.equal(got.view(torch.int32), want.view(torch.int32)), f"call {call}"


def test_noalloc_rejects_problems_past_the_static_scratch(cuda):
    b, h, s = 1, 1, 2 << 20  # D alone needs 8 MiB > 4 MiB
    assert _abi.bwd_workspace_bytes(b, h, s) > _abi.NOALLOC_SCRATCH_BYTES
    fake = 1 << 20
    s3 = (s * 192, 64, 192)
    rc = _abi.bwd_noalloc(fake, s3, fake, s3, fake, s3, fake, fake, fake, s3, fake, b, h, s, 64,
                          0.125, 0, None)
    assert rc == _abi.CFA_ERR_WORKSPACE
    # the other argument errors keep their own codes
    assert _abi.bwd_noalloc(fake, s3, fake, s3, fake, s3, fake, fake, fake, s3, fake, b, h, s, 32,
                            0.125, 0, None) == _abi.CFA_ERR_HEAD_DIM
    assert _abi.bwd_noalloc(None, s3, fake, s3, fake, s3, fake, fake, fake, s3, fake, 1, 1, 64, 64,
                            0.125, 0, None) == _abi.CFA_ERR_NULL
