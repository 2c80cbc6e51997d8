# SPDX-License-Identifier: MIT OR Apache-2.0
"""Test helper: one forward + backward of a fused projection through the C ABI with an explicit
head-dim-64 kernel pair -- "tc" (cfa_fwd_f32_d64 / cfa_bwd_f32_d64, the tensor-core pair) or
"ffma" (cfa_fwd_f32_d64_ffma / cfa_bwd_f32_d64_ffma, the CUDA-core pair)."""

from __future__ import annotations

import torch

from candle_fused_attn import _abi


def run_pair(pair: str, qkv: torch.Tensor, dout: torch.Tensor | None, h: int, scale: float,
             causal: bool, dev, fast: bool = True):
    """qkv [b, s, 3 h 64], dout [b, s, h 64] (CPU or device) -> (O [b, s, h 64], L [b, h, s],
    dqkv [b, s, 3 h 64] or None), device tensors. `fast`: the workspace with the dQ partials."""
    fwd = {"tc": _abi.fwd, "ffma": _abi.fwd_ffma}[pair]
    bwd = {"tc": _abi.bwd, "ffma": _abi.bwd_ffma}[pair]
    x = qkv.to(dev).contiguous()
    b, s, _ = x.shape
    st = (x.stride(0), 64, x.stride(1))
    base = x.data_ptr()
    ptrs = (base, base + 4 * h * 64, base + 8 * h * 64)
    o = torch.empty(b, s, h, 64, device=dev)
    lse = torch.empty(b, h, s, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    _abi.check(fwd(ptrs[0], st, ptrs[1], st, ptrs[2], st, o.data_ptr(), lse.data_ptr(), b, h, s,
                   64, scale, causal, stream), f"{pair} forward")
    if dout is None:
        return o.reshape(b, s, h * 64), lse, None
    g = dout.to(dev).contiguous()
    gst = (g.stride(0), 64, g.stride(1))
    nbytes = (_abi.bwd_workspace_bytes_fast if fast else _abi.bwd_workspace_bytes)(b, h, s)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    dqkv = torch.empty(b, s, 3, h, 64, device=dev)
    _abi.check(bwd(ptrs[0], st, ptrs[1], st, ptrs[2], st, o.data_ptr(), lse.data_ptr(),
                   g.data_ptr(), gst, dqkv.data_ptr(), ws.data_ptr(), nbytes, b, h, s, 64, scale,
                   causal, stream), f"{pair} backward")
    _abi.check(_abi.bwd_status(ws.data_ptr(), stream), f"{pair} backward status")
    return o.reshape(b, s, h * 64), lse, dqkv.reshape(b, s, 3 * h * 64)
