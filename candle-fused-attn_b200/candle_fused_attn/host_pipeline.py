# SPDX-License-Identifier: MIT OR Apache-2.0
"""Forward + backward for callers whose tensors live in host memory.

A caller holding the fused projection and dO in (pinned) host memory, and wanting O and dqkv
back in host memory, pays two PCIe transfers per step that dwarf the kernels (canvas: 94 MB in,
94 MB out, against ~0.6 ms of compute). `HostPipeline` streams the batch through the GPU in
chunks on three CUDA streams -- host->device copies, kernels, device->host copies -- with
`slots` device buffers in rotation, so both copy directions and the kernels overlap. The op is
batch-separable and its kernels are independent of the batch size, so the chunked results are
bit-identical to one whole-batch call (tests/test_host_pipeline_gpu.py).

Kernels run through the C ABI (include/cfa.h) exactly as `fused_attention_qkv` and its backward
do; the buffers are allocated once, at construction.
"""

from __future__ import annotations

import torch

from . import _abi
from .sharding import shard_range

__all__ = ["HostPipeline"]


class HostPipeline:
    """fused_attention_qkv forward + backward from host buffers to host buffers.

    batch, heads, seq: the problem (qkv [batch, seq, 3*heads*64], dO [batch, seq, heads*64]).
    chunks: batch chunks per step; slots: device buffer sets, rotating over chunks and steps
    (>= 2 to overlap: the H2D copy of one chunk or step runs during the kernels and the D2H copy of
    the previous one). Measured on a B200 at the canvas shape (b64 h6 s240), steps back to back:
    1 chunk x 2 slots 2.11-2.15 ms per step, 2 chunks 2.16 ms, 4 chunks 2.27-2.46 ms, against a
    1.92-1.95 ms floor for moving 94 MB each way over PCIe at once: once consecutive steps overlap,
    splitting a step only adds per-chunk overhead and smaller, less efficient kernel launches.
    """

    def __init__(self, batch: int, heads: int, seq: int, scale: float, causal: bool,
                 device: torch.device, chunks: int = 1, slots: int = 2):
        self.b, self.h, self.s = batch, heads, seq
        self.scale, self.causal = float(scale), bool(causal)
        self.dev = torch.device(device)
        self.chunks = max(1, min(chunks, batch))
        self.ranges = [shard_range(batch, self.chunks, c) for c in range(self.chunks)]
        cb = max(hi - lo for lo, hi in self.ranges)
        hd = heads * 64
        n = max(1, slots)
        f32 = dict(dtype=torch.float32, device=self.dev)
        self.qkv = [torch.empty(cb, seq, 3 * hd, **f32) for _ in range(n)]
        self.dout = [torch.empty(cb, seq, hd, **f32) for _ in range(n)]
        self.o = [torch.empty(cb, seq, heads, 64, **f32) for _ in range(n)]
        self.lse = [torch.empty(cb, heads, seq, **f32) for _ in range(n)]
        self.dqkv = [torch.empty(cb, seq, 3, heads, 64, **f32) for _ in range(n)]
        self.ws_bytes = _abi.bwd_workspace_bytes_fast(cb, heads, seq)
        self.ws = [torch.empty(self.ws_bytes, dtype=torch.uint8, device=self.dev)
                   for _ in range(n)]
        self.h2d = torch.cuda.Stream(self.dev)
        self.comp = torch.cuda.Stream(self.dev)
        self.d2h = torch.cuda.Stream(self.dev)
        self.loaded = [torch.cuda.Event() for _ in range(n)]
        self.computed = [torch.cuda.Event() for _ in range(n)]
        self.unloaded = [torch.cuda.Event() for _ in range(n)]
        self.used = [False] * n
        self.next_slot = 0  # slots rotate across chunks and across steps

    def _kernels(self, slot: int, b: int) -> None:
        from . import _raise_if_expired  # an earlier call's expired bounded wait raises here
        _raise_if_expired()
        h, s = self.h, self.s
        x, g = self.qkv[slot], self.dout[slot]
        st = (x.stride(0), 64, x.stride(1))
        gst = (g.stride(0), 64, g.stride(1))
        base = x.data_ptr()
        q, k, v = base, base + 4 * h * 64, base + 8 * h * 64
        stream = self.comp.cuda_stream
        rc = _abi.fwd(q, st, k, st, v, st, self.o[slot].data_ptr(), self.lse[slot].data_ptr(),
                      b, h, s, 64, self.scale, self.causal, stream)
        if rc == _abi.CFA_OK:
            rc = _abi.bwd(q, st, k, st, v, st, self.o[slot].data_ptr(),
                          self.lse[slot].data_ptr(), g.data_ptr(), gst,
                          self.dqkv[slot].data_ptr(), self.ws[slot].data_ptr(), self.ws_bytes,
                          b, h, s, 64, self.scale, self.causal, stream)
        if rc != _abi.CFA_OK:
            raise RuntimeError(_abi.strerror(rc))

    def step(self, qkv: torch.Tensor, dout: torch.Tensor, o_out: torch.Tensor,
             dqkv_out: torch.Tensor) -> None:
        """Queue one forward + backward: qkv [b, s, 3hd] and dout [b, s, hd] (host, pinned) in,
        O [b, s, hd] and dqkv [b, s, 3hd] (host, pinned) out. Asynchronous; `synchronize()`
        waits for the outputs."""
        n = len(self.qkv)
        hd = self.h * 64
        for lo, hi in self.ranges:
            slot, b = self.next_slot, hi - lo
            self.next_slot = (slot + 1) % n
            with torch.cuda.stream(self.h2d):
                if self.used[slot]:
                    self.h2d.wait_event(self.computed[slot])  # inputs of the slot consumed
                self.qkv[slot][:b].copy_(qkv[lo:hi], non_blocking=True)
                self.dout[slot][:b].copy_(dout[lo:hi], non_blocking=True)
                self.loaded[slot].record(self.h2d)
            self.comp.wait_event(self.loaded[slot])
            if self.used[slot]:
                self.comp.wait_event(self.unloaded[slot])  # outputs of the slot copied out
            self._kernels(slot, b)
            self.computed[slot].record(self.comp)
            with torch.cuda.stream(self.d2h):
                self.d2h.wait_event(self.computed[slot])
                o_out[lo:hi].copy_(self.o[slot][:b].view(b, self.s, hd), non_blocking=True)
                dqkv_out[lo:hi].copy_(self.dqkv[slot][:b].view(b, self.s, 3 * hd),
                                      non_blocking=True)
                self.unloaded[slot].record(self.d2h)
            self.used[slot] = True

    def synchronize(self) -> None:
        self.d2h.synchronize()

    def record_done(self, event: torch.cuda.Event) -> None:
        """Record `event` on the device->host stream (after every queued output copy)."""
        event.record(self.d2h)
