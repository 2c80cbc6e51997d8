# SPDX-License-Identifier: MIT OR Apache-2.0
"""candle_fused_attn -- fused fp32 scaled-dot-product attention for B200 (sm_100a).

The public API of the candle-fused-attn crate (src/lib.rs), over torch tensors, on the C ABI of
include/cfa.h:

- `fused_attention_qkv(qkv, heads, scale, causal)` (src/lib.rs:110-125): the fused projection
  `[batch, seq, 3*heads*64]` -> merged output `[batch, seq, heads*64]`; its backward writes ONE
  gradient laid out like `qkv`.
- `fused_attention(q, k, v, scale, causal)` (src/lib.rs:143-161): `[batch, heads, seq, 64]` with
  any strides -> `[batch, heads, seq, 64]`, a transposed view of a dense `[batch, seq, heads, 64]`
  buffer (merge-heads ready).
- `CUDA_HEAD_DIM` (src/lib.rs:91): 64, the head dim of the reference's CUDA path; `HEAD_DIMS`:
  the head dims these kernels take, (32, 64, 128) -- 32 and 128 extend the reference's CUDA path
  (its ROADMAP.md "head_dim 32 and 128"; its CPU path takes any head dim).

Both read their operands in place when `head_dim` is contiguous and the offset and every other
stride are multiples of 4 floats, and copy them to a contiguous tensor first otherwise (the
reference's alignment gate, src/lib.rs:111-118, :165-178). The saved state between forward and
backward is the row log-sum-exp L `[batch, heads, seq]` (src/lib.rs:301-315); the backward
recomputes P from it.

Device only: the CUDA kernels are the product; the reference's CPU composed path lives in the
test oracle (oracle/), never here. A CPU tensor, a dtype other than float32, a head_dim not in
`HEAD_DIMS`, or a missing libcfa.so raise `FusedAttentionError` / `ImportError`.

Next to the path, the projection of the reference's training step (examples/tutorial.rs:103-118):
- `broadcast_matmul(x, w)`: candle's `Tensor::broadcast_matmul` as the step uses it, x [..., k] times
  w [k, n], differentiable in both (dx = dy w^T, dw = x^T dy), on the tensor-core GEMM of the C ABI
  (`cfa_matmul_f32`); `matmul(a, b)` is the 2-D product itself.

Failure detection: every device-side wait of the kernels is bounded. An expired wait (results
invalid) is written by the kernel into a page-locked host flag this module registers with the C
ABI (`cfa_error_sink`), so the next call of any function here raises `FusedAttentionError`
without synchronising; `check_status()` synchronises first and raises for the calls before it.
"""

from __future__ import annotations

import ctypes

import torch

from . import _abi

__all__ = [
    "check_status",
    "CUDA_HEAD_DIM",
    "HEAD_DIMS",
    "FusedAttentionError",
    "fused_attention",
    "fused_attention_qkv",
    "float4_aligned",
    "qkv_geometry",
    "attention_forward",
    "attention_backward",
    "matmul",
    "broadcast_matmul",
    "HostPipeline",
]

CUDA_HEAD_DIM = 64  # src/lib.rs:91
HEAD_DIMS = _abi.HEAD_DIMS  # (32, 64, 128)


def _check_head_dim(d: int) -> None:
    if d not in HEAD_DIMS:
        raise FusedAttentionError(
            f"fused_attention: the CUDA kernels take head_dim {CUDA_HEAD_DIM} "
            f"(and 32 or 128), got {d}")


class FusedAttentionError(RuntimeError):
    """The crate's `candle_core::Error::Msg` (messages prefixed `fused_attention:`)."""


# ---------------------------------------------------------------------------------------------
# Host-side geometry (src/lib.rs:165-220)
# ---------------------------------------------------------------------------------------------

def float4_aligned(t: torch.Tensor) -> bool:
    """src/lib.rs:165-168: offset and (batch, head, seq) strides multiples of 4, d contiguous."""
    st = t.stride()
    return (t.dim() == 4 and t.storage_offset() % 4 == 0 and st[3] == 1
            and st[0] % 4 == 0 and st[1] % 4 == 0 and st[2] % 4 == 0)


def _float4_rows(t: torch.Tensor) -> torch.Tensor:
    """src/lib.rs:172-178: `t` when float4-aligned, else a contiguous copy."""
    return t if float4_aligned(t) else t.contiguous()


def _bhs_strides(t: torch.Tensor, who: str = "fused_attention") -> tuple[int, int, int]:
    """src/lib.rs:181-188: (sb, sh, ss) of a [b, h, s, d] layout with d contiguous."""
    st = t.stride()
    if len(st) != 4 or st[3] != 1:
        raise FusedAttentionError(
            f"{who}: [b, h, s, d] with d contiguous expected, strides {list(st)}")
    return st[0], st[1], st[2]


def qkv_geometry(shape, stride, heads: int):
    """src/lib.rs:191-206: ((b, h, s, d), [sb, d, ss], [0, hd, 2hd]) of a qkv projection layout."""
    if len(shape) != 3:
        raise FusedAttentionError(f"fused_attention_qkv: rank-3 qkv expected, shape {list(shape)}")
    b, s, three_hd = shape
    if heads == 0 or three_hd % (3 * heads) != 0:
        raise FusedAttentionError(
            f"fused_attention_qkv: last dimension {three_hd} is not 3 x {heads} heads x head_dim")
    hd = three_hd // 3
    d = hd // heads
    if stride[2] != 1:
        raise FusedAttentionError(
            f"fused_attention_qkv: the last dimension must be contiguous, strides {list(stride)}")
    return (b, heads, s, d), (stride[0], d, stride[1]), (0, hd, 2 * hd)


def _check_shapes(q, k, v):
    """src/lib.rs:209-220: q, k, v share one [b, h, s, d] shape."""
    if q.dim() != 4 or k.shape != q.shape or v.shape != q.shape:
        raise FusedAttentionError(
            "fused_attention: q, k, v must share one [b, h, s, d] shape, got "
            f"{list(q.shape)} {list(k.shape)} {list(v.shape)}")
    return tuple(q.shape)


def _check_device(*ts: torch.Tensor, who: str) -> torch.device:
    dev = ts[0].device
    for t in ts:
        if t.dtype != torch.float32:
            raise FusedAttentionError(f"{who}: f32 only")
        if t.device.type != "cuda":
            raise FusedAttentionError(
                f"{who}: CUDA tensors required (the CPU composed path is the test oracle)")
        if t.device != dev:
            raise FusedAttentionError(f"{who}: q, k, v on different devices")
    return dev


def _aligned_grad(g: torch.Tensor) -> torch.Tensor:
    """src/lib.rs:370-380: the gradient itself when float4-aligned rows, else a contiguous copy."""
    st = g.stride()
    ok = (g.storage_offset() % 4 == 0 and st[-1] == 1
          and all(x == 1 or x % 4 == 0 for x in st))
    return g if ok else g.contiguous()


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


# ---------------------------------------------------------------------------------------------
# Failure detection: the host-visible error flag (cfa_error_sink)
# ---------------------------------------------------------------------------------------------

_sink_tensor: torch.Tensor | None = None


def _sink_flag() -> ctypes.c_int32:
    """The registered page-locked flag (created and registered on first use, with CUDA up)."""
    global _sink_tensor
    if _sink_tensor is None:
        t = torch.zeros(1, dtype=torch.int32).pin_memory()
        st = _abi.error_sink(t.data_ptr())
        if st != _abi.CFA_OK:
            raise FusedAttentionError(_abi.strerror(st))
        _sink_tensor = t
    return ctypes.c_int32.from_address(_sink_tensor.data_ptr())


def _raise_if_expired() -> None:
    """Raise (once) for a bounded wait that expired in a kernel launched earlier: the flag is read
    as it stands, with no synchronisation, so kernels still running are not covered."""
    flag = _sink_flag()
    code = flag.value
    if code != 0:
        flag.value = 0
        raise FusedAttentionError(_abi.strerror(code))


def check_status(device: torch.device | int | None = None) -> None:
    """Synchronise `device` (default: the current one) and raise `FusedAttentionError` if a bounded
    device-side wait of any earlier call expired (their results are then invalid)."""
    torch.cuda.synchronize(device)
    _raise_if_expired()


# ---------------------------------------------------------------------------------------------
# Launch wrappers (the src/cuda.rs role, over the C ABI)
# ---------------------------------------------------------------------------------------------

def attention_forward(q_ptr, qs, k_ptr, ks, v_ptr, vs, dims, scale, causal, device):
    """One forward over device operands given as (pointer, (sb, sh, ss)): returns (O [b, s, h, d],
    L [b, h, s]) as fresh tensors (the role of src/cuda.rs:140-185)."""
    b, h, s, d = dims
    _check_head_dim(d)
    _raise_if_expired()
    o = torch.empty((b, s, h, d), dtype=torch.float32, device=device)
    lse = torch.empty((b, h, s), dtype=torch.float32, device=device)
    fwd = _abi.fwd if d == CUDA_HEAD_DIM else _abi.fwd_hd
    with torch.cuda.device(device):
        st = fwd(q_ptr, qs, k_ptr, ks, v_ptr, vs, o.data_ptr(), lse.data_ptr(),
                 b, h, s, d, float(scale), causal, _stream(device))
    if st != _abi.CFA_OK:
        raise FusedAttentionError(_abi.strerror(st))
    return o, lse


def attention_backward(q_ptr, qs, k_ptr, ks, v_ptr, vs, o, lse, do_ptr, dos, dims, scale, causal,
                       device, check_status: bool = False):
    """One backward: dqkv [b, s, 3, h, d] (the role of src/cuda.rs:190-260). The scratch comes
    from torch's caching allocator; `check_status` synchronises and reads the device error flag."""
    b, h, s, d = dims
    _check_head_dim(d)
    _raise_if_expired()
    if not (o.is_contiguous() and lse.is_contiguous()):
        raise FusedAttentionError("fused_attention: O and L must be contiguous")
    dqkv = torch.empty((b, s, 3, h, d), dtype=torch.float32, device=device)
    # The larger workspace enables the no-wait dQ path (same bits); torch's caching allocator
    # recycles it across steps.
    ws_bytes = _abi.bwd_workspace_bytes_fast_hd(b, h, s, d)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=device)
    bwd = _abi.bwd if d == CUDA_HEAD_DIM else _abi.bwd_hd
    with torch.cuda.device(device):
        stream = _stream(device)
        st = bwd(q_ptr, qs, k_ptr, ks, v_ptr, vs, o.data_ptr(), lse.data_ptr(), do_ptr, dos,
                 dqkv.data_ptr(), ws.data_ptr(), ws_bytes, b, h, s, d, float(scale), causal,
                 stream)
        if st == _abi.CFA_OK and check_status:
            st = _abi.bwd_status(ws.data_ptr(), stream)
    if st != _abi.CFA_OK:
        raise FusedAttentionError(_abi.strerror(st))
    return dqkv


# ---------------------------------------------------------------------------------------------
# The two custom ops (src/lib.rs:383-590) as autograd functions
# ---------------------------------------------------------------------------------------------

class _FusedAttention(torch.autograd.Function):
    """CustomOp3 `FusedAttention` (src/lib.rs:383-491): [b, h, s, d] in, [b, s, h, d] out."""

    @staticmethod
    def forward(ctx, q, k, v, scale, causal):
        dims = _check_shapes(q, k, v)
        dev = _check_device(q, k, v, who="fused_attention")
        if not all(float4_aligned(t) for t in (q, k, v)):
            raise FusedAttentionError("fused_attention: rows must be 16-byte aligned")
        o, lse = attention_forward(q.data_ptr(), _bhs_strides(q), k.data_ptr(), _bhs_strides(k),
                                   v.data_ptr(), _bhs_strides(v), dims, scale, causal, dev)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.scale, ctx.causal, ctx.dims = scale, causal, dims
        return o

    @staticmethod
    def backward(ctx, grad):
        q, k, v, o, lse = ctx.saved_tensors
        grad = _aligned_grad(grad)
        gb, gs, gh, _ = grad.stride()
        dqkv = attention_backward(
            q.data_ptr(), _bhs_strides(q), k.data_ptr(), _bhs_strides(k), v.data_ptr(),
            _bhs_strides(v), o, lse, grad.data_ptr(), (gb, gh, gs), ctx.dims, ctx.scale,
            ctx.causal, q.device)
        part = lambda i: dqkv[:, :, i].transpose(1, 2)  # noqa: E731  (src/lib.rs:484)
        return part(0), part(1), part(2), None, None


class _FusedAttentionQkv(torch.autograd.Function):
    """CustomOp1 `FusedAttentionQkv` (src/lib.rs:494-590): qkv in, merged [b, s, h*d] out."""

    @staticmethod
    def forward(ctx, qkv, heads, scale, causal):
        _check_device(qkv, who="fused_attention_qkv")
        dims, strides, offs = qkv_geometry(tuple(qkv.shape), qkv.stride(), heads)
        if qkv.storage_offset() % 4 != 0 or any(x % 4 != 0 for x in strides):
            raise FusedAttentionError("fused_attention_qkv: rows must be 16-byte aligned")
        base = qkv.data_ptr()
        o, lse = attention_forward(base + 4 * offs[0], strides, base + 4 * offs[1], strides,
                                   base + 4 * offs[2], strides, dims, scale, causal, qkv.device)
        ctx.save_for_backward(qkv, o, lse)
        ctx.heads, ctx.scale, ctx.causal = heads, scale, causal
        b, h, s, d = dims
        return o.view(b, s, h * d)

    @staticmethod
    def backward(ctx, grad):
        qkv, o, lse = ctx.saved_tensors
        grad = _aligned_grad(grad)
        dims, strides, offs = qkv_geometry(tuple(qkv.shape), qkv.stride(), ctx.heads)
        b, h, s, d = dims
        if grad.dim() != 3:
            raise FusedAttentionError("fused_attention_qkv: rank-3 gradient expected")
        gb, gs, _ = grad.stride()
        base = qkv.data_ptr()
        dqkv = attention_backward(
            base + 4 * offs[0], strides, base + 4 * offs[1], strides, base + 4 * offs[2], strides,
            o, lse, grad.data_ptr(), (gb, d, gs), dims, ctx.scale, ctx.causal, qkv.device)
        return dqkv.view(b, s, 3 * h * d), None, None, None


def fused_attention_qkv(qkv: torch.Tensor, heads: int, scale: float, causal: bool) -> torch.Tensor:
    """src/lib.rs:110-125. `qkv` [batch, seq, 3*heads*d] f32 on CUDA -> [batch, seq, heads*d], d in
    HEAD_DIMS."""
    st = qkv.stride()
    aligned = (qkv.dim() == 3 and qkv.storage_offset() % 4 == 0 and st[2] == 1
               and st[0] % 4 == 0 and st[1] % 4 == 0)
    if not aligned:
        qkv = qkv.contiguous()
    return _FusedAttentionQkv.apply(qkv, int(heads), float(scale), bool(causal))


def fused_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
                    causal: bool) -> torch.Tensor:
    """src/lib.rs:143-161. q, k, v [batch, heads, seq, d] f32 on CUDA (d in HEAD_DIMS), any
    strides -> [batch, heads, seq, d] (a transposed view of a dense [batch, seq, heads, d] buffer)."""
    q, k, v = _float4_rows(q), _float4_rows(k), _float4_rows(v)
    return _FusedAttention.apply(q, k, v, float(scale), bool(causal)).transpose(1, 2)


# ---------------------------------------------------------------------------------------------
# The projection next to the path (examples/tutorial.rs:103-118): candle's broadcast_matmul
# ---------------------------------------------------------------------------------------------

def matmul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """C = a b for 2-D f32 CUDA tensors (a [m, k], b [k, n], any strides: transposed and strided
    views are read in place) on the tensor-core GEMM: three bf16 parts per operand, fp32 sums,
    bit-identical across reruns."""
    dev = _check_device(a, b, who="matmul")
    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[0]:
        raise FusedAttentionError(
            f"matmul: shape mismatch {tuple(a.shape)} x {tuple(b.shape)}")
    _raise_if_expired()
    m, k = a.shape
    n = b.shape[1]
    ldc = (n + 3) // 4 * 4  # 16-byte rows
    c = torch.empty((m, ldc), dtype=torch.float32, device=dev)
    ws_bytes = _abi.matmul_workspace_bytes(m, n, k)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes else None
    with torch.cuda.device(dev):
        st = _abi.matmul(a.data_ptr(), a.stride(0), a.stride(1), b.data_ptr(), b.stride(0),
                         b.stride(1), c.data_ptr(), ldc, m, n, k,
                         ws.data_ptr() if ws is not None else None, ws_bytes, _stream(dev))
    if st != _abi.CFA_OK:
        raise FusedAttentionError(f"matmul: {_abi.strerror(st)}")
    return c if ldc == n else c[:, :n]


class _Matmul(torch.autograd.Function):
    """a [m, k] b [k, n]; the backward's two products run on the same kernel, reading the saved
    operands transposed in place: da = dc b^T, db = a^T dc."""

    @staticmethod
    def forward(ctx, a, b):
        ctx.save_for_backward(a, b)
        return matmul(a, b)

    @staticmethod
    def backward(ctx, grad):
        a, b = ctx.saved_tensors
        da = matmul(grad, b.t()) if ctx.needs_input_grad[0] else None
        db = matmul(a.t(), grad) if ctx.needs_input_grad[1] else None
        return da, db


def broadcast_matmul(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """candle's `Tensor::broadcast_matmul(x, w)` as the reference's training step uses it
    (examples/tutorial.rs:110): x [..., k] times a 2-D w [k, n] -> [..., n], f32 on CUDA, with
    gradients for both (the step trains w: tutorial.rs:113-117)."""
    if w.dim() != 2 or x.dim() < 1 or x.shape[-1] != w.shape[0]:
        raise FusedAttentionError(
            f"broadcast_matmul: shape mismatch {tuple(x.shape)} x {tuple(w.shape)}")
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    return _Matmul.apply(x2, w).reshape(*lead, w.shape[1])


from .host_pipeline import HostPipeline  # noqa: E402  (uses _abi; public host-buffer API)
