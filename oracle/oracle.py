# SPDX-License-Identifier: MIT OR Apache-2.0
"""TEST INFRASTRUCTURE -- the CPU oracle.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may import this module; the
product (candle_fused_attn, libcfa.so) never does.

Two independent restatements of the reference's CPU semantics:

- `forward` / `backward`: ctypes over liboracle.so (oracle/oracle.cpp), the C++ restatement of
  composed_forward / composed_backward (src/lib.rs:241-299) with gather_cpu (src/lib.rs:223-238)
  and the output layouts (src/lib.rs:318-323, :581-588), in fp32 or fp64, multithreaded over
  (batch, head) slices.
- `matmul`: the training step's projection (examples/tutorial.rs:110, :113), C = A B with every
  output's products summed in k order by fused multiply-adds, fp32 or fp64.
- `composed_autograd`: the composed attention differentiated by torch autograd on CPU, the role
  of the reference test's own independent reference (tests/parity.rs:54-75, :119-123), any dtype.

Parity pinning: the reference's CPU path (candle 0.11 / gemm) cannot be built here (no cargo).
The C++ restatement is pinned by tolerance against outputs of the reference's own CUDA kernel,
stored as fixtures in tests/golden/ (made by tests/golden/make_golden.py on a B200), at the
reference's CUDA-vs-CPU band (tests/parity.rs:210-221).
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

_lib = None
_i64 = ctypes.c_int64
_p = ctypes.c_void_p
_s3 = ctypes.POINTER(ctypes.c_int64)


def load():
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.is_file():
        raise ImportError(f"oracle: {LIB_PATH} missing; run `make -C oracle`")
    lib = ctypes.CDLL(str(LIB_PATH))
    fwd_args = [_p, _s3, _p, _s3, _p, _s3, _i64, _i64, _i64, _i64, ctypes.c_double, ctypes.c_int,
                _p, _p, ctypes.c_int, _i64, _i64]
    bwd_args = [_p, _s3, _p, _s3, _p, _s3, _p, _p, _p, _s3, _i64, _i64, _i64, _i64,
                ctypes.c_double, ctypes.c_int, _p, ctypes.c_int, _i64, _i64]
    for name, args in (("oracle_fwd_f32", fwd_args), ("oracle_fwd_f64", fwd_args),
                       ("oracle_bwd_f32", bwd_args), ("oracle_bwd_f64", bwd_args)):
        fn = getattr(lib, name)
        fn.restype = None
        fn.argtypes = args
    for name in ("oracle_matmul_f32", "oracle_matmul_f64"):
        fn = getattr(lib, name)
        fn.restype = None
        fn.argtypes = [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _i64, ctypes.c_int]
    lib.oracle_max_threads.restype = ctypes.c_int
    _lib = lib
    return lib


def max_threads() -> int:
    return int(load().oracle_max_threads())


def _s(t: torch.Tensor):
    """(pointer, (sb, sh, ss)) of a CPU fp32 [b, h, s, d] operand with d contiguous."""
    if t.device.type != "cpu" or t.dtype != torch.float32:
        raise TypeError("oracle: CPU float32 operands expected")
    st = t.stride()
    if t.dim() != 4 or st[3] != 1:
        raise ValueError("oracle: [b, h, s, d] with d contiguous expected")
    return t.data_ptr(), (ctypes.c_int64 * 3)(st[0], st[1], st[2])


def forward(q, k, v, scale: float, causal: bool, dtype=torch.float32, threads: int = 0,
            bh_range=None):
    """composed_forward on (batch, head) slices: (O [b, s, h, d], L [b, h, s]) in `dtype`."""
    b, h, s, d = q.shape
    o = torch.zeros((b, s, h, d), dtype=dtype)
    lse = torch.zeros((b, h, s), dtype=dtype)
    lo, hi = bh_range if bh_range is not None else (0, b * h)
    fn = load().oracle_fwd_f32 if dtype == torch.float32 else load().oracle_fwd_f64
    (qp, qs), (kp, ks), (vp, vs) = _s(q), _s(k), _s(v)
    fn(qp, qs, kp, ks, vp, vs, b, h, s, d, float(scale), int(bool(causal)), o.data_ptr(),
       lse.data_ptr(), int(threads), lo, hi)
    return o, lse


def backward(q, k, v, o, lse, dout, scale: float, causal: bool, threads: int = 0, bh_range=None):
    """composed_backward on (batch, head) slices: dqkv [b, s, 3, h, d], in the dtype of `o`."""
    b, h, s, d = q.shape
    dtype = o.dtype
    o = o.contiguous()
    lse = lse.contiguous()
    dqkv = torch.zeros((b, s, 3, h, d), dtype=dtype)
    lo, hi = bh_range if bh_range is not None else (0, b * h)
    fn = load().oracle_bwd_f32 if dtype == torch.float32 else load().oracle_bwd_f64
    (qp, qs), (kp, ks), (vp, vs), (gp, gs) = _s(q), _s(k), _s(v), _s(dout)
    fn(qp, qs, kp, ks, vp, vs, o.data_ptr(), lse.data_ptr(), gp, gs, b, h, s, d, float(scale),
       int(bool(causal)), dqkv.data_ptr(), int(threads), lo, hi)
    return dqkv


def qkv_views(qkv: torch.Tensor, heads: int):
    """The head-split views of a [b, s, 3*h*d] projection (tests/parity.rs:40-51): q, k, v
    [b, h, s, d], non-contiguous."""
    b, s, three_hd = qkv.shape
    hd = three_hd // 3
    d = hd // heads

    def split(i):
        return qkv.narrow(2, i * hd, hd).reshape(b, s, heads, d).transpose(1, 2)

    return split(0), split(1), split(2)


def heads_view(x: torch.Tensor, heads: int):
    """[b, s, h*d] -> [b, h, s, d] view."""
    b, s, hd = x.shape
    return x.reshape(b, s, heads, hd // heads).transpose(1, 2)


def qkv_forward_backward(qkv, dout, heads, scale, causal, dtype=torch.float32, threads=0):
    """The fused-qkv op's oracle: (O [b, s, h*d], L [b, h, s], dqkv [b, s, 3*h*d]) from the
    projection and dO [b, s, h*d], both fp32 on CPU."""
    q, k, v = qkv_views(qkv, heads)
    o, lse = forward(q, k, v, scale, causal, dtype=dtype, threads=threads)
    g = heads_view(dout, heads)
    dqkv = backward(q, k, v, o, lse, g, scale, causal, threads=threads)
    b, s, _ = qkv.shape
    return o.reshape(b, s, -1), lse, dqkv.reshape(b, s, -1)


def composed_autograd(qkv, dout, heads, scale, causal, dtype=torch.float64):
    """Independent check: the composed attention (tests/parity.rs:54-75) differentiated by torch
    autograd with the loss head sum(out * dout) (tests/parity.rs:119-123). Returns (O, dqkv)."""
    x = qkv.detach().to(dtype).requires_grad_(True)
    q, k, v = qkv_views(x, heads)
    b, s, _ = qkv.shape
    sc = (q @ k.transpose(-2, -1)) * scale
    if causal:
        mask = torch.ones(s, s, dtype=torch.bool).triu(1)
        sc = sc.masked_fill(mask, float("-inf"))
    p = torch.softmax(sc, dim=-1)
    o = (p @ v).transpose(1, 2).reshape(b, s, -1)
    (o * dout.to(dtype)).sum().backward()
    return o.detach(), x.grad.detach()


def closed_form_inputs(b, s, h, d):
    """tests/parity.rs:126-138: x_i = sin(i * 0.618034) * 1.5 (the projection) and
    w_i = cos(i * 0.414213) (the loss weights = dO), computed in f32 as the Rust test does."""
    i = torch.arange(b * s * 3 * h * d, dtype=torch.float32)
    x = torch.sin(i * torch.tensor(0.618034, dtype=torch.float32)) * 1.5
    j = torch.arange(b * s * h * d, dtype=torch.float32)
    w = torch.cos(j * torch.tensor(0.414213, dtype=torch.float32))
    return x.reshape(b, s, 3 * h * d), w.reshape(b, s, h * d)


def seeded_inputs(b, h, s, seed, qkv_scale=1.0, d=64):
    """bench/compare.py:496-503: torch.Generator seeded, qkv [b, s, 3*h*d] then dout [b, s, h*d],
    N(0, 1), drawn on the CPU; qkv optionally scaled (the canvas config uses 0.5). The reference
    draws head dim 64; d is this build's extension to the head dims 32 and 128."""
    g = torch.Generator().manual_seed(seed)
    hd = h * d
    qkv = torch.randn(b, s, 3 * hd, generator=g)
    dout = torch.randn(b, s, hd, generator=g)
    if qkv_scale != 1.0:
        qkv = qkv * qkv_scale
    return qkv, dout


def normwise(got: torch.Tensor, ref: torch.Tensor) -> float:
    """Normwise relative error ||got - ref||_F / ||ref||_F in fp64 (bench/compare.py:525-527)."""
    g, r = got.double(), ref.double()
    return float((g - r).norm() / r.norm())


def env_threads() -> int:
    return int(os.environ.get("ORACLE_THREADS", "0"))


def matmul(a: torch.Tensor, b: torch.Tensor, dtype=torch.float32, threads: int = 0) -> torch.Tensor:
    """C = a b for 2-D fp32 CPU tensors (any strides), fp32 (`oracle_matmul_f32`) or fp64 output."""
    assert a.dtype == torch.float32 and b.dtype == torch.float32 and a.device.type == "cpu"
    assert a.dim() == 2 and b.dim() == 2 and a.shape[1] == b.shape[0]
    m, k = a.shape
    n = b.shape[1]
    c = torch.empty((m, n), dtype=dtype)
    fn = load().oracle_matmul_f32 if dtype == torch.float32 else load().oracle_matmul_f64
    fn(a.data_ptr(), a.stride(0), a.stride(1), b.data_ptr(), b.stride(0), b.stride(1),
       c.data_ptr(), m, n, k, threads or env_threads())
    return c
