# SPDX-License-Identifier: MIT OR Apache-2.0
"""ctypes binding of baseline/_ref/libfattn_ref.so: the reference's own kernels
(kernels/fused_attn.cu, compiled from source for sm_100a) launched as src/cuda.rs launches them.

Used as the same-GPU speed bar (bench.py) and as a second check in tests/. Not part of the
product path."""

from __future__ import annotations

import ctypes
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_ref" / "libfattn_ref.so"
_lib = None


def available() -> bool:
    return LIB_PATH.is_file()


def load():
    global _lib
    if _lib is None:
        if not LIB_PATH.is_file():
            raise ImportError(f"{LIB_PATH} missing: `make -C baseline` where the reference tree is")
        lib = ctypes.CDLL(str(LIB_PATH))
        p, i, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
        s3 = ctypes.POINTER(ctypes.c_int64)
        lib.ref_fwd.restype = i
        lib.ref_fwd.argtypes = [p, p, p, p, p, i, i, i, f, i, s3, s3, s3, p]
        lib.ref_bwd.restype = i
        lib.ref_bwd.argtypes = [p, p, p, p, p, p, p, p, i, i, i, f, i, s3, s3, s3, s3, p]
        lib.ref_bwd_workspace_bytes.restype = ctypes.c_size_t
        lib.ref_bwd_workspace_bytes.argtypes = [i, i, i]
        _lib = lib
    return _lib


def _s3(st):
    return (ctypes.c_int64 * 3)(*st)


class RefQkv:
    """The reference kernels on a fused qkv projection [b, s, 3*h*64] (device, fp32), with buffers
    allocated once (outside any timed region) like cudarc's allocations in src/cuda.rs."""

    def __init__(self, qkv: torch.Tensor, heads: int, scale: float, causal: bool):
        b, s, three_hd = qkv.shape
        self.b, self.h, self.s = b, heads, s
        self.hd = three_hd // 3
        self.qkv, self.scale, self.causal = qkv, float(scale), int(bool(causal))
        self.st = _s3((qkv.stride(0), 64, qkv.stride(1)))
        dev = qkv.device
        self.o = torch.empty(b, s, heads * 64, device=dev)
        self.lse = torch.empty(b, heads, s, device=dev)
        self.dqkv = torch.empty(b, s, 3 * heads * 64, device=dev)
        self.ws = torch.empty(load().ref_bwd_workspace_bytes(b, heads, s), dtype=torch.uint8,
                              device=dev)

    def _ptrs(self):
        base = self.qkv.data_ptr()
        return base, base + 4 * self.hd, base + 4 * 2 * self.hd

    def forward(self, stream=None):
        s = torch.cuda.current_stream().cuda_stream if stream is None else stream
        q, k, v = self._ptrs()
        rc = load().ref_fwd(q, k, v, self.o.data_ptr(), self.lse.data_ptr(), self.b, self.h,
                            self.s, self.scale, self.causal, self.st, self.st, self.st, s)
        if rc != 0:
            raise RuntimeError(f"ref_fwd failed ({rc})")

    def backward(self, dout: torch.Tensor, stream=None):
        s = torch.cuda.current_stream().cuda_stream if stream is None else stream
        q, k, v = self._ptrs()
        gs = _s3((dout.stride(0), 64, dout.stride(1)))
        rc = load().ref_bwd(q, k, v, self.o.data_ptr(), self.lse.data_ptr(), dout.data_ptr(),
                            self.dqkv.data_ptr(), self.ws.data_ptr(), self.b, self.h, self.s,
                            self.scale, self.causal, self.st, self.st, self.st, gs, s)
        if rc != 0:
            raise RuntimeError(f"ref_bwd failed ({rc})")


class RefAttention:
    """The reference kernels on [b, h, s, 64] views q, k, v (any float4-aligned strides) and dO
    (same shape), buffers allocated once."""

    def __init__(self, q, k, v, scale: float, causal: bool):
        b, h, s, _ = q.shape
        self.b, self.h, self.s = b, h, s
        self.q, self.k, self.v = q, k, v
        self.scale, self.causal = float(scale), int(bool(causal))
        self.qs, self.ks, self.vs = (_s3(t.stride()[:3]) for t in (q, k, v))
        dev = q.device
        self.o = torch.empty(b, s, h, 64, device=dev)
        self.lse = torch.empty(b, h, s, device=dev)
        self.dqkv = torch.empty(b, s, 3, h, 64, device=dev)
        self.ws = torch.empty(load().ref_bwd_workspace_bytes(b, h, s), dtype=torch.uint8,
                              device=dev)

    def forward(self, stream):
        rc = load().ref_fwd(self.q.data_ptr(), self.k.data_ptr(), self.v.data_ptr(),
                            self.o.data_ptr(), self.lse.data_ptr(), self.b, self.h, self.s,
                            self.scale, self.causal, self.qs, self.ks, self.vs, stream)
        if rc != 0:
            raise RuntimeError(f"ref_fwd failed ({rc})")

    def backward(self, d_o, stream):
        rc = load().ref_bwd(self.q.data_ptr(), self.k.data_ptr(), self.v.data_ptr(),
                            self.o.data_ptr(), self.lse.data_ptr(), d_o.data_ptr(),
                            self.dqkv.data_ptr(), self.ws.data_ptr(), self.b, self.h, self.s,
                            self.scale, self.causal, self.qs, self.ks, self.vs,
                            _s3(d_o.stride()[:3]), stream)
        if rc != 0:
            raise RuntimeError(f"ref_bwd failed ({rc})")
