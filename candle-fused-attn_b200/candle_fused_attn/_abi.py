# SPDX-License-Identifier: MIT OR Apache-2.0
"""ctypes binding of the C ABI in include/cfa.h (libcfa.so, built in-tree for sm_100a).

This is the Python twin of the Rust `extern "C"` shim that replaces the reference's launch layer
(src/cuda.rs): the same entry points a Rust, C or C++ caller binds. Loading fails loudly when the
library is missing; there is no fallback of any kind.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_NAME = "libcfa.so"
LIB_PATH = Path(__file__).resolve().parent / LIB_NAME

# include/cfa.h enum cfa_status
CFA_OK = 0
CFA_ERR_HEAD_DIM = 1
CFA_ERR_ALIGNMENT = 2
CFA_ERR_SHAPE = 3
CFA_ERR_OVERFLOW = 4
CFA_ERR_NULL = 5
CFA_ERR_WORKSPACE = 6
CFA_ERR_LAUNCH = 7
CFA_ERR_TIMEOUT = 8
CFA_ERR_CUDA = 9

# Every symbol include/cfa.h declares.
EXPORTS = (
    "cfa_fwd_f32_d64",
    "cfa_bwd_workspace_bytes",
    "cfa_bwd_workspace_bytes_fast",
    "cfa_bwd_f32_d64",
    "cfa_bwd_f32_d64_noalloc",
    "cfa_bwd_status",
    "cfa_selftest_bounded_wait",
    "cfa_strerror",
    "cfa_abi_version",
    "cfa_fwd_f32",
    "cfa_bwd_workspace_bytes_hd",
    "cfa_bwd_workspace_bytes_fast_hd",
    "cfa_bwd_f32",
    "cfa_fwd_status",
    "cfa_fwd_f32_d64_ffma",
    "cfa_bwd_f32_d64_ffma",
    "cfa_bwd_noalloc_status",
    "cfa_error_sink",
    "cfa_matmul_workspace_bytes",
    "cfa_matmul_f32",
    "cfa_matmul_status",
    "cfa_fwd_f32_ffma",
    "cfa_bwd_f32_ffma",
)

# Head dims the generic entry points (cfa_fwd_f32, cfa_bwd_f32) take; the _d64 ones take 64 only,
# as the reference's CUDA path does (src/lib.rs:91).
HEAD_DIMS = (32, 64, 128)

_i64 = ctypes.c_int64
_p = ctypes.c_void_p
_strides = ctypes.POINTER(ctypes.c_int64)

_lib: ctypes.CDLL | None = None


class CfaError(RuntimeError):
    """A non-zero status from the C ABI, with its code and `cfa_strerror` text."""

    def __init__(self, status: int, where: str):
        self.status = status
        super().__init__(f"{strerror(status)} (status {status}, {where})")


def load() -> ctypes.CDLL:
    """The loaded library (loaded once, argument types declared)."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("CFA_LIBRARY", LIB_PATH))
    if not path.is_file():
        raise ImportError(
            f"candle_fused_attn: {path} is missing; build it with `python __graft_entry__.py build` "
            "(nvcc, sm_100a). There is no CPU or PyTorch fallback.")
    lib = ctypes.CDLL(str(path))
    lib.cfa_fwd_f32_d64.restype = ctypes.c_int
    lib.cfa_fwd_f32_d64.argtypes = [
        _p, _strides, _p, _strides, _p, _strides, _p, _p,
        _i64, _i64, _i64, _i64, ctypes.c_float, ctypes.c_int, _p]
    lib.cfa_bwd_workspace_bytes.restype = ctypes.c_size_t
    lib.cfa_bwd_workspace_bytes.argtypes = [_i64, _i64, _i64]
    lib.cfa_bwd_workspace_bytes_fast.restype = ctypes.c_size_t
    lib.cfa_bwd_workspace_bytes_fast.argtypes = [_i64, _i64, _i64]
    lib.cfa_bwd_f32_d64.restype = ctypes.c_int
    lib.cfa_bwd_f32_d64.argtypes = [
        _p, _strides, _p, _strides, _p, _strides, _p, _p, _p, _strides, _p, _p, ctypes.c_size_t,
        _i64, _i64, _i64, _i64, ctypes.c_float, ctypes.c_int, _p]
    lib.cfa_bwd_status.restype = ctypes.c_int
    lib.cfa_bwd_status.argtypes = [_p, _p]
    lib.cfa_selftest_bounded_wait.restype = ctypes.c_int
    lib.cfa_selftest_bounded_wait.argtypes = [_p, _i64, ctypes.c_int, _p]
    lib.cfa_strerror.restype = ctypes.c_char_p
    lib.cfa_strerror.argtypes = [ctypes.c_int]
    lib.cfa_abi_version.restype = ctypes.c_int
    lib.cfa_abi_version.argtypes = []
    lib.cfa_fwd_f32.restype = ctypes.c_int
    lib.cfa_fwd_f32.argtypes = lib.cfa_fwd_f32_d64.argtypes
    lib.cfa_bwd_f32.restype = ctypes.c_int
    lib.cfa_bwd_f32.argtypes = lib.cfa_bwd_f32_d64.argtypes
    lib.cfa_fwd_f32_d64_ffma.restype = ctypes.c_int
    lib.cfa_fwd_f32_d64_ffma.argtypes = lib.cfa_fwd_f32_d64.argtypes
    lib.cfa_bwd_f32_d64_ffma.restype = ctypes.c_int
    lib.cfa_bwd_f32_d64_ffma.argtypes = lib.cfa_bwd_f32_d64.argtypes
    lib.cfa_fwd_f32_ffma.restype = ctypes.c_int
    lib.cfa_fwd_f32_ffma.argtypes = lib.cfa_fwd_f32_d64.argtypes
    lib.cfa_bwd_f32_ffma.restype = ctypes.c_int
    lib.cfa_bwd_f32_ffma.argtypes = lib.cfa_bwd_f32_d64.argtypes
    lib.cfa_bwd_noalloc_status.restype = ctypes.c_int
    lib.cfa_bwd_noalloc_status.argtypes = [_p]
    lib.cfa_error_sink.restype = ctypes.c_int
    lib.cfa_error_sink.argtypes = [_p]
    lib.cfa_fwd_status.restype = ctypes.c_int
    lib.cfa_fwd_status.argtypes = [_p]
    lib.cfa_matmul_workspace_bytes.restype = ctypes.c_size_t
    lib.cfa_matmul_workspace_bytes.argtypes = [_i64, _i64, _i64]
    lib.cfa_matmul_f32.restype = ctypes.c_int
    lib.cfa_matmul_f32.argtypes = [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _i64, _i64,
                                   _p, ctypes.c_size_t, _p]
    lib.cfa_matmul_status.restype = ctypes.c_int
    lib.cfa_matmul_status.argtypes = [_p]
    for name in ("cfa_bwd_workspace_bytes_hd", "cfa_bwd_workspace_bytes_fast_hd"):
        fn = getattr(lib, name)
        fn.restype = ctypes.c_size_t
        fn.argtypes = [_i64, _i64, _i64, _i64]
    _lib = lib
    return lib


def strerror(status: int) -> str:
    return load().cfa_strerror(int(status)).decode()


def strides3(s) -> ctypes.Array:
    """A (batch, head, seq) stride triple as the `const int64_t[3]` the ABI takes."""
    return (ctypes.c_int64 * 3)(*(int(x) for x in s))


def check(status: int, where: str) -> None:
    if status != CFA_OK:
        raise CfaError(status, where)


def fwd(q_ptr, qs, k_ptr, ks, v_ptr, vs, o_ptr, lse_ptr, b, h, s, d, scale, causal, stream) -> int:
    """cfa_fwd_f32_d64; returns the status."""
    return load().cfa_fwd_f32_d64(
        q_ptr, strides3(qs), k_ptr, strides3(ks), v_ptr, strides3(vs), o_ptr, lse_ptr,
        b, h, s, d, ctypes.c_float(scale), int(bool(causal)), stream)


def bwd_workspace_bytes(b, h, s) -> int:
    return int(load().cfa_bwd_workspace_bytes(b, h, s))


def bwd_workspace_bytes_fast(b, h, s) -> int:
    return int(load().cfa_bwd_workspace_bytes_fast(b, h, s))


def bwd(q_ptr, qs, k_ptr, ks, v_ptr, vs, o_ptr, lse_ptr, do_ptr, dos, dqkv_ptr, ws_ptr, ws_bytes,
        b, h, s, d, scale, causal, stream) -> int:
    """cfa_bwd_f32_d64; returns the status."""
    return load().cfa_bwd_f32_d64(
        q_ptr, strides3(qs), k_ptr, strides3(ks), v_ptr, strides3(vs), o_ptr, lse_ptr,
        do_ptr, strides3(dos), dqkv_ptr, ws_ptr, ws_bytes, b, h, s, d,
        ctypes.c_float(scale), int(bool(causal)), stream)


def fwd_hd(q_ptr, qs, k_ptr, ks, v_ptr, vs, o_ptr, lse_ptr, b, h, s, d, scale, causal,
           stream) -> int:
    """cfa_fwd_f32 (head dim d in HEAD_DIMS); returns the status."""
    return load().cfa_fwd_f32(
        q_ptr, strides3(qs), k_ptr, strides3(ks), v_ptr, strides3(vs), o_ptr, lse_ptr,
        b, h, s, d, ctypes.c_float(scale), int(bool(causal)), stream)


def fwd_ffma(q_ptr, qs, k_ptr, ks, v_ptr, vs, o_ptr, lse_ptr, b, h, s, d, scale, causal,
             stream) -> int:
    """cfa_fwd_f32_d64_ffma (the CUDA-core pair's forward); returns the status."""
    return load().cfa_fwd_f32_d64_ffma(
        q_ptr, strides3(qs), k_ptr, strides3(ks), v_ptr, strides3(vs), o_ptr, lse_ptr,
        b, h, s, d, ctypes.c_float(scale), int(bool(causal)), stream)


def bwd_ffma(q_ptr, qs, k_ptr, ks, v_ptr, vs, o_ptr, lse_ptr, do_ptr, dos, dqkv_ptr, ws_ptr,
             ws_bytes, b, h, s, d, scale, causal, stream) -> int:
    """cfa_bwd_f32_d64_ffma (the CUDA-core pair's backward; L from fwd_ffma); the status."""
    return load().cfa_bwd_f32_d64_ffma(
        q_ptr, strides3(qs), k_ptr, strides3(ks), v_ptr, strides3(vs), o_ptr, lse_ptr,
        do_ptr, strides3(dos), dqkv_ptr, ws_ptr, ws_bytes, b, h, s, d,
        ctypes.c_float(scale), int(bool(causal)), stream)


def fwd_hd_ffma(q_ptr, qs, k_ptr, ks, v_ptr, vs, o_ptr, lse_ptr, b, h, s, d, scale, causal,
                stream) -> int:
    """cfa_fwd_f32_ffma (the CUDA-core pair at head dim d in HEAD_DIMS); returns the status."""
    return load().cfa_fwd_f32_ffma(
        q_ptr, strides3(qs), k_ptr, strides3(ks), v_ptr, strides3(vs), o_ptr, lse_ptr,
        b, h, s, d, ctypes.c_float(scale), int(bool(causal)), stream)


def bwd_hd_ffma(q_ptr, qs, k_ptr, ks, v_ptr, vs, o_ptr, lse_ptr, do_ptr, dos, dqkv_ptr, ws_ptr,
                ws_bytes, b, h, s, d, scale, causal, stream) -> int:
    """cfa_bwd_f32_ffma (L from fwd_hd_ffma); returns the status."""
    return load().cfa_bwd_f32_ffma(
        q_ptr, strides3(qs), k_ptr, strides3(ks), v_ptr, strides3(vs), o_ptr, lse_ptr,
        do_ptr, strides3(dos), dqkv_ptr, ws_ptr, ws_bytes, b, h, s, d,
        ctypes.c_float(scale), int(bool(causal)), stream)


def bwd_workspace_bytes_hd(b, h, s, d) -> int:
    return int(load().cfa_bwd_workspace_bytes_hd(b, h, s, d))


def bwd_workspace_bytes_fast_hd(b, h, s, d) -> int:
    return int(load().cfa_bwd_workspace_bytes_fast_hd(b, h, s, d))


def bwd_hd(q_ptr, qs, k_ptr, ks, v_ptr, vs, o_ptr, lse_ptr, do_ptr, dos, dqkv_ptr, ws_ptr,
           ws_bytes, b, h, s, d, scale, causal, stream) -> int:
    """cfa_bwd_f32 (head dim d in HEAD_DIMS); returns the status."""
    return load().cfa_bwd_f32(
        q_ptr, strides3(qs), k_ptr, strides3(ks), v_ptr, strides3(vs), o_ptr, lse_ptr,
        do_ptr, strides3(dos), dqkv_ptr, ws_ptr, ws_bytes, b, h, s, d,
        ctypes.c_float(scale), int(bool(causal)), stream)


def bwd_status(ws_ptr, stream) -> int:
    return load().cfa_bwd_status(ws_ptr, stream)


def error_sink(host_ptr) -> int:
    """cfa_error_sink: register a page-locked host int (its address; None unregisters) that every
    bounded-wait expiry reaches without a synchronisation. Returns the status."""
    return load().cfa_error_sink(host_ptr)


def bwd_noalloc_status(stream) -> int:
    """cfa_bwd_noalloc_status: synchronises `stream`; CFA_ERR_TIMEOUT if the last no-allocation
    backward on the current device had a bounded wait expire."""
    return load().cfa_bwd_noalloc_status(stream)


def fwd_status(stream) -> int:
    """Synchronises `stream`; CFA_ERR_TIMEOUT if a tensor-core forward's bounded wait expired."""
    return load().cfa_fwd_status(stream)


def selftest_bounded_wait(ws_ptr, timeout_ns, blocks, stream) -> int:
    return load().cfa_selftest_bounded_wait(ws_ptr, int(timeout_ns), int(blocks), stream)


NOALLOC_SCRATCH_BYTES = 4 << 20  # include/cfa.h CFA_NOALLOC_SCRATCH_BYTES


def bwd_noalloc(q_ptr, qs, k_ptr, ks, v_ptr, vs, o_ptr, lse_ptr, do_ptr, dos, dqkv_ptr,
                b, h, s, d, scale, causal, stream) -> int:
    """cfa_bwd_f32_d64_noalloc: the backward with its scratch in the library's static device
    array, for callers that cannot allocate device memory. Returns the status."""
    fn = load().cfa_bwd_f32_d64_noalloc
    if fn.argtypes is None:
        fn.restype = ctypes.c_int
        fn.argtypes = [_p, _strides, _p, _strides, _p, _strides, _p, _p, _p, _strides, _p,
                       _i64, _i64, _i64, _i64, ctypes.c_float, ctypes.c_int, _p]
    return fn(q_ptr, strides3(qs), k_ptr, strides3(ks), v_ptr, strides3(vs), o_ptr, lse_ptr,
              do_ptr, strides3(dos), dqkv_ptr, b, h, s, d, ctypes.c_float(scale),
              int(bool(causal)), stream)


def matmul_workspace_bytes(m, n, k) -> int:
    return int(load().cfa_matmul_workspace_bytes(m, n, k))


def matmul(a_ptr, a_rs, a_cs, b_ptr, b_rs, b_cs, c_ptr, c_rs, m, n, k, ws_ptr, ws_bytes,
           stream) -> int:
    """cfa_matmul_f32: C (m x n, rows c_rs apart) = A (m x k) B (k x n), each operand through its
    (row, column) strides; returns the status."""
    return load().cfa_matmul_f32(a_ptr, a_rs, a_cs, b_ptr, b_rs, b_cs, c_ptr, c_rs, m, n, k,
                                 ws_ptr, ws_bytes, stream)


def matmul_status(stream) -> int:
    return load().cfa_matmul_status(stream)
