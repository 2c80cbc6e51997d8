# SPDX-License-Identifier: MIT OR Apache-2.0
"""The C ABI on the CPU: libcfa.so loads, exports every symbol include/cfa.h declares, and rejects
bad arguments before touching a device (so these run without a GPU)."""

import re
import subprocess
from pathlib import Path

import pytest

from candle_fused_attn import _abi

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "cfa.h"


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\**\s+\**(cfa_\w+)\s*\(", text, re.M)))


def test_header_declares_the_abi():
    assert declared_functions() == sorted(_abi.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = _abi.load()
    for name in declared_functions():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(_abi.LIB_PATH)],
                         capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r" T (cfa_\w+)", out))
    assert set(declared_functions()) <= exported


def test_version_and_strerror():
    lib = _abi.load()
    assert lib.cfa_abi_version() >> 16 == 2
    for code in range(10):
        msg = _abi.strerror(code)
        assert msg.startswith("fused_attention:")
    assert "head_dim 64" in _abi.strerror(_abi.CFA_ERR_HEAD_DIM)
    assert "unknown" in _abi.strerror(12345)


def test_workspace_formula():
    # ticket/err header 256 B + turn counters + D, each 256-aligned
    b, h, s = 64, 6, 240
    nqt = (s + 63) // 64
    turn = (b * h * nqt * 4 + 255) // 256 * 256
    dsum = (b * h * s * 4 + 255) // 256 * 256
    assert _abi.bwd_workspace_bytes(b, h, s) == 256 + turn + dsum
    assert _abi.bwd_workspace_bytes(0, 6, 240) == 256
    # the no-wait dQ path adds one partial per key block of 64 (s <= 1024 only)
    nkb = (s + 63) // 64
    assert _abi.bwd_workspace_bytes_fast(b, h, s) == 256 + turn + dsum + nkb * b * h * s * 64 * 4
    assert _abi.bwd_workspace_bytes_fast(4, 16, 8192) == _abi.bwd_workspace_bytes(4, 16, 8192)
    assert _abi.bwd_workspace_bytes_fast(1, 1, 1024) > _abi.bwd_workspace_bytes(1, 1, 1024)
    assert _abi.bwd_workspace_bytes_fast(1, 1, 1025) == _abi.bwd_workspace_bytes(1, 1, 1025)


def test_workspace_formula_head_dims():
    """The head-dim-generic sizes: the same layout, the dQ partials holding head_dim floats a row;
    unsupported head dims get the minimal size (their calls return CFA_ERR_HEAD_DIM)."""
    b, h, s = 64, 6, 240
    assert _abi.bwd_workspace_bytes_hd(b, h, s, 64) == _abi.bwd_workspace_bytes(b, h, s)
    assert _abi.bwd_workspace_bytes_fast_hd(b, h, s, 64) == _abi.bwd_workspace_bytes_fast(b, h, s)
    base = _abi.bwd_workspace_bytes(b, h, s)
    part64 = _abi.bwd_workspace_bytes_fast(b, h, s) - base
    for d in (32, 128):
        assert _abi.bwd_workspace_bytes_hd(b, h, s, d) == base
        assert _abi.bwd_workspace_bytes_fast_hd(b, h, s, d) - base == part64 * d // 64
    for d in (0, 16, 48, 256):
        assert _abi.bwd_workspace_bytes_hd(b, h, s, d) == 256
        assert _abi.bwd_workspace_bytes_fast_hd(b, h, s, d) == 256


FAKE = 1 << 20  # a 16-byte aligned non-null "device pointer" never dereferenced by these checks


def fwd(ptrs=(FAKE,) * 5, strides=((64 * 240, 64, 64),) * 3, dims=(2, 3, 240, 64)):
    q, k, v, o, lse = ptrs
    return _abi.fwd(q, strides[0], k, strides[1], v, strides[2], o, lse, *dims, 0.125, 0, None)


def test_rejects_head_dim():
    # the _d64 entry points keep the reference's gate (src/cuda.rs:85-93)
    assert fwd(dims=(2, 3, 240, 32)) == _abi.CFA_ERR_HEAD_DIM
    assert fwd(dims=(2, 3, 240, 128)) == _abi.CFA_ERR_HEAD_DIM


def test_generic_entry_points_reject_other_head_dims():
    """cfa_fwd_f32 / cfa_bwd_f32 take 32, 64 and 128; anything else fails before any device work
    (empty problems included, as the _d64 ones do for head dims other than 64)."""
    for d in (0, 16, 48, 96, 256):
        st = (64 * 240, d, d)
        assert _abi.fwd_hd(FAKE, st, FAKE, st, FAKE, st, FAKE, FAKE, 2, 3, 240, d, 0.1, 0,
                           None) == _abi.CFA_ERR_HEAD_DIM
        assert _abi.bwd_hd(FAKE, st, FAKE, st, FAKE, st, FAKE, FAKE, FAKE, st, FAKE, FAKE, 1 << 30,
                           2, 3, 240, d, 0.1, 0, None) == _abi.CFA_ERR_HEAD_DIM
    for d in (32, 128):  # empty problems are fine for the supported head dims, no launch
        st = (0, 0, 0)
        assert _abi.fwd_hd(0, st, 0, st, 0, st, 0, 0, 0, 3, 240, d, 0.1, 0, None) == _abi.CFA_OK


def test_empty_problem_is_ok_and_launches_nothing():
    # audit B2: the reference panics on empty inputs; here they are a no-op.
    assert fwd(ptrs=(None,) * 5, dims=(0, 3, 240, 64)) == _abi.CFA_OK
    assert fwd(ptrs=(None,) * 5, dims=(2, 0, 240, 64)) == _abi.CFA_OK
    assert fwd(ptrs=(None,) * 5, dims=(2, 3, 0, 64)) == _abi.CFA_OK


def test_rejects_negative_null_misaligned_overflow():
    assert fwd(dims=(-1, 3, 240, 64)) == _abi.CFA_ERR_SHAPE
    assert fwd(ptrs=(FAKE, None, FAKE, FAKE, FAKE)) == _abi.CFA_ERR_NULL
    assert fwd(ptrs=(FAKE + 4, FAKE, FAKE, FAKE, FAKE)) == _abi.CFA_ERR_ALIGNMENT
    assert fwd(strides=((64 * 240, 64, 66),) * 3) == _abi.CFA_ERR_ALIGNMENT
    assert fwd(dims=(1 << 20, 1 << 10, 1 << 10, 64)) == _abi.CFA_ERR_OVERFLOW


def test_bwd_rejects_small_or_misaligned_workspace():
    s3 = (64 * 240, 64, 64)
    need = _abi.bwd_workspace_bytes(2, 3, 240)
    args = dict(b=2, h=3, s=240, d=64, scale=0.125, causal=0, stream=None)

    def call(ws, nbytes):
        return _abi.bwd(FAKE, s3, FAKE, s3, FAKE, s3, FAKE, FAKE, FAKE, s3, FAKE, ws, nbytes,
                        **args)

    assert call(FAKE, need - 1) == _abi.CFA_ERR_WORKSPACE
    assert call(FAKE + 16, need) == _abi.CFA_ERR_WORKSPACE
    assert call(None, need) == _abi.CFA_ERR_NULL


def test_null_status_query():
    assert _abi.bwd_status(None, None) == _abi.CFA_ERR_NULL


def test_ffma_pair_entry_points_check_arguments():
    """The CUDA-core pair's entry points apply the head-dim-64 checks of the default ones before
    touching a device."""
    st = (1024, 256, 64)
    lib = _abi.load()
    for fwd in (_abi.fwd, _abi.fwd_ffma):
        assert fwd(FAKE, st, FAKE, st, FAKE, st, FAKE, FAKE, 1, 1, 8, 32, 0.1, 0,
                   None) == _abi.CFA_ERR_HEAD_DIM
        assert fwd(FAKE, st, FAKE, st, FAKE, st, FAKE, FAKE, 0, 1, 8, 64, 0.1, 0,
                   None) == _abi.CFA_OK
        assert fwd(None, st, FAKE, st, FAKE, st, FAKE, FAKE, 1, 1, 8, 64, 0.1, 0,
                   None) == _abi.CFA_ERR_NULL
        assert fwd(FAKE + 4, st, FAKE, st, FAKE, st, FAKE, FAKE, 1, 1, 8, 64, 0.1, 0,
                   None) == _abi.CFA_ERR_ALIGNMENT
    for bwd in (_abi.bwd, _abi.bwd_ffma):
        assert bwd(FAKE, st, FAKE, st, FAKE, st, FAKE, FAKE, FAKE, st, FAKE, FAKE, 1 << 20,
                   1, 1, 8, 128, 0.1, 0, None) == _abi.CFA_ERR_HEAD_DIM
        assert bwd(FAKE, st, FAKE, st, FAKE, st, FAKE, FAKE, FAKE, st, FAKE, FAKE, 16,
                   1, 1, 8, 64, 0.1, 0, None) == _abi.CFA_ERR_WORKSPACE
    assert not hasattr(_abi, "fwd_select")
    with pytest.raises(AttributeError):
        lib.cfa_fwd_select  # one pair per entry point: no process-wide switch


def test_error_sink_host_checks():
    """cfa_error_sink: NULL unregisters (always OK); a misaligned address is refused before any
    CUDA call."""
    assert _abi.error_sink(None) == _abi.CFA_OK
    assert _abi.error_sink(FAKE + 2) == _abi.CFA_ERR_ALIGNMENT
    assert _abi.error_sink(None) == _abi.CFA_OK


def test_noalloc_checks_before_scratch_size():
    """The no-allocation backward reports a bad head dim, an empty problem and a null pointer as
    such -- checked before the scratch size, so a huge problem with head dim 32 is a head-dim
    error, not a workspace one -- and an oversized problem as CFA_ERR_WORKSPACE."""
    st = (1024, 256, 64)
    args = lambda q, b, h, s, d: (q, st, FAKE, st, FAKE, st, FAKE, FAKE, FAKE, st, FAKE,  # noqa
                                  b, h, s, d, 0.125, 0, None)
    assert _abi.bwd_noalloc(*args(FAKE, 64, 6, 240, 32)) == _abi.CFA_ERR_HEAD_DIM
    assert _abi.bwd_noalloc(*args(FAKE, 1 << 20, 64, 1 << 12, 32)) == _abi.CFA_ERR_HEAD_DIM
    assert _abi.bwd_noalloc(*args(None, 64, 6, 240, 64)) == _abi.CFA_ERR_NULL
    assert _abi.bwd_noalloc(*args(FAKE, 0, 6, 240, 64)) == _abi.CFA_OK
    assert _abi.bwd_noalloc(*args(FAKE, -1, 6, 240, 64)) == _abi.CFA_ERR_SHAPE
    assert _abi.bwd_noalloc(*args(FAKE, 1 << 30, 1 << 30, 1 << 30, 64)) == _abi.CFA_ERR_OVERFLOW
    assert _abi.bwd_noalloc(*args(FAKE, 64, 64, 1024, 64)) == _abi.CFA_ERR_WORKSPACE


def test_matmul_checks_arguments():
    """cfa_matmul_f32's host-side checks (no launch): empty problems, negative or huge sizes, null
    pointers, C's 16-byte rows, the workspace (size and 256-byte alignment)."""
    need = _abi.matmul_workspace_bytes(300, 200, 100)
    assert need > 0 and _abi.matmul_workspace_bytes(0, 5, 5) == 0

    def call(m=300, n=200, k=100, a=FAKE, b=FAKE, c=FAKE, ldc=200, ws=FAKE, nbytes=need):
        return _abi.matmul(a, 100, 1, b, 200, 1, c, ldc, m, n, k, ws, nbytes, None)

    assert call(m=0) == _abi.CFA_OK and call(n=0, c=None) == _abi.CFA_OK
    assert call(m=-1) == _abi.CFA_ERR_SHAPE
    assert call(k=1 << 31) == _abi.CFA_ERR_OVERFLOW
    assert call(a=None) == _abi.CFA_ERR_NULL and call(ws=None) == _abi.CFA_ERR_NULL
    assert call(c=FAKE + 4) == _abi.CFA_ERR_ALIGNMENT
    assert call(ldc=202) == _abi.CFA_ERR_ALIGNMENT
    assert call(nbytes=need - 1) == _abi.CFA_ERR_WORKSPACE
    assert call(ws=FAKE + 16) == _abi.CFA_ERR_WORKSPACE


def test_matmul_workspace_grows_with_the_parts():
    """The workspace holds both operands' bf16 parts (6 bytes an element, 128 x 16 blocks) and, when
    K is cut into chunks (few output tiles), their partial tiles."""
    m, n, k = 15360, 1152, 384
    parts = (m // 128 + n // 128) * (k // 16) * 3 * 128 * 16 * 2
    assert _abi.matmul_workspace_bytes(m, n, k) >= parts
    m, n, k = 384, 1152, 15360  # 27 output tiles: K in chunks
    parts = (m // 128 + n // 128) * (k // 16) * 3 * 128 * 16 * 2
    assert _abi.matmul_workspace_bytes(m, n, k) >= parts + 2 * m * n * 4
