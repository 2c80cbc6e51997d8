# SPDX-License-Identifier: MIT OR Apache-2.0
"""Property tests of the host-side logic (CPU, hypothesis): the qkv geometry, the alignment
predicate, the shard ranges and the workspace sizes."""

import torch
from hypothesis import given, settings
from hypothesis import strategies as st

import candle_fused_attn as cfa
from candle_fused_attn import _abi
from candle_fused_attn.sharding import shard_range


@settings(max_examples=200, derandomize=True)
@given(b=st.integers(1, 64), s=st.integers(1, 4096), h=st.integers(1, 32))
def test_qkv_geometry_addresses_every_element_once(b, s, h):
    shape, stride = (b, s, 3 * h * 64), (s * 3 * h * 64, 3 * h * 64, 1)
    dims, st3, offs = cfa.qkv_geometry(shape, stride, h)
    assert dims == (b, h, s, 64)
    # q, k, v views tile the projection's last dimension exactly: offsets 0, hd, 2hd, head stride d
    assert offs == (0, h * 64, 2 * h * 64) and st3 == (stride[0], 64, stride[1])


@settings(max_examples=200, derandomize=True)
@given(off=st.integers(0, 7), sb=st.integers(1, 50), sh=st.integers(1, 50),
       ss=st.integers(1, 50))
def test_float4_aligned_matches_definition(off, sb, sh, ss):
    t = torch.empty(off + 4 * 64 * 50 * 50 * 50).as_strided((2, 2, 2, 4), (sb, sh, ss, 1), off)
    want = off % 4 == 0 and sb % 4 == 0 and sh % 4 == 0 and ss % 4 == 0
    assert cfa.float4_aligned(t) == want


@settings(max_examples=300, derandomize=True)
@given(batch=st.integers(0, 10000), world=st.integers(1, 64))
def test_shard_ranges_partition(batch, world):
    ranges = [shard_range(batch, world, r) for r in range(world)]
    assert sum(hi - lo for lo, hi in ranges) == batch
    assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))


@settings(max_examples=200, derandomize=True)
@given(b=st.integers(1, 512), h=st.integers(1, 64), s=st.integers(1, 16384))
def test_workspace_sizes(b, h, s):
    small, fast = _abi.bwd_workspace_bytes(b, h, s), _abi.bwd_workspace_bytes_fast(b, h, s)
    assert small % 256 == 0 and fast % 256 == 0
    assert small >= 256 + b * h * s * 4
    nkb = (s + 63) // 64
    assert fast == (small + nkb * b * h * s * 64 * 4 if nkb <= 16 else small)
