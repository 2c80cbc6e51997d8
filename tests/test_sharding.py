# SPDX-License-Identifier: MIT OR Apache-2.0
"""Batch sharding on CPU ranks (gloo, world_size 2): the shard ranges, and that the oracle run
shard by shard and all-gathered is bit-identical to the whole-batch run (the property the GPU
kernels are tested for on NCCL ranks in tests/test_multigpu_gpu.py)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from candle_fused_attn.sharding import gather_batches, shard_range


def test_shard_range_covers_batch():
    for batch in (1, 7, 64, 512):
        for world in (1, 2, 3, 8):
            ranges = [shard_range(batch, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == batch
            for (a, b), (c, d) in zip(ranges, ranges[1:]):
                assert b == c
            sizes = [hi - lo for lo, hi in ranges]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, batch, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from oracle import oracle
        qkv, dout = oracle.seeded_inputs(batch, 2, 33, 9)
        lo, hi = shard_range(batch, world, rank)
        o, lse, g = oracle.qkv_forward_backward(qkv[lo:hi], dout[lo:hi], 2, 0.125, True,
                                                threads=1)
        pad = -(-batch // world)
        og = gather_batches(o, world, dist, pad)
        gg = gather_batches(g, world, dist, pad)
        if rank == 0:
            o_all, _, g_all = oracle.qkv_forward_backward(qkv, dout, 2, 0.125, True, threads=1)
            out.put((torch.equal(og, o_all), torch.equal(gg, g_all)))
    finally:
        dist.destroy_process_group()


def test_gloo_world2_shards_gather_bitwise():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, 5, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=5) == (True, True)
