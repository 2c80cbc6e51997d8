# SPDX-License-Identifier: MIT OR Apache-2.0
"""Batch-sharded runs on several GPUs (one process per GPU, NCCL): every rank runs the kernels on
its contiguous batch shard with no exchange; NCCL all-gathers O and dqkv only to check them, and
rank 0 compares them bit for bit with the whole batch run on one GPU (BASELINE configs[4] in
small: qkv [16 * world, 240, 1152], 6 heads, non-causal; and a causal s = 1024 case)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, cases, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        import candle_fused_attn as cfa
        from candle_fused_attn.sharding import gather_batches, shard_range
        from oracle import oracle
        results = []
        for (batch, h, s, causal) in cases:
            qkv, dout = oracle.seeded_inputs(batch, h, s, 3, 0.5)
            lo, hi = shard_range(batch, world, rank)

            def run(x, g):
                x = x.to(dev).requires_grad_(True)
                o = cfa.fused_attention_qkv(x, h, 0.125, causal)
                o.backward(g.to(dev))
                return o.detach(), x.grad

            o, g = run(qkv[lo:hi], dout[lo:hi])
            pad = -(-batch // world)
            og, gg = gather_batches(o, world, dist, pad), gather_batches(g, world, dist, pad)
            if rank == 0:
                o1, g1 = run(qkv, dout)
                results.append(torch.equal(og.view(torch.int32), o1.view(torch.int32)) and
                               torch.equal(gg.view(torch.int32), g1.view(torch.int32)))
        if rank == 0:
            out.put(results)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_sharded_runs_are_bitwise_equal_to_one_gpu():
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip(f"needs 2+ GPUs, found {n}")
    world = min(n, 8)
    cases = [(16 * world, 6, 240, False), (2 * world + 1, 4, 1024, True)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, cases, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=10) == [True, True]
