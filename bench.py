# SPDX-License-Identifier: MIT OR Apache-2.0
"""Benchmark: fused fp32 attention forward + backward at the canvas shape, per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: fused_attention_qkv on qkv [64, 240, 1152] (6 heads x 64,
N(0,1) * 0.5, seeded), scale 1/8, non-causal, dO [64, 240, 384] N(0, 1); one step = one forward
+ one backward. Under torchrun with N GPUs every rank owns a 64-batch shard (weak scaling; at N=8
the job is BASELINE.json configs[4], qkv [512, 240, 1152] split 8 ways) and there is no collective
on the data path: NCCL only carries the barrier and the max-over-ranks time.

One JSON line on rank 0:
  value      whole-job TFLOP/s (algorithmic 14 b h s^2 d per step) with inputs resident in HBM,
             over K steps timed with CUDA events between barriers; inputs rotate over 3 sets
             (> L2) so no step starts from a warm L2;
  e2e        the same metric through the public host-buffer API (HostPipeline: pinned qkv, dO
             copied in and O, dqkv copied out inside the timed region, batch chunks overlapping
             both copy directions with the kernels); the plain fused_attention_qkv + autograd
             path with unoverlapped copies is reported beside it;
  roofline   the backward kernel (the dominant one; at head dim 64 and s <= 1024 the tensor-core
             kernel): achieved = 10 b h s^2 d / its event-timed duration, against the split
             scheme's fp32 ceiling -- the measured bf16 tensor peak of MEASURED_PEAKS.json over
             the 6 bf16 products each fp32 product takes; the FFMA peak (148 SMs x 128 FMA/clk
             x 2 x the measured max SM clock) beside it;
  ref_kernel the reference's own kernels (kernels/fused_attn.cu built for sm_100a) on the same
             inputs, same GPU, alternating rounds with ours;
  cpu_baseline  the CPU oracle (a port of the reference's composed path) on every host core.
`--impl reference` times the reference's CPU composed path (the oracle port) alone.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "candle-fused-attn_b200"))
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

B_PER_GPU, H, S, D = 64, 6, 240, 64
SCALE, CAUSAL = 0.125, False
N_SETS = 3
METRIC = "fwd+bwd TFLOP/s, fused_attention_qkv b64*h6*s240*d64 fp32 non-causal (per-GPU shard)"
WORKLOAD = "canvas qkv [64,240,1152] per GPU (BASELINE configs[1]; N=8 = configs[4])"


def flops(b, h, s, d, causal, which="fwdbwd"):
    p = s * (s + 1) // 2 if causal else s * s
    k = {"fwd": 4, "bwd": 10, "fwdbwd": 14}[which]
    return k * b * h * p * d


def peaks():
    try:
        mp = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        mp = {}
    mhz = float(mp.get("sm_max_mhz", 1965.0))
    return {
        "ffma_tflops": 148 * 128 * 2 * mhz * 1e6 / 1e12,
        "bf16_tflops": float(mp.get("bf16_tflops", 1590.0)),
        "hbm_gbs": float(mp.get("hbm_gbs", 6650.0)),
        "source": ("FFMA: 148 SMs x 128 FMA/clk x 2 x sm_max_mhz " + str(mhz) +
                   (" (MEASURED_PEAKS.json)" if "sm_max_mhz" in mp else " (fallback)")),
    }


class Clocks:
    """nvidia-smi samples during the timed region (the profiling recipe's clocks line)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def wait_first(self, timeout: float = 5.0) -> None:
        """Block until nvidia-smi has produced a sample (it needs ~0.1-0.5 s to start)."""
        t_end = time.time() + timeout
        while self.proc is not None and not self.lines and time.time() < t_end:
            time.sleep(0.05)

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = [[c.strip() for c in ln.split(",")] for ln in self.lines if ln]
        rows = [r for r in rows if len(r) >= 9]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows)}


def make_inputs(rank: int, b: int):
    from oracle import oracle  # the seeded generator only (bench/compare.py:496-503)
    return oracle.seeded_inputs(b, H, S, seed=1000 + rank, qkv_scale=0.5)


class OursStep:
    """One forward + backward through the C ABI on preallocated device buffers. pair: "tc" (the
    head-dim-64 entry points, the tensor-core pair) or "ffma" (the CUDA-core pair's entry points)."""

    def __init__(self, qkv, dout, pair="tc"):
        from candle_fused_attn import _abi
        self.abi = _abi
        self.fwd_fn = _abi.fwd if pair == "tc" else _abi.fwd_ffma
        self.bwd_fn = _abi.bwd if pair == "tc" else _abi.bwd_ffma
        b = qkv.shape[0]
        self.b = b
        dev = qkv.device
        self.qkv, self.dout = qkv, dout
        self.o = torch.empty(b, S, H, D, device=dev)
        self.lse = torch.empty(b, H, S, device=dev)
        self.dqkv = torch.empty(b, S, 3, H, D, device=dev)
        self.ws_bytes = _abi.bwd_workspace_bytes_fast(b, H, S)
        self.ws = torch.empty(self.ws_bytes, dtype=torch.uint8, device=dev)
        base = qkv.data_ptr()
        self.ptr = (base, base + 4 * H * D, base + 4 * 2 * H * D)
        self.st = (qkv.stride(0), D, qkv.stride(1))
        self.gst = (dout.stride(0), D, dout.stride(1))

    def fwd(self, stream):
        rc = self.fwd_fn(self.ptr[0], self.st, self.ptr[1], self.st, self.ptr[2], self.st,
                         self.o.data_ptr(), self.lse.data_ptr(), self.b, H, S, D, SCALE, CAUSAL,
                         stream)
        if rc:
            raise RuntimeError(self.abi.strerror(rc))

    def bwd(self, stream):
        rc = self.bwd_fn(self.ptr[0], self.st, self.ptr[1], self.st, self.ptr[2], self.st,
                         self.o.data_ptr(), self.lse.data_ptr(), self.dout.data_ptr(), self.gst,
                         self.dqkv.data_ptr(), self.ws.data_ptr(), self.ws_bytes, self.b, H, S,
                         D, SCALE, CAUSAL, stream)
        if rc:
            raise RuntimeError(self.abi.strerror(rc))


class OursViews:
    """Forward + backward through the C ABI on [b, h, s, d] views q, k, v and dO (head dim 64 via
    the _d64 entry points, 32 and 128 via the generic ones; scale 1/sqrt(d))."""

    def __init__(self, q, k, v, d_o, causal):
        from candle_fused_attn import _abi
        self.abi = _abi
        b, h, s, d = q.shape
        self.dims = (b, h, s, d)
        self.scale = SCALE if d == 64 else d ** -0.5
        self.fwd_fn = _abi.fwd if d == 64 else _abi.fwd_hd
        self.bwd_fn = _abi.bwd if d == 64 else _abi.bwd_hd
        self.q, self.k, self.v, self.d_o, self.causal = q, k, v, d_o, causal
        dev = q.device
        self.o = torch.empty(b, s, h, d, device=dev)
        self.lse = torch.empty(b, h, s, device=dev)
        self.dqkv = torch.empty(b, s, 3, h, d, device=dev)
        self.ws_bytes = _abi.bwd_workspace_bytes_fast_hd(b, h, s, d)
        self.ws = torch.empty(self.ws_bytes, dtype=torch.uint8, device=dev)

    def forward(self, stream):
        st = [t.stride()[:3] for t in (self.q, self.k, self.v)]
        rc = self.fwd_fn(self.q.data_ptr(), st[0], self.k.data_ptr(), st[1], self.v.data_ptr(),
                         st[2], self.o.data_ptr(), self.lse.data_ptr(), *self.dims, self.scale,
                         self.causal, stream)
        if rc:
            raise RuntimeError(self.abi.strerror(rc))

    def backward(self, d_o, stream):
        st = [t.stride()[:3] for t in (self.q, self.k, self.v)]
        rc = self.bwd_fn(self.q.data_ptr(), st[0], self.k.data_ptr(), st[1], self.v.data_ptr(),
                         st[2], self.o.data_ptr(), self.lse.data_ptr(), d_o.data_ptr(),
                         d_o.stride()[:3], self.dqkv.data_ptr(), self.ws.data_ptr(),
                         self.ws_bytes, *self.dims, self.scale, self.causal, stream)
        if rc:
            raise RuntimeError(self.abi.strerror(rc))


def suite(args):
    """Every BASELINE.json config on one GPU: ours and the reference's own kernels, forward and
    forward + backward, alternating rounds; one JSON line per config."""
    from baseline import ref_kernel
    from oracle import oracle
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    sh = stream.cuda_stream
    pk = peaks()

    def views_qkv(b, h, s, d, causal, seed, qscale):
        qkv, dout = oracle.seeded_inputs(b, h, s, seed, qscale, d=d)
        x, g = qkv.to(dev), dout.to(dev)
        q, k, v = oracle.qkv_views(x, h)
        return q, k, v, oracle.heads_view(g, h)

    def views_general(b, h, s, d, causal, seed, _):
        gen = torch.Generator().manual_seed(seed)
        q, k, v, d_o = (torch.randn(b, h, s, 64, generator=gen).to(dev) for _ in range(4))
        return q, k, v, d_o

    def views_strided(b, h, s, d, causal, seed, _):
        gen = torch.Generator().manual_seed(seed)
        x = torch.randn(b, s, 3, h, 64, generator=gen).to(dev)
        d_o = torch.randn(b, h, s, 64, generator=gen).to(dev)
        q, k, v = (x[:, :, i].permute(0, 2, 1, 3) for i in range(3))
        return q, k, v, d_o

    configs = [
        ("general [2,4,128,64] contiguous", 2, 4, 128, 64, False, views_general, 1.0),
        ("canvas qkv [64,240,1152]", 64, 6, 240, 64, False, views_qkv, 0.5),
        ("strided views of [16,1024,3,12,64], causal", 16, 12, 1024, 64, True, views_strided, 1.0),
        ("long qkv [4,8192,3072], causal", 4, 16, 8192, 64, True, views_qkv, 0.5),
        # head dims 32 and 128: this build's extension (the reference kernel takes 64 only)
        ("canvas-shaped qkv [64,240,1152], 12 heads of 32", 64, 12, 240, 32, False, views_qkv, 0.5),
        ("canvas-shaped qkv [64,240,1152], 3 heads of 128", 64, 3, 240, 128, False, views_qkv, 0.5),
        ("long qkv [4,8192,3072], 8 heads of 128, causal", 4, 8, 8192, 128, True, views_qkv, 0.5),
    ]
    if args.only:
        configs = [c for c in configs if args.only in c[0]]
    for name, b, h, s, d, causal, make, qscale in configs:
        q, k, v, d_o = make(b, h, s, d, causal, 0, qscale)
        impls = {"ours": OursViews(q, k, v, d_o, causal),
                 "reference_kernel": ref_kernel.RefAttention(q, k, v, SCALE, causal)
                 if ref_kernel.available() and d == 64 else None}
        f_fwd, f_all = flops(b, h, s, d, causal, "fwd"), flops(b, h, s, d, causal)
        steps = max(3, min(args.steps, int(2e11 // f_all) + 1))
        res = {}
        for _ in range(args.warmup):
            for im in impls.values():
                if im is not None:
                    im.forward(sh)
                    im.backward(d_o, sh)
        rounds = {n: {"fwd": [], "fwdbwd": []} for n in impls}
        for _ in range(3):
            for n, im in impls.items():
                if im is None:
                    continue
                rounds[n]["fwd"].append(timed(lambda i: im.forward(sh), steps, stream))
                rounds[n]["fwdbwd"].append(
                    timed(lambda i: (im.forward(sh), im.backward(d_o, sh)), steps, stream))
        for n, r in rounds.items():
            if not r["fwd"]:
                res[n] = None
                continue
            fm, am = statistics.median(r["fwd"]), statistics.median(r["fwdbwd"])
            res[n] = {"fwd_ms": fm, "fwdbwd_ms": am,
                      "fwd_tflops": f_fwd / fm / 1e9, "fwdbwd_tflops": f_all / am / 1e9,
                      "fwdbwd_frac_ffma": f_all / am / 1e9 / pk["ffma_tflops"]}
        line = {"suite": name, "b": b, "h": h, "s": s, "d": d, "causal": causal, "steps": steps,
                "gflop_fwd": f_fwd / 1e9, "gflop_fwdbwd": f_all / 1e9, **res}
        if res.get("reference_kernel"):
            line["speedup_fwdbwd"] = res["reference_kernel"]["fwdbwd_ms"] / res["ours"]["fwdbwd_ms"]
            line["speedup_fwd"] = res["reference_kernel"]["fwd_ms"] / res["ours"]["fwd_ms"]
        print(json.dumps(line), flush=True)
        del impls, q, k, v, d_o
        torch.cuda.empty_cache()


def timed(fn, steps, stream, sync=None):
    """ms per call of fn(i) over `steps` calls, CUDA events on `stream`."""
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if sync:
        sync()
    torch.cuda.synchronize()
    e0.record(stream)
    for i in range(steps):
        fn(i)
    e1.record(stream)
    e1.synchronize()
    if sync:
        sync()
    return e0.elapsed_time(e1) / steps


def cpu_baseline(b: int, seconds: float = 10.0, max_reps: int = 50):
    """The oracle (a port of the reference's composed CPU path) on all host cores, full canvas
    fwd + bwd repeated until ~`seconds` of CPU work."""
    from oracle import oracle
    qkv, dout = oracle.seeded_inputs(b, H, S, seed=1000, qkv_scale=0.5)
    threads = oracle.max_threads()
    oracle.qkv_forward_backward(qkv, dout, H, SCALE, CAUSAL, threads=threads)  # warm
    t0 = time.perf_counter()
    reps = 0
    while reps < max_reps and (reps == 0 or time.perf_counter() - t0 < seconds):
        oracle.qkv_forward_backward(qkv, dout, H, SCALE, CAUSAL, threads=threads)
        reps += 1
    dt = (time.perf_counter() - t0) / reps
    return {"value": flops(b, H, S, D, CAUSAL) / dt / 1e12, "unit": "TFLOP/s", "cores": threads,
            "kind": "port", "ms_per_step": dt * 1e3,
            "sample": f"full canvas fwd+bwd (b{b} h{H} s{S}), {reps} reps, fp32, "
                      f"oracle/oracle.cpp on {threads} threads"}


def waves(args):
    """Wave quantisation at the canvas shape: the head-dim-64 forward and backward (prep + main, the
    fast workspace) at s = 240, 6 heads, over batches around the canvas's 64. Both kernels run one
    block per SM, 12 blocks per batch row, so a batch of b fills 12 b / 148 waves; the times show
    what the canvas's partial last wave (5.19 waves) costs. CUDA events per call, L2 flushed
    between steps, median of `steps`; one JSON line per batch."""
    from candle_fused_attn import _abi
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    sh = torch.cuda.current_stream(dev).cuda_stream
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # > 126 MB L2
    gen = torch.Generator().manual_seed(0)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    for b in (49, 56, 61, 62, 64, 74):
        x = (torch.randn(b, S, 3 * H * D, generator=gen) * 0.5).to(dev)
        g = torch.randn(b, S, H, D, generator=gen).to(dev)
        st, gst = (x.stride(0), D, x.stride(1)), (g.stride(0), D, g.stride(1))
        p = [x.data_ptr() + 4 * i * H * D for i in range(3)]
        o = torch.empty(b, S, H, D, device=dev)
        lse = torch.empty(b, H, S, device=dev)
        nb = _abi.bwd_workspace_bytes_fast(b, H, S)
        ws = torch.empty(nb, dtype=torch.uint8, device=dev)
        dqkv = torch.empty(b, S, 3, H, D, device=dev)

        def fwd():
            _abi.check(_abi.fwd(p[0], st, p[1], st, p[2], st, o.data_ptr(), lse.data_ptr(), b, H,
                                S, D, SCALE, CAUSAL, sh), "fwd")

        def bwd():
            _abi.check(_abi.bwd(p[0], st, p[1], st, p[2], st, o.data_ptr(), lse.data_ptr(),
                                g.data_ptr(), gst, dqkv.data_ptr(), ws.data_ptr(), nb, b, H, S, D,
                                SCALE, CAUSAL, sh), "bwd")

        for _ in range(args.warmup):
            fwd()
            bwd()
        tf, tb = [], []
        for _ in range(args.steps):
            flush.zero_()
            e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            e[0].record()
            fwd()
            e[1].record()
            bwd()
            e[2].record()
            torch.cuda.synchronize()
            tf.append(e[0].elapsed_time(e[1]))
            tb.append(e[1].elapsed_time(e[2]))
        _abi.check(_abi.bwd_status(ws.data_ptr(), sh), "bwd_status")
        print(json.dumps({"mode": "waves", "batch": b, "heads": H, "seq_len": S, "blocks": 12 * b,
                          "waves": round(12 * b / sms, 3),
                          "fwd_us": round(1000 * statistics.median(tf), 1),
                          "bwd_us": round(1000 * statistics.median(tb), 1)}), flush=True)


def train(args):
    """The reference's training step (examples/tutorial.rs:103-118) at the canvas: qkv =
    x.broadcast_matmul(W_qkv) -> fused_attention_qkv -> mean-squared loss -> backward (the
    attention's dqkv, then W's gradient x^T dqkv) -> W -= 0.1 dW, with x [64, 240, 384], W [384,
    1152] * 0.02 and the target seeded N(0, 1). The projection and its gradient run on the
    tensor-core GEMM (cfa_matmul_f32: split pass + product kernel, + the chunk sum for x^T dqkv),
    the attention on the tensor-core pair; the loss and the update are torch elementwise ops.
    CUDA events, L2 flushed between steps, median of `steps`. Also the two GEMM legs alone
    (roofline against the split-bf16 ceiling) and torch's fp32 matmul (cuBLAS SGEMM, TF32 off) on
    the same shapes. One JSON line."""
    import candle_fused_attn as cfa
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    torch.backends.cuda.matmul.allow_tf32 = False
    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # > 126 MB L2
    hid = H * D
    gen = torch.Generator().manual_seed(0)
    x = torch.randn(B_PER_GPU, S, hid, generator=gen).to(dev)
    w = (torch.randn(hid, 3 * hid, generator=gen) * 0.02).to(dev).requires_grad_(True)
    target = torch.randn(B_PER_GPU, S, hid, generator=gen).to(dev)

    def step(_):
        qkv = cfa.broadcast_matmul(x, w)
        out = cfa.fused_attention_qkv(qkv, H, SCALE, CAUSAL)
        loss = ((out - target) ** 2).mean()
        loss.backward()
        with torch.no_grad():
            w.sub_(0.1 * w.grad)
        w.grad = None
        return loss

    def median_ms(fn, steps):
        ts = []
        for i in range(steps):
            flush.zero_()
            ts.append(timed(fn, 1, stream))
        return statistics.median(ts)

    for i in range(args.warmup):
        step(i)
    step_ms = median_ms(step, args.steps)
    cfa.check_status()

    x2 = x.reshape(-1, hid)
    dy = torch.randn(B_PER_GPU * S, 3 * hid, generator=gen).to(dev)
    wd = w.detach()
    legs = {}
    m, k, n = x2.shape[0], hid, 3 * hid
    gflop = 2.0 * m * k * n / 1e9
    pk = peaks()
    ceiling = pk["bf16_tflops"] / 6
    for name, ours, theirs in (
            ("projection x W", lambda i: cfa.matmul(x2, wd), lambda i: x2 @ wd),
            ("weight gradient x^T dqkv", lambda i: cfa.matmul(x2.t(), dy), lambda i: x2.t() @ dy)):
        for i in range(3):
            ours(i), theirs(i)
        t_o, t_r = median_ms(ours, args.steps), median_ms(theirs, args.steps)
        tf = gflop / t_o
        legs[name] = {"ms": t_o, "tflops": tf, "frac_of_split_ceiling": tf / ceiling,
                      "cublas_fp32_ms": t_r, "speedup_vs_cublas_fp32": t_r / t_o}
    cfa.check_status()
    att = flops(B_PER_GPU, H, S, D, CAUSAL)
    total = att + 2 * 2.0 * m * k * n
    print(json.dumps({
        "mode": "train", "metric": "tutorial training step (x W_qkv, fused attention, MSE, dW)",
        "unit": "ms", "value": step_ms, "higher_is_better": False,
        "tflops": total / (step_ms * 1e-3) / 1e12, "dtype": "f32",
        "config": {"workload": "examples/tutorial.rs:103-118 at the canvas: x [64, 240, 384], "
                               "W_qkv [384, 1152], 6 heads of 64, scale 0.125", "l2": "flushed"},
        "data": "synthetic (seeded N(0,1) x and target, W N(0,1)*0.02)",
        "gemm_legs": legs, "split_ceiling_tflops": ceiling,
        "gpu_launches_per_step": 8,
    }), flush=True)


def config_of(world: int) -> dict:
    """The `config` of both arms' JSON lines (the same workload, the same keys)."""
    return {"workload": WORKLOAD, "global_batch": B_PER_GPU * world, "seq_len": S, "heads": H,
            "head_dim": D, "causal": CAUSAL, "parallelism": f"batch-shard x{world}",
            "l2": f"inputs rotate over {N_SETS} sets of ~190 MB (> 126 MB L2)"}


def run_reference_arm(args, rank, world):
    if rank != 0:
        return
    res = cpu_baseline(B_PER_GPU, seconds=max(2.0, 1.0 * args.steps))
    line = {
        "impl": "reference", "metric": METRIC, "value": res["value"], "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": res["ms_per_step"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1)*0.5)",
        "config": config_of(world),
        "cpu_baseline": {k: res[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": res["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "the reference's CPU composed path (src/lib.rs:241-299) as the C++ oracle port; "
                "candle itself cannot be built here (no cargo)",
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-ref-kernel", action="store_true")
    ap.add_argument("--only", default="", help="suite: run the configs whose name contains this")
    ap.add_argument("--head-dim", type=int, default=D,
                    help="kernels mode: the canvas-shaped projection as heads of this dim (32, 128)")
    ap.add_argument("--pair", choices=["tc", "ffma"], default="tc",
                    help="kernels mode: the head-dim-64 kernel pair of the fwd+bwd step (tc: the "
                         "tensor-core pair, the default; ffma: the CUDA-core pair)")
    ap.add_argument("--mode", choices=["full", "kernels", "suite", "waves", "train"],
                    default="full",
                    help="kernels: warm-up + `steps` plain steps, no timing (for ncu); "
                         "suite: every BASELINE config, ours vs the reference kernel; "
                         "waves: canvas-shaped fwd / bwd times over batches around 64; "
                         "train: the reference's training step with its projection")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference_arm(args, rank, world)
    if args.mode == "suite":
        return suite(args)
    if args.mode == "waves":
        return waves(args)
    if args.mode == "train":
        return train(args)

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    def barrier():
        if dist is not None:
            dist.barrier()

    b = B_PER_GPU
    stream = torch.cuda.current_stream(dev)
    sh = stream.cuda_stream
    if args.mode == "kernels" and args.head_dim != D:
        # the canvas-shaped projection [64, 240, 1152] as 384 / d heads of d (d = 32: the
        # tensor-core pair; d = 128: csrc/hd_ffma.cu)
        from oracle import oracle
        d = args.head_dim
        h = H * D // d
        views = []
        for i in range(N_SETS):
            qkv, dout = oracle.seeded_inputs(b, h, S, 1000 + i, 0.5, d=d)
            x, g = qkv.to(dev), dout.to(dev)
            q, k, v = oracle.qkv_views(x, h)
            views.append(OursViews(q, k, v, oracle.heads_view(g, h), CAUSAL))
        for i in range(args.warmup + args.steps):
            vw = views[i % N_SETS]
            vw.forward(sh)
            vw.backward(vw.d_o, sh)
        torch.cuda.synchronize()
        return
    sets = []
    for i in range(N_SETS):
        qkv, dout = make_inputs(rank * N_SETS + i, b)
        sets.append(OursStep(qkv.to(dev), dout.to(dev),
                             args.pair if args.mode == "kernels" else "tc"))
    torch.cuda.synchronize()

    def step(i):
        st = sets[i % N_SETS]
        st.fwd(sh)
        st.bwd(sh)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()

    if args.mode == "kernels":  # a fixed, short launch sequence for ncu
        for i in range(args.steps):
            step(i)
        torch.cuda.synchronize()
        if dist is not None:
            dist.destroy_process_group()
        return

    # device-resident throughput, K steps between barriers, max over ranks. The clock sampler
    # runs through a >= 1 s loaded lead-in and the timed region (which alone can be ~10 ms).
    with Clocks(local) as clk:
        clk.wait_first()
        t_end, i = time.time() + 1.0, 0
        while time.time() < t_end:
            step(i)
            i += 1
            if i % 64 == 0:
                torch.cuda.synchronize()
        ms = timed(step, args.steps, stream, sync=barrier)
    ms_t = torch.tensor([ms], device=dev)
    if dist is not None:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = float(ms_t.item())
    total_flops = flops(b * world, H, S, D, CAUSAL)
    value = total_flops / (ms_max * 1e-3) / 1e12

    # per-kernel split: forward alone, backward alone (prep + main), same rotation
    fwd_ms = timed(lambda i: sets[i % N_SETS].fwd(sh), args.steps, stream)
    bwd_ms = timed(lambda i: sets[i % N_SETS].bwd(sh), args.steps, stream)
    if sets[0].abi.fwd_status(sh) != sets[0].abi.CFA_OK:
        raise RuntimeError("tensor-core forward: a bounded wait expired")

    # e2e through the public API with pinned host buffers: HostPipeline streams batch chunks
    # through H2D / kernels / D2H on three streams (the timed region spans every copy).
    import candle_fused_attn as cfa
    from candle_fused_attn.host_pipeline import HostPipeline
    hq = [s.qkv.cpu().pin_memory() for s in sets]
    hg = [s.dout.cpu().pin_memory() for s in sets]
    ho = torch.empty(b, S, H * D).pin_memory()
    hd = torch.empty(b, S, 3 * H * D).pin_memory()
    pipe = HostPipeline(b, H, S, SCALE, CAUSAL, dev, chunks=1, slots=2)

    def e2e_timed(steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        e0.record(pipe.h2d)
        for i in range(steps):
            pipe.step(hq[i % N_SETS], hg[i % N_SETS], ho, hd)
        pipe.record_done(e1)
        e1.synchronize()
        barrier()
        return e0.elapsed_time(e1) / steps

    for i in range(args.warmup):
        pipe.step(hq[i % N_SETS], hg[i % N_SETS], ho, hd)
    pipe.synchronize()
    e2e_ms = e2e_timed(args.steps)
    e2e_t = torch.tensor([e2e_ms], device=dev)
    if dist is not None:
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
    e2e_ms = float(e2e_t.item())

    # the floor e2e is measured against: the same bytes, both directions at once, no kernels (all
    # ranks copy concurrently, as in the e2e; the host side of a box is shared between them)
    fq, fg = torch.empty_like(sets[0].qkv), torch.empty_like(sets[0].dout)

    def copy_step(i):
        cur = torch.cuda.current_stream()
        pipe.h2d.wait_stream(cur)
        pipe.d2h.wait_stream(cur)
        with torch.cuda.stream(pipe.h2d):
            fq.copy_(hq[i % N_SETS], non_blocking=True)
            fg.copy_(hg[i % N_SETS], non_blocking=True)
        with torch.cuda.stream(pipe.d2h):
            ho.copy_(sets[i % N_SETS].dout.view(b, S, H * D), non_blocking=True)
            hd.copy_(sets[i % N_SETS].qkv.view(b, S, 3 * H * D), non_blocking=True)
        cur.wait_stream(pipe.h2d)
        cur.wait_stream(pipe.d2h)

    for i in range(3):
        copy_step(i)
    floor_ms = timed(copy_step, args.steps, torch.cuda.current_stream(), sync=barrier)
    floor_t = torch.tensor([floor_ms], device=dev)
    if dist is not None:
        dist.all_reduce(floor_t, op=dist.ReduceOp.MAX)
    floor_ms = float(floor_t.item())
    del fq, fg

    # the same through fused_attention_qkv + autograd, one whole-batch call, copies not overlapped
    def autograd_step(i):
        x = hq[i % N_SETS].to(dev, non_blocking=True).requires_grad_(True)
        g = hg[i % N_SETS].to(dev, non_blocking=True)
        o = cfa.fused_attention_qkv(x, H, SCALE, CAUSAL)
        o.backward(g)
        ho.copy_(o.detach(), non_blocking=True)
        hd.copy_(x.grad, non_blocking=True)

    for i in range(args.warmup):
        autograd_step(i)
    autograd_ms = timed(autograd_step, args.steps, stream, sync=barrier)

    # the reference's own kernels on the same GPU, alternating rounds with ours
    ref = None
    if rank == 0 and not args.no_ref_kernel:
        from baseline import ref_kernel
        if ref_kernel.available():
            rs = [ref_kernel.RefQkv(s.qkv, H, SCALE, CAUSAL) for s in sets]

            def ref_step(i):
                r = rs[i % N_SETS]
                r.forward(sh)
                r.backward(sets[i % N_SETS].dout, sh)

            for i in range(args.warmup):
                ref_step(i)
            ours_r, ref_r = [], []
            for _ in range(3):
                ref_r.append(timed(ref_step, args.steps, stream))
                ours_r.append(timed(step, args.steps, stream))
            ref_fwd = timed(lambda i: rs[i % N_SETS].forward(sh), args.steps, stream)
            ref = {"ms_per_step": statistics.median(ref_r),
                   "tflops": flops(b, H, S, D, CAUSAL) / statistics.median(ref_r) / 1e9,
                   "fwd_ms": ref_fwd,
                   "ours_ms_same_rounds": statistics.median(ours_r),
                   "speedup": statistics.median(ref_r) / statistics.median(ours_r),
                   "source": "kernels/fused_attn.cu (reference v0.4.0) built from source for "
                             "sm_100a, launched as src/cuda.rs:140-260"}

    if dist is not None:
        barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    pk = peaks()
    try:  # DRAM bytes of one backward call from the committed ncu capture (profiles/)
        traffic = json.loads((ROOT / "profiles" / "roofline_traffic.json").read_text())
        traffic = float(traffic["dram_bytes_per_call"])
    except (OSError, ValueError, KeyError):
        traffic = None
    bwd_flops = flops(b, H, S, D, CAUSAL, "bwd")
    achieved = bwd_flops / (bwd_ms * 1e-3) / 1e12
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1)*0.5 qkv, N(0,1) dO)",
        "config": config_of(world),
        "tflops_per_gpu": value / world,
        "fwd_ms": fwd_ms, "bwd_ms": bwd_ms,
        "fwd_tflops": flops(b, H, S, D, CAUSAL, "fwd") / (fwd_ms * 1e-3) / 1e12,
        "e2e": {"value": total_flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": (sets[0].qkv.numel() + sets[0].dout.numel()) * 4,
                "d2h_bytes_per_step": (ho.numel() + hd.numel()) * 4,
                "path": "candle_fused_attn.HostPipeline (pinned host qkv, dO in; O, dqkv out; "
                        "1 chunk per step, 2 buffer slots over H2D / kernel / D2H streams: "
                        "consecutive steps overlap their copies)",
                "copy_floor_ms": floor_ms,
                "copy_floor": "the same bytes copied both ways at once with no kernel, every "
                              "rank concurrently, max over ranks",
                "autograd_ms_per_step": autograd_ms,
                "autograd_path": "fused_attention_qkv + autograd backward, whole batch, copies "
                                 "not overlapped"},
        "roofline": {"bound": "tensor",
                     "pipe": "tcgen05 bf16 (fp32 operands as 3 bf16 parts, 6 products per fp32 "
                             "product, one TMEM accumulator per 64-element window, small products "
                             "first, promoted into fp32 registers)",
                     "kernel": "backward (prep + main, one cfa_bwd_f32_d64 call: bwd_tc_kernel)",
                     "achieved": achieved, "peak": pk["bf16_tflops"] / 6, "unit": "TFLOP/s",
                     "frac": achieved / (pk["bf16_tflops"] / 6), "traffic": traffic,
                     "traffic_unit": "bytes per backward call (ncu, profiles/roofline_traffic.json)",
                     "peak_source": f"MEASURED_PEAKS.json bf16_tflops {pk['bf16_tflops']} / 6 "
                                    "split products",
                     "ffma_peak": pk["ffma_tflops"], "ffma_frac": achieved / pk["ffma_tflops"],
                     "ffma_peak_source": pk["source"],
                     "fwd_frac": flops(b, H, S, D, CAUSAL, "fwd") / (fwd_ms * 1e-3) / 1e12
                     / (pk["bf16_tflops"] / 6)},
        "gpu_launches": 3 * args.steps,
        "clocks": clk.summary(),
        "ref_kernel": ref,
    }
    if not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline(b)
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
