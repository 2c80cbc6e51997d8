# SPDX-License-Identifier: MIT OR Apache-2.0
"""bench.py's reference arm on the CPU: `--impl reference` times the reference's CPU path (the C++
oracle port) and prints one JSON line with the keys the driver reads; under torchrun only rank 0
runs and prints, and every rank exits 0. Needs no GPU."""

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
ARGS = ["bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3"]


def _lines(out):
    return [json.loads(l) for l in out.splitlines() if l.startswith("{")]


def _check(line, n):
    assert line["impl"] == "reference"
    assert line["n_gpus"] == n and line["steps"] == 1 and line["warmup"] == 3
    assert line["value"] > 0 and line["higher_is_better"] is True
    assert line["unit"] == "TFLOP/s" and line["dtype"] == "f32"
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"], "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_reference_arm_one_process():
    r = subprocess.run([sys.executable] + ARGS, cwd=ROOT, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _lines(r.stdout)
    assert len(lines) == 1
    _check(lines[0], 1)


def test_reference_arm_two_ranks_print_once():
    env = dict(os.environ, OMP_NUM_THREADS="1")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", "29547"] + ARGS + ["--gpus", "2"]
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _lines(r.stdout)
    assert len(lines) == 1
    _check(lines[0], 2)
