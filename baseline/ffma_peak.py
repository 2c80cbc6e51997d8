# SPDX-License-Identifier: MIT OR Apache-2.0
"""Measurement tooling: the B200's fp32 FMA throughput, scalar FFMA vs packed fma.rn.f32x2, from
baseline/ffma_peak.cu (built by `make -C baseline ffma`), with the SM clock sampled alongside.

    make -C baseline ffma && python baseline/ffma_peak.py
"""
import ctypes
import subprocess
from pathlib import Path

import torch

lib = ctypes.CDLL(str(Path(__file__).resolve().parent / "_ref" / "libffma_peak.so"))
lib.ffma_peak_run.restype = ctypes.c_float
lib.ffma_peak_run.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                              ctypes.c_int]
sms = torch.cuda.get_device_properties(0).multi_processor_count
out = torch.empty(sms * 8 * 256, device="cuda")
iters, reps = 20000, 5
for packed in (0, 1):
    for per_sm in (4, 8):
        blocks = sms * per_sm
        ms = lib.ffma_peak_run(packed, out.data_ptr(), blocks, iters, reps)
        flop = 2.0 * blocks * 256 * iters * 16 * reps
        clk = subprocess.run(["nvidia-smi", "--query-gpu=clocks.sm", "--format=csv,noheader"],
                             capture_output=True, text=True).stdout.strip()
        print(f"{'fma.rn.f32x2' if packed else 'fmaf (FFMA)'}: {blocks} blocks x 256 threads, "
              f"{ms / reps:.3f} ms/launch, {flop / (ms * 1e-3) / 1e12:.1f} TFLOP/s "
              f"(SM clock after: {clk})")
