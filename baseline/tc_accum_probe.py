# SPDX-License-Identifier: MIT OR Apache-2.0
"""Measurement tooling: runs baseline/tc_accum_probe.cu (built by `make -C baseline probe`) on a
B200 and reports how often the tensor core's fp32 accumulation matches a round-to-nearest and a
truncating model, plus two crisp single-product cases around 1.0.

    make -C baseline probe && python baseline/tc_accum_probe.py
"""
import ctypes
import sys
from pathlib import Path

import torch

lib = ctypes.CDLL(sys.argv[1] if len(sys.argv) > 1 else
                  str(Path(__file__).resolve().parent / "_ref" / "libtc_probe.so"))
lib.run_probe.argtypes = [ctypes.c_int] + [ctypes.c_void_p] * 4 + [ctypes.c_int] * 3 + [ctypes.c_void_p]
dev = torch.device("cuda:0")
torch.manual_seed(0)

def rz32(x):
    y = x.float().double()
    over = y.abs() > x.abs()
    y2 = torch.nextafter(y.float(), torch.zeros_like(y.float())).double()
    return torch.where(over, y2, y)

def rn32(x): return x.float().double()

def to_tf32(x):
    i = x.float().contiguous().view(torch.int32)
    return (i & ~0x1FFF).view(torch.float32)

def run(kind, K, N, use_c, scaleA=1.0, Cscale=1.0):
    if kind == 1:
        A = (torch.randn(128, K) * scaleA).to(torch.bfloat16); B = torch.randn(N, K).to(torch.bfloat16)
        kstep = 16
    else:
        A = to_tf32(torch.randn(128, K) * scaleA); B = to_tf32(torch.randn(N, K)); kstep = 8
    C0 = (torch.randn(128, N) * Cscale).float()
    Ad, Bd, Cd = A.to(dev), B.to(dev), C0.to(dev)
    D = torch.zeros(128, N, device=dev); st = torch.zeros(1, dtype=torch.int32, device=dev)
    rc = lib.run_probe(kind, Ad.data_ptr(), Bd.data_ptr(), Cd.data_ptr(), D.data_ptr(), K, N, use_c, st.data_ptr())
    assert rc == 0 and st.item() == 0, (rc, st.item())
    D = D.cpu().double()
    A64, B64 = A.double(), B.double()
    res = {}
    for name, rnd in (("RN", rn32), ("RZ", rz32)):
        acc = C0.double() if use_c else torch.zeros(128, N, dtype=torch.float64)
        for ks in range(K // kstep):
            part = A64[:, ks*kstep:(ks+1)*kstep] @ B64[:, ks*kstep:(ks+1)*kstep].T
            acc = rnd(acc + part)
        res[name] = (acc == D).float().mean().item()
    exact = (C0.double() if use_c else 0) + A64 @ B64.T
    ulp = (exact.float().double() - torch.nextafter(exact.float(), torch.full_like(exact.float(), float('inf'))).double()).abs()
    err = ((D - exact) / ulp)
    return res, err.mean().item(), err.abs().max().item()

for kind in (1, 2):
    for K in (16, 64, 256):
        for use_c in (0, 1):
            for sa, cs in ((1.0, 1.0), (1.0, 100.0), (0.01, 1.0)):
                r, bias, mx = run(kind, K, 64, use_c, sa, cs)
                print(f"kind={'bf16' if kind==1 else 'tf32'} K={K:3d} C={use_c} scaleA={sa} Cscale={cs}: match RN={r['RN']:.4f} RZ={r['RZ']:.4f} | err vs exact in ulps: mean {bias:+.3f} max {mx:.2f}")
# crisp case: C0 = 1.0, one product 0.75 ulp(1) above / below
for sign in (1, -1):
    A = torch.zeros(128, 16).to(torch.bfloat16); B = torch.zeros(64, 16).to(torch.bfloat16)
    A[:, 0] = 1.5 * 2**-12 * sign; B[:, 0] = 2**-12
    C0 = torch.ones(128, 64)
    D = torch.zeros(128, 64, device=dev); st = torch.zeros(1, dtype=torch.int32, device=dev)
    Ad, Bd, Cd = A.to(dev), B.to(dev), C0.to(dev)
    lib.run_probe(1, Ad.data_ptr(), Bd.data_ptr(), Cd.data_ptr(), D.data_ptr(), 16, 64, 1, st.data_ptr())
    v = D[0, 0].item()
    print(f"crisp 1 + {sign}*0.75ulp -> {v!r}  (RN gives {1 + sign*2**-23 if sign>0 else 1 - 2**-24!r}, RZ gives {1.0 if sign>0 else 1 - 2**-24!r})")
    A[:, 0] = 1.0 * 2**-12 * sign; A[:, 1] = 0.5 * 2**-12 * sign; B[:, 1] = 2**-12
    Ad = A.to(dev)
    lib.run_probe(1, Ad.data_ptr(), Bd.data_ptr(), Cd.data_ptr(), D.data_ptr(), 16, 64, 1, st.data_ptr())
    print(f"crisp split into two products -> {D[0,0].item()!r}")
