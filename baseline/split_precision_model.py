# SPDX-License-Identifier: MIT OR Apache-2.0
"""Measurement tooling (CPU): a numerical model of split-precision tensor-core GEMMs inside the
attention forward + backward, against plain sequential-FFMA fp32, both scored normwise against
fp64 on canvas-shaped slices (s = 240, d = 64, seeded N(0,1)*0.5 inputs).

Schemes: bf16 x3 split with 6 or 9 products, tf32 x2 (3 products) / x3 (6 products); the MMA
accumulation modelled as round-to-nearest or truncating, into one accumulator or separate
high/low-order accumulators; and "promoted" variants, in which the (truncating) TMEM accumulators
start fresh every W MMA steps and each window's sums are added into fp32 registers with
round-to-nearest (W = 4 steps of 16 = 64 elements); and the one-accumulator window with the small
products first and the high-order ones last, the scheme csrc/fwd_tc.cu and csrc/bwd_tc.cu use.

    python baseline/split_precision_model.py
"""
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
from oracle import oracle  # noqa: E402  (the seeded input generator)
torch.manual_seed(0)

def rz32(x):  # round float64 -> float32 toward zero
    y = x.float().double()
    over = y.abs() > x.abs()
    y2 = torch.nextafter(y.float(), torch.zeros_like(y.float())).double()
    return torch.where(over, y2, y)

def rn32(x): return x.float().double()

def split_bf16(x, n):
    parts = []; r = x.double()
    for _ in range(n):
        p = r.to(torch.bfloat16).double(); parts.append(p); r = r - p
    return parts

def split_tf32(x, n):
    parts=[]; r=x.double()
    for _ in range(n):
        # tf32: 10 explicit mantissa bits, RN
        f = r.float(); i = f.view(torch.int32)
        i = ((i + 0x1000) & ~0x1FFF)
        p = i.view(torch.float32).double(); parts.append(p); r = r - p
    return parts

def tc_gemm(A, B, scheme, rnd, K=16, sep=True):
    # A [m,k], B [k,n] fp32 values (as float64). returns fp32 values (float64 container)
    kind, n = scheme
    sp = split_bf16 if kind == 'bf16' else split_tf32
    As, Bs = sp(A, n), sp(B, n)
    if kind == 'bf16' and n == 3: pairs = [(0,0),(0,1),(1,0),(0,2),(1,1),(2,0)]
    elif kind == 'bf16' and n == 2: pairs = [(0,0),(0,1),(1,0)]
    elif kind == 'tf32' and n == 2: pairs = [(0,0),(0,1),(1,0)]
    elif kind == 'bf16' and n == 9: pairs = [(i,j) for i in range(3) for j in range(3)]; As, Bs = sp(A,3), sp(B,3)
    elif kind == 'tf32' and n == 3: pairs = [(0,0),(0,1),(1,0),(0,2),(1,1),(2,0)]
    m, kk = A.shape; nn = B.shape[1]
    big = torch.zeros(m, nn, dtype=torch.float64); small = torch.zeros(m, nn, dtype=torch.float64)
    for c in range(0, kk, K):
        for (i, j) in pairs:
            part = As[i][:, c:c+K] @ Bs[j][c:c+K, :]   # exact-ish in fp64
            if sep and (i, j) != (0, 0): small = rnd(small + part)
            else: big = rnd(big + part)
    return rnd(big + small) if sep else big

PAIRS6 = [(0, 0), (0, 1), (1, 0), (0, 2), (1, 1), (2, 0)]


def tc_promoted(A, B, kind='bf16', n=3, K=16, W=4, sep=True, tmem_rnd=None):
    """MMA steps of K reduction elements; TMEM accumulators (big / small, or one) fresh every W
    steps and truncating per step; at each window's end its sums are added into fp32 registers
    round-to-nearest; the result is big + small, round-to-nearest."""
    tmem_rnd = tmem_rnd or rz32
    sp = split_bf16 if kind == 'bf16' else split_tf32
    As, Bs = sp(A, n), sp(B, n)
    pairs = PAIRS6 if n == 3 else [(0, 0), (0, 1), (1, 0)]
    m, kk = A.shape; nn = B.shape[1]
    rb = torch.zeros(m, nn, dtype=torch.float64); rs = torch.zeros_like(rb)
    tb = torch.zeros_like(rb); ts = torch.zeros_like(rb); steps = 0
    for c in range(0, kk, K):
        for (i, j) in pairs:
            part = As[i][:, c:c+K] @ Bs[j][c:c+K, :]
            if sep and (i, j) != (0, 0): ts = tmem_rnd(ts + part)
            else: tb = tmem_rnd(tb + part)
        steps += 1
        if steps == W or c + K >= kk:
            rb = rn32(rb + tb); rs = rn32(rs + ts)
            tb = torch.zeros_like(rb); ts = torch.zeros_like(rb); steps = 0
    return rn32(rb + rs) if sep else rb


def tc_small_first(A, B, K=16, W=4):
    """The tensor-core pair's scheme (csrc/fwd_tc.cu, csrc/bwd_tc.cu): bf16 x3, 6 products, ONE
    truncating TMEM accumulator per window of W steps; within a window the five small products of
    every step are issued first and the W high-order A0 B0 steps last; each window is added into
    fp32 registers round-to-nearest."""
    As, Bs = split_bf16(A, 3), split_bf16(B, 3)
    m, kk = A.shape; nn = B.shape[1]
    r = torch.zeros(m, nn, dtype=torch.float64)
    for w0 in range(0, kk, K * W):
        steps = range(w0, min(kk, w0 + K * W), K)
        t = torch.zeros_like(r)
        for c in steps:
            for (i, j) in PAIRS6[1:]:
                t = rz32(t + As[i][:, c:c+K] @ Bs[j][c:c+K, :])
        for c in steps:
            t = rz32(t + As[0][:, c:c+K] @ Bs[0][c:c+K, :])
        r = rn32(r + t)
    return r


def ffma_gemm(A, B):  # sequential fp32 fma over k: emulate with float64 product + rn32 each step
    m, kk = A.shape; nn = B.shape[1]; acc = torch.zeros(m, nn, dtype=torch.float64)
    for c in range(kk):
        acc = rn32(acc + A[:, c:c+1] * B[c:c+1, :])
    return acc

def attention(q, k, v, do, scale, gemm):
    # composed math with fp32 elementwise, GEMMs by `gemm`. all [s,d] float64 holding fp32 values
    S = rn32(gemm(q, k.T) * scale)
    m = S.max(dim=1, keepdim=True).values
    P = rn32(torch.exp(rn32(S - m)).float().double())
    l = rn32(P.sum(1, keepdim=True))
    P = rn32(P / l)
    O = gemm(P, v)
    L = rn32(m + torch.log(l))
    # backward (recompute P from L)
    P2 = rn32(torch.exp(rn32(rn32(gemm(q, k.T) * scale) - L)))
    dV = gemm(P2.T.contiguous(), do)
    dP = gemm(do, v.T.contiguous())
    D = rn32((do * O).sum(1, keepdim=True))
    dS = rn32(P2 * rn32(dP - D))
    dQ = rn32(gemm(dS, k) * scale)
    dK = rn32(gemm(dS.T.contiguous(), q) * scale)
    return O, dQ, dK, dV

SCHEMES = [
    ('ffma', ffma_gemm),
    ('bf16x3(6) RN sep', lambda A,B: tc_gemm(A,B,('bf16',3),rn32)),
    ('bf16x3(6) RZ sep', lambda A,B: tc_gemm(A,B,('bf16',3),rz32)),
    ('bf16x3(6) RZ one acc', lambda A,B: tc_gemm(A,B,('bf16',3),rz32,sep=False)),
    ('bf16x9 RZ sep', lambda A,B: tc_gemm(A,B,('bf16',9),rz32)),
    ('tf32x2(3) RN sep', lambda A,B: tc_gemm(A,B,('tf32',2),rn32,K=8)),
    ('tf32x3(6) RZ sep', lambda A,B: tc_gemm(A,B,('tf32',3),rz32,K=8)),
    ('bf16x3(6) RZ sep, promoted W=1', lambda A,B: tc_promoted(A,B,W=1)),
    ('bf16x3(6) RZ sep, promoted W=4', lambda A,B: tc_promoted(A,B,W=4)),
    ('bf16x3(6) RZ one, promoted W=4', lambda A,B: tc_promoted(A,B,W=4,sep=False)),
    ('bf16x3(6) RZ sep, no promotion', lambda A,B: tc_promoted(A,B,W=10**9)),
    ('tf32x2(3) RZ sep, promoted W=2', lambda A,B: tc_promoted(A,B,'tf32',2,8,W=2)),
    ('bf16x3(6) RZ one, small first, W=4', tc_small_first),
]


def normwise_errors(schemes=SCHEMES, n_slices=4):
    """Normwise error against fp64 of O, dQ, dK, dV per scheme, over the first n_slices (b, h)
    slices of the seeded canvas-shaped input (s = 240, d = 64)."""
    qkv, dout = oracle.seeded_inputs(2, 2, 240, 0, 0.5)
    q4, k4, v4 = oracle.qkv_views(qkv, 2); g4 = oracle.heads_view(dout, 2)
    res = {}
    for bh in range(n_slices):
        b, h = divmod(bh, 2)
        q, k, v, do = (t[b, h].double() for t in (q4, k4, v4, g4))
        S = (q@k.T)*0.125; m=S.max(1,keepdim=True).values; P=torch.exp(S-m); l=P.sum(1,keepdim=True); P=P/l; O=P@v
        dV=P.T@do; dP=do@v.T; D=(do*O).sum(1,keepdim=True); dS=P*(dP-D); dQ=dS@k*0.125; dK=dS.T@q*0.125
        truth=(O,dQ,dK,dV)
        for name, gemm in schemes:
            out = attention(q, k, v, do, 0.125, gemm)
            acc = res.setdefault(name, [[0,0] for _ in range(4)])
            for i in range(4):
                acc[i][0] += float(((out[i]-truth[i])**2).sum()); acc[i][1] += float((truth[i]**2).sum())
    return {name: [(a/b)**0.5 for a, b in acc] for name, acc in res.items()}



def online_forward(q, k, v, scale, gemm, halves=False, tile=64):
    """O of the online-softmax forward in fp32 (the tensor-core forward's order: per 64-key tile,
    m and l updated, O rescaled and P V added). halves=True runs the key tiles as two independent
    online passes (first half, second half of the tiles) merged by one log-sum-exp combine -- the
    planned tail split, which every block would run so that a tile's bits do not depend on where
    it lands in the grid."""
    def run(t0, t1):
        m = torch.full((q.shape[0], 1), -float("inf"), dtype=torch.float64)
        l = torch.zeros_like(m)
        o = torch.zeros(q.shape[0], v.shape[1], dtype=torch.float64)
        for t in range(t0, t1):
            kt, vt = k[t * tile:(t + 1) * tile], v[t * tile:(t + 1) * tile]
            s_ = rn32(gemm(q, kt.T.contiguous()) * scale)
            m_new = torch.maximum(m, s_.max(1, keepdim=True).values)
            alpha = rn32(torch.exp(rn32(m - m_new)))
            p_ = rn32(torch.exp(rn32(s_ - m_new)))
            l = rn32(rn32(l * alpha) + rn32(p_.sum(1, keepdim=True)))
            o = rn32(rn32(o * alpha) + gemm(p_, vt))
            m = m_new
        return m, l, o
    nt = (k.shape[0] + tile - 1) // tile
    if not halves:
        m, l, o = run(0, nt)
        return rn32(o / l)
    h = (nt + 1) // 2
    m1, l1, o1 = run(0, h)
    m2, l2, o2 = run(h, nt)
    m = torch.maximum(m1, m2)
    a1, a2 = rn32(torch.exp(rn32(m1 - m))), rn32(torch.exp(rn32(m2 - m)))
    l = rn32(rn32(l1 * a1) + rn32(l2 * a2))
    o = rn32(rn32(o1 * a1) + rn32(o2 * a2))
    return rn32(o / l)


def halves_errors(n_slices=4):
    """Normwise O error against fp64: the online forward on the pair's product scheme, whole vs
    two halves combined (and plain FFMA for scale), over the seeded canvas-shaped slices."""
    qkv, _ = oracle.seeded_inputs(2, 2, 240, 0, 0.5)
    q4, k4, v4 = oracle.qkv_views(qkv, 2)
    acc = {"ffma whole": [0.0, 0.0], "pair whole": [0.0, 0.0], "pair halves": [0.0, 0.0]}
    for bh in range(n_slices):
        b, h = divmod(bh, 2)
        q, k, v = (t[b, h].double() for t in (q4, k4, v4))
        S = (q @ k.T) * 0.125
        P = torch.softmax(S, 1)
        truth = P @ v
        for name, gemm, halves in (("ffma whole", ffma_gemm, False),
                                   ("pair whole", tc_small_first, False),
                                   ("pair halves", tc_small_first, True)):
            out = online_forward(q, k, v, 0.125, gemm, halves)
            acc[name][0] += float(((out - truth) ** 2).sum())
            acc[name][1] += float((truth ** 2).sum())
    return {n: (a / b) ** 0.5 for n, (a, b) in acc.items()}

if __name__ == "__main__":
    if "--halves" in sys.argv:
        for name, e in halves_errors().items():
            print(f"{name:12s} O={e:.3e}")
        sys.exit(0)
    for name, errs in normwise_errors().items():
        print(f"{name:22s} " + " ".join(f"{p}={e:.2e}" for p, e in zip("O dQ dK dV".split(), errs)))
