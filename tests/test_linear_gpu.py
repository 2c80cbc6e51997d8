# SPDX-License-Identifier: MIT OR Apache-2.0
"""The projection next to the path on the tensor-core GEMM (`cfa_matmul_f32`, `matmul`,
`broadcast_matmul`) against the oracle's products.

The reference's training step (examples/tutorial.rs:103-118) computes qkv = x.broadcast_matmul(W)
before fused_attention_qkv and trains W with the gradient x^T dqkv. The oracle restates that
product (every output sums its k products in order by fused multiply-adds) in fp32 and fp64.

Bands, per output element (|A||B| the product of the absolute operands):
- error model: |C - C64| <= (24 + 2 nwin) 2^-24 (|A||B|)_ij, nwin = ceil(k / 64): the split's
  dropped part products (below 2^-25 of |a b|), the truncating tensor-core sums inside one
  64-element window (at most 4 steps at the window's magnitude, 20 at 2^-8 of it) and one
  round-to-nearest per window fold and per K chunk.
- accuracy: at the training step's shapes the error against fp64 is at or below the oracle's
  fp32 product's (normwise).
Reruns are bit-identical.
"""

import math

import pytest
import torch

import candle_fused_attn as cfa
from oracle import oracle

pytestmark = pytest.mark.gpu

U = 2.0 ** -24


def model_band(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    k = a.shape[1]
    nwin = max(1, math.ceil(k / 64))
    return (24 + 2 * nwin) * U * (a.abs().double() @ b.abs().double())


def check(got: torch.Tensor, a: torch.Tensor, b: torch.Tensor, name: str) -> None:
    r64 = oracle.matmul(a, b, dtype=torch.float64)
    err = (got.double() - r64).abs()
    band = model_band(a, b)
    bad = int((err > band).sum())
    assert bad == 0, f"{name}: {bad} elements beyond the model band (max err {err.max():.2e})"


def operand(x: torch.Tensor, kind: str, dev) -> torch.Tensor:
    """x on the device as: 'row' (row-major), 't' (a transposed view of a column-major copy: the
    other orientation, read in place), 'pad' (row-major rows padded to a larger stride)."""
    if kind == "row":
        return x.to(dev)
    if kind == "t":
        return x.t().contiguous().to(dev).t()
    rows, cols = x.shape
    buf = torch.zeros(rows, cols + 12, device=dev)
    buf[:, :cols] = x.to(dev)
    return buf[:, :cols]


@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (3, 5, 7), (17, 33, 16), (100, 130, 64),
                                   (130, 257, 129), (257, 100, 1000), (128, 128, 128),
                                   (1, 300, 200), (300, 1, 200), (513, 384, 4099)])
@pytest.mark.parametrize("ka,kb", [("row", "row"), ("t", "row"), ("row", "t"), ("t", "t"),
                                   ("pad", "pad")])
def test_shapes_and_orientations(cuda, m, n, k, ka, kb):
    g = torch.Generator().manual_seed(m * 7919 + n * 31 + k)
    a = torch.randn(m, k, generator=g)
    b = torch.randn(k, n, generator=g)
    got = cfa.matmul(operand(a, ka, cuda), operand(b, kb, cuda))
    cfa.check_status()
    assert got.shape == (m, n)
    check(got.cpu(), a, b, f"{m}x{n}x{k} {ka}/{kb}")


def test_zero_k_and_empty(cuda):
    a = torch.empty(5, 0, device=cuda)
    b = torch.empty(0, 7, device=cuda)
    c = cfa.matmul(a, b)
    assert c.shape == (5, 7) and bool((c == 0).all())
    assert cfa.matmul(torch.empty(0, 3, device=cuda), torch.ones(3, 4, device=cuda)).shape == (0, 4)
    assert cfa.matmul(torch.ones(4, 3, device=cuda), torch.empty(3, 0, device=cuda)).shape == (4, 0)


def test_unaligned_and_strided_operands(cuda):
    """Operands at a 1-float offset, with odd row strides, or with no unit stride at all are
    gathered by the split pass in place."""
    g = torch.Generator().manual_seed(5)
    a = torch.randn(70, 45, generator=g)
    b = torch.randn(45, 33, generator=g)
    abuf = torch.zeros(70 * 45 + 1, device=cuda)
    abuf[1:] = a.reshape(-1).to(cuda)
    got = cfa.matmul(abuf[1:].view(70, 45), b.to(cuda))
    check(got.cpu(), a, b, "offset operand")
    bbuf = torch.zeros(45, 33, 3, device=cuda)  # element (k, n) at 99 k + 3 n: no unit stride
    bbuf[:, :, 1] = b.to(cuda)
    got = cfa.matmul(a.to(cuda), bbuf[:, :, 1])
    check(got.cpu(), a, b, "no unit stride")


def test_rerun_bitwise(cuda):
    g = torch.Generator().manual_seed(11)
    a = torch.randn(1000, 384, generator=g).to(cuda)
    b = torch.randn(384, 1152, generator=g).to(cuda)
    c1 = cfa.matmul(a, b)
    c2 = cfa.matmul(a, b)
    assert torch.equal(c1, c2)
    # K chunked (few output tiles): the partial tiles are summed in chunk order, every rerun.
    x = torch.randn(4000, 384, generator=g).to(cuda)
    y = torch.randn(4000, 256, generator=g).to(cuda)
    d1 = cfa.matmul(x.t(), y)
    d2 = cfa.matmul(x.t(), y)
    assert torch.equal(d1, d2)


# The training step's shapes at the canvas (examples/tutorial.rs:103-118 with bench/compare.py's
# trainer geometry: batch 64, seq 240, hidden 384 = 6 heads of 64): x [64, 240, 384],
# W_qkv [384, 1152] * 0.02, and the gradient dqkv [64, 240, 1152].
B, S, HID = 64, 240, 384


def canvas_operands():
    g = torch.Generator().manual_seed(2024)
    x = torch.randn(B, S, HID, generator=g)
    w = torch.randn(HID, 3 * HID, generator=g) * 0.02
    dy = torch.randn(B, S, 3 * HID, generator=g)
    return x, w, dy


def accuracy_vs_oracle(got, a, b, name, rows=None, cols=None):
    """Normwise error against fp64 at or below the oracle's fp32 product's, on a row / column
    subset (the product of a row subset of A, or a column subset of B)."""
    if rows is not None:
        a = a[rows]
        got = got[rows]
    if cols is not None:
        b = b[:, cols]
        got = got[:, cols]
    a, b = a.contiguous(), b.contiguous()
    check(got, a, b, name)
    r64 = oracle.matmul(a, b, dtype=torch.float64)
    r32 = oracle.matmul(a, b)
    ours = (got.double() - r64).norm() / r64.norm()
    theirs = (r32.double() - r64).norm() / r64.norm()
    assert ours <= theirs, f"{name}: normwise {ours:.3e} above the fp32 oracle's {theirs:.3e}"


def test_canvas_projection(cuda):
    x, w, _ = canvas_operands()
    qkv = cfa.broadcast_matmul(x.to(cuda), w.to(cuda))
    cfa.check_status()
    assert qkv.shape == (B, S, 3 * HID)
    accuracy_vs_oracle(qkv.reshape(-1, 3 * HID).cpu(), x.reshape(-1, HID), w, "x W",
                       rows=slice(0, 2048))


def test_canvas_weight_gradient(cuda):
    """dW = x^T dqkv: k = 15360, 27 output tiles -> K cut into chunks."""
    x, _, dy = canvas_operands()
    x2, dy2 = x.reshape(-1, HID), dy.reshape(-1, 3 * HID)
    dw = cfa.matmul(x2.to(cuda).t(), dy2.to(cuda))
    cfa.check_status()
    accuracy_vs_oracle(dw.cpu(), x2.t(), dy2, "x^T dY", cols=slice(0, 160))


def test_canvas_input_gradient(cuda):
    """dx = dqkv W^T (W^T read in place: K contiguous)."""
    _, w, dy = canvas_operands()
    dy2 = dy.reshape(-1, 3 * HID)
    dx = cfa.matmul(dy2.to(cuda), w.to(cuda).t())
    cfa.check_status()
    accuracy_vs_oracle(dx.cpu(), dy2, w.t(), "dY W^T", rows=slice(0, 1024))


def test_broadcast_matmul_autograd(cuda):
    g = torch.Generator().manual_seed(3)
    x = torch.randn(3, 50, 96, generator=g)
    w = torch.randn(96, 200, generator=g) * 0.1
    dy = torch.randn(3, 50, 200, generator=g)
    xd = x.to(cuda).requires_grad_(True)
    wd = w.to(cuda).requires_grad_(True)
    y = cfa.broadcast_matmul(xd, wd)
    y.backward(dy.to(cuda))
    cfa.check_status()
    x2, dy2 = x.reshape(-1, 96), dy.reshape(-1, 200)
    check(y.detach().reshape(-1, 200).cpu(), x2, w, "y")
    check(xd.grad.reshape(-1, 96).cpu(), dy2, w.t().contiguous(), "dx")
    check(wd.grad.cpu(), x2.t().contiguous(), dy2, "dw")


def test_training_step_against_oracle(cuda):
    """One step of the reference's training loop (tutorial.rs:109-117) -- projection, fused
    attention, mean-squared loss, the gradient of W_qkv -- on the device path and on the oracle
    path (oracle product, oracle attention forward and backward, oracle product), batch 2."""
    g = torch.Generator().manual_seed(7)
    b, s, heads, d = 2, 240, 6, 64
    hid = heads * d
    x = torch.randn(b, s, hid, generator=g)
    w = torch.randn(hid, 3 * hid, generator=g) * 0.02
    target = torch.randn(b, s, hid, generator=g)
    scale = 0.125

    wd = w.to(cuda).requires_grad_(True)
    qkv = cfa.broadcast_matmul(x.to(cuda), wd)
    out = cfa.fused_attention_qkv(qkv, heads, scale, False)
    loss = ((out - target.to(cuda)) ** 2).mean()
    loss.backward()
    cfa.check_status()

    # The oracle path: product, attention forward, the loss gradient, backward, product.
    qkv_o = oracle.matmul(x.reshape(-1, hid), w).reshape(b, s, 3 * hid)
    out_o, _, _ = oracle.qkv_forward_backward(qkv_o, torch.zeros(b, s, hid), heads, scale, False)
    dout = 2.0 * (out_o - target) / out_o.numel()
    _, _, dqkv = oracle.qkv_forward_backward(qkv_o, dout, heads, scale, False)
    dw_o = oracle.matmul(x.reshape(-1, hid).t().contiguous(), dqkv.reshape(-1, 3 * hid))

    assert abs(loss.item() - ((out_o - target) ** 2).mean().item()) <= 1e-6 * loss.item()
    dw = wd.grad.cpu()
    rel = (dw - dw_o).norm() / dw_o.norm()
    assert rel < 1e-5, f"dW normwise {rel:.2e} from the oracle path"
