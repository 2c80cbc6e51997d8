# SPDX-License-Identifier: MIT OR Apache-2.0
"""The tensor-core forward (csrc/fwd_tc.cu) against the CPU oracle: the forward of every head-dim-64
call through cfa_fwd_f32_d64 / cfa_fwd_f32 and the Python API.

Same bar as the FFMA forward (tests/parity.rs:161-167, :210-221 and the north star): 1e-5
normwise and a 5e-6 max-abs band (scaled by the output magnitude) against the fp32 composed path
on the reference tests' shapes and edge cases (lengths 1, 7, 33, 97, 129, 240, 300; causal and not;
the fused projection and strided views); bit-identical reruns and batch splits; the backward run
on its outputs within the same band; accuracy against fp64 at or below the FFMA forward's, as the
north star requires of a split-precision tensor-core path; and the device error flag clear.
"""

import pytest
import torch

import candle_fused_attn as cfa
from candle_fused_attn import _abi
from oracle import oracle
from pairs import run_pair

pytestmark = pytest.mark.gpu

BAND_NORMWISE = 1e-5


@pytest.fixture
def tc(cuda):
    return cuda


def status_ok():
    assert _abi.fwd_status(torch.cuda.current_stream().cuda_stream) == _abi.CFA_OK


def check(got, ref, name):
    band = 5e-6 * max(1.0, ref.abs().max().item())
    err = (got - ref).abs().max().item()
    assert err < band, f"{name} max-abs {err:.2e} > {band:.2e}"
    nw = oracle.normwise(got, ref)
    assert nw < BAND_NORMWISE, f"{name} normwise {nw:.2e}"


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("bsh", [(2, 7, 3), (1, 1, 1), (1, 33, 2), (2, 240, 6), (1, 97, 2),
                                 (1, 129, 2), (2, 300, 2)])
def test_forward_matches_cpu(tc, bsh, causal):
    b, s, h = bsh
    qkv, _ = oracle.closed_form_inputs(b, s, h, 64)
    q, k, v = oracle.qkv_views(qkv, h)
    o_ref, l_ref = oracle.forward(q, k, v, 0.125, causal)
    out = cfa.fused_attention_qkv(qkv.to(tc), h, 0.125, causal)
    status_ok()
    check(out.cpu(), o_ref.reshape(b, s, -1), "O")


@pytest.mark.parametrize("causal", [False, True])
def test_strided_views(tc, causal):
    """fused_attention on permuted views of one [b, s, 3, h, 64] tensor (the strided config)."""
    b, s, h = 2, 200, 3
    g = torch.Generator().manual_seed(3)
    x = torch.randn(b, s, 3, h, 64, generator=g)
    q, k, v = (x[:, :, i].permute(0, 2, 1, 3) for i in range(3))
    o_ref, _ = oracle.forward(q, k, v, 0.125, causal)
    xd = x.to(tc)
    qd, kd, vd = (xd[:, :, i].permute(0, 2, 1, 3) for i in range(3))
    out = cfa.fused_attention(qd, kd, vd, 0.125, causal)
    status_ok()
    check(out.transpose(1, 2).cpu(), o_ref, "O")


def test_reruns_and_batch_split_bit_identical(tc):
    qkv, _ = oracle.seeded_inputs(8, 6, 240, 5, 0.5)
    x = qkv.to(tc)
    runs = [cfa.fused_attention_qkv(x, 6, 0.125, False) for _ in range(3)]
    halves = torch.cat([cfa.fused_attention_qkv(x[:4], 6, 0.125, False),
                        cfa.fused_attention_qkv(x[4:], 6, 0.125, False)])
    status_ok()
    for r in runs[1:] + [halves]:
        assert torch.equal(r, runs[0])


@pytest.mark.parametrize("causal", [False, True])
def test_backward_on_tc_forward(tc, causal):
    """The backward recomputes P from the forward's L: gradients within the band."""
    b, s, h = 2, 240, 6
    qkv, w = oracle.closed_form_inputs(b, s, h, 64)
    o_ref, _, g_ref = oracle.qkv_forward_backward(qkv, w, h, 0.125, causal)
    x = qkv.to(tc).requires_grad_(True)
    out = cfa.fused_attention_qkv(x, h, 0.125, causal)
    (out * w.to(tc)).sum().backward()
    status_ok()
    check(out.detach().cpu(), o_ref, "O")
    check(x.grad.cpu(), g_ref, "dqkv")


def test_accuracy_vs_fp64(tc):
    """Canvas-shaped slices: O's normwise error against the fp64 composed path at or below the FFMA
    forward's (the north star's condition for a split-precision tensor-core path)."""
    b, h, s = 8, 6, 240
    qkv, _ = oracle.seeded_inputs(b, h, s, 0, 0.5)
    q, k, v = oracle.qkv_views(qkv, h)
    o64, _ = oracle.forward(q, k, v, 0.125, False, dtype=torch.float64)
    o64 = o64.reshape(b, s, -1)
    x = qkv.to(tc)
    o_tc = cfa.fused_attention_qkv(x, h, 0.125, False).cpu().double()
    status_ok()
    o_ff = run_pair("ffma", qkv, None, h, 0.125, False, tc)[0].cpu().double()
    e_tc, e_ff = oracle.normwise(o_tc, o64), oracle.normwise(o_ff, o64)
    print(f"O vs fp64: tensor cores {e_tc:.3e}, FFMA {e_ff:.3e}")
    assert e_tc <= e_ff, (e_tc, e_ff)


def test_long_causal_slice(tc):
    """s = 1024 causal: 8 query tiles of 128, the diagonal tiles masked inside."""
    b, s, h = 1, 1024, 2
    qkv, _ = oracle.seeded_inputs(b, h, s, 11, 0.5)
    q, k, v = oracle.qkv_views(qkv, h)
    o_ref, _ = oracle.forward(q, k, v, 0.125, True)
    out = cfa.fused_attention_qkv(qkv.to(tc), h, 0.125, True)
    status_ok()
    check(out.cpu(), o_ref.reshape(b, s, -1), "O")


def test_one_pair_per_entry_point(cuda):
    """Head dim 64 has one kernel pair per entry point and no process-wide switch: the Python API
    (with or without autograd) runs the tensor-core pair, bit for bit the C ABI's default entry
    points; the CUDA-core pair is reached only through its own entry points and differs."""
    qkv, dout = oracle.seeded_inputs(2, 6, 240, 9, 0.5)
    x = qkv.to(cuda)
    o_abi, _, g_abi = run_pair("tc", qkv, dout, 6, 0.125, False, cuda)
    o_ffma, _, _ = run_pair("ffma", qkv, dout, 6, 0.125, False, cuda)
    with torch.no_grad():
        o_nograd = cfa.fused_attention_qkv(x, 6, 0.125, False)
    xg = x.clone().requires_grad_(True)
    o_train = cfa.fused_attention_qkv(xg, 6, 0.125, False)
    o_train.backward(dout.to(cuda))
    status_ok()
    assert torch.equal(o_nograd, o_abi) and torch.equal(o_train.detach(), o_abi)
    assert torch.equal(xg.grad, g_abi)
    assert not torch.equal(o_ffma, o_abi)


def test_two_users_mixing_pairs(cuda):
    """Two users in one process, one on each pair, their forwards and backwards interleaved: each
    gets its own pair's results bit for bit (nothing one does changes the other's kernels), and
    both stay within the band of the CPU composed path."""
    b, s, h = 2, 200, 3
    qkv, dout = oracle.seeded_inputs(b, h, s, 21, 0.5)
    o_ref, _, g_ref = oracle.qkv_forward_backward(qkv, dout, h, 0.125, True)
    alone = {p: run_pair(p, qkv, dout, h, 0.125, True, cuda) for p in ("tc", "ffma")}
    # interleaved: user A (tensor cores, through the public API) and user B (the CUDA-core pair)
    xa = qkv.to(cuda).requires_grad_(True)
    oa = cfa.fused_attention_qkv(xa, h, 0.125, True)
    ob, _, gb = run_pair("ffma", qkv, dout, h, 0.125, True, cuda)
    oa.backward(dout.to(cuda))
    status_ok()
    assert torch.equal(oa.detach(), alone["tc"][0]) and torch.equal(xa.grad, alone["tc"][2])
    assert torch.equal(ob, alone["ffma"][0]) and torch.equal(gb, alone["ffma"][2])
    for o, g in ((oa.detach(), xa.grad), (ob, gb)):
        assert oracle.normwise(o.cpu(), o_ref.reshape(b, s, -1)) < BAND_NORMWISE
        assert oracle.normwise(g.cpu(), g_ref.reshape(b, s, -1)) < BAND_NORMWISE


def test_pair_accuracy_vs_ffma(cuda):
    """Forward and backward of the tensor-core pair against the fp64 composed path at the canvas
    shape (8 of its batches): O, dQ, dK, dV each at or below the FFMA pair's error (the north
    star's condition for a split-precision tensor-core path)."""
    b, h, s = 8, 6, 240
    qkv, dout = oracle.seeded_inputs(b, h, s, 0, 0.5)
    o64, _, g64 = oracle.qkv_forward_backward(qkv, dout, h, 0.125, False, dtype=torch.float64)
    g64 = g64.reshape(b, s, 3, h * 64)

    def errors(pair):
        out, _, g = run_pair(pair, qkv, dout, h, 0.125, False, cuda)
        g = g.cpu().double().reshape(b, s, 3, h * 64)
        return {"O": oracle.normwise(out.cpu().double(), o64),
                **{n: oracle.normwise(g[:, :, i], g64[:, :, i]) for i, n in enumerate(("dQ", "dK", "dV"))}}

    e_tc, e_ff = errors("tc"), errors("ffma")
    status_ok()
    print("tensor cores vs fp64:", {k: f"{v:.3e}" for k, v in e_tc.items()})
    print("FFMA         vs fp64:", {k: f"{v:.3e}" for k, v in e_ff.items()})
    for k in e_tc:
        assert e_tc[k] <= e_ff[k], (k, e_tc[k], e_ff[k])
