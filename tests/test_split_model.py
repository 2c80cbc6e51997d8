# SPDX-License-Identifier: MIT OR Apache-2.0
"""The accumulation scheme of the tensor-core pair, checked on its numerical model (CPU).

The tensor core's fp32 accumulation truncates (measured on the B200 by baseline/tc_accum_probe.cu),
so a split-precision path only meets the north star's bar -- normwise error against fp64 at or below
plain sequential-FFMA fp32 on every output -- if the truncating sums run over short windows in the
right order. baseline/split_precision_model.py models the attention forward and backward with each
scheme's GEMMs; this test pins the two facts the kernels (csrc/fwd_tc.cu, csrc/bwd_tc.cu) rest on,
on one seeded canvas-shaped (b, h) slice:

- one accumulator per 64-element window, the five small products of every K-step first and the
  high-order A0 B0 steps last, each window promoted into fp32 registers: at or below FFMA on O, dQ,
  dK and dV;
- the same accumulator fed in plain step order: above FFMA (the order is what makes it work).

It also checks, on the same model, that a forward run as two online-softmax halves merged by one
log-sum-exp combine (a way to split the last wave's tiles over two SMs) keeps O's accuracy.

The measured counterpart on the GPU is tests/test_fwd_tc_gpu.py::test_pair_accuracy_vs_ffma."""

import importlib.util
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def model():
    spec = importlib.util.spec_from_file_location(
        "split_precision_model", ROOT / "baseline" / "split_precision_model.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_small_first_window_at_or_below_ffma(model):
    schemes = [("ffma", model.ffma_gemm), ("small first", model.tc_small_first),
               ("step order", lambda a, b: model.tc_promoted(a, b, W=4, sep=False))]
    err = model.normwise_errors(schemes, n_slices=1)
    for i, out in enumerate("O dQ dK dV".split()):
        assert err["small first"][i] <= err["ffma"][i], (out, err)
        assert err["step order"][i] > err["ffma"][i], (out, err)


def test_forward_in_two_halves_keeps_its_accuracy(model):
    # The planned wave-tail split: every forward tile as two online-softmax halves merged by one
    # log-sum-exp combine. Modelled on the pair's product scheme, O's error against fp64 must stay
    # where the single pass has it (and below plain FFMA).
    err = model.halves_errors(n_slices=2)
    assert err["pair halves"] <= 1.05 * err["pair whole"], err
    assert err["pair halves"] < err["ffma whole"], err
