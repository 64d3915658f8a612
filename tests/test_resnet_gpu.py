"""Connect4 ResNet tower on tensor cores (implicit-GEMM 3x3 convolutions)
against the CPU oracle.

Tolerances (max-abs, policy probabilities and values): the 21-convolution
residual tower with a sharp policy amplifies operand rounding -- bf16
activations 2e-2 (a CPU simulation of the same rounding gives 1.3e-2), fp16
activations 2e-3 (simulation 1.8e-3; measured on B200 8e-4)."""
import numpy as np
import pytest
import torch

import graphzero_b200 as gz
import oracle

pytestmark = pytest.mark.gpu


def run(net, boards, side):
    n = side.shape[0]
    d_b = torch.from_numpy(np.ascontiguousarray(boards)).cuda()
    d_s = torch.from_numpy(np.ascontiguousarray(side)).cuda()
    pi = torch.full((n, 7), float("nan"), device="cuda")
    v = torch.full((n,), float("nan"), device="cuda")
    net.predict_batch(d_b, d_s, n, pi, v)
    torch.cuda.synchronize()
    return pi.cpu().numpy(), v.cpu().numpy()


@pytest.mark.parametrize("prec,tol", [(gz.PREC_BF16, 2e-2), (gz.PREC_FP16, 2e-3)])
def test_resnet_matches_oracle(cuda, prec, tol):
    w = gz.synth_weights(gz.CONNECT4, gz.RESNET, seed=31)
    net = gz.Net(gz.CONNECT4, gz.RESNET, precision=prec, max_batch=512)
    assert net.kernel_name.startswith("resnet_tc_")
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
    assert np.abs(pi[idx] - opi).max() < 2e-2 and np.abs(v[idx] - ov).max() < 2e-2
    net.check()
