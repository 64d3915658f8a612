"""Connect4 ResNet training on the GPU: the loss and its gradient against
torch autograd on an independent fp64 restatement (BN in inference form,
statistics fixed), Adam against torch.optim.Adam on the trained entries,
fixed BN statistics, bit-for-bit reproducible steps, a loss that falls under
INeuralNet::train, and predictions that follow the new weights.

Tolerances: loss terms 1e-5 relative; gradient max-abs error 1e-4 of the
largest gradient entry, and per tensor 2e-3 of that tensor's largest entry
(fp32 accumulation through 21 convolutions against fp64); weights after
Adam 1e-6 (same gradients, fp32 against fp32)."""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

import graphzero_b200 as gz
import oracle
from helpers import res_blob_views, resnet_frozen_mask, torch_resnet, torch_resnet_loss

pytestmark = pytest.mark.gpu
G = gz.CONNECT4
BOUNDS = json.loads((Path(__file__).resolve().parent / "golden" / "rounding_bounds.json").read_text())["resnet"]


def batch(n, seed):
    boards, side = gz.synth_positions(G, n, seed=seed)
    rng = np.random.default_rng(seed)
    pi = rng.dirichlet(np.full(7, 0.5), size=n).astype(np.float32)
    v = rng.uniform(-1, 1, n).astype(np.float32)
    return boards, side, pi, v


def dev(*arrays):
    return [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in arrays]


def resnet(n, seed=81):
    net = gz.Net(G, gz.RESNET, max_batch=n)
    net.load_weights(gz.synth_weights(G, gz.RESNET, seed=seed, bias_scale=0.3))
    return net


@pytest.mark.parametrize("n", [1, 6, 37])
def test_resnet_gradient_matches_autograd(cuda, n):
    w = gz.synth_weights(G, gz.RESNET, seed=81, bias_scale=0.3)
    net = resnet(n)
    b, s, pi, v = batch(n, seed=82 + n)
    d = dev(b, s, pi, v)
    grad = torch.full((net.weight_count(),), float("nan"), device="cuda")
    lp, lv = net.loss_grad(*d, n, grad)
    rlp, rlv, rgrad = torch_resnet_loss(w, b, s, pi, v)
    assert abs(lp - rlp) <= 1e-5 * max(1.0, abs(rlp)), (lp, rlp)
    assert abs(lv - rlv) <= 1e-5 * max(1.0, abs(rlv)), (lv, rlv)
    g = grad.cpu().numpy()
    assert np.isfinite(g).all()
    assert (g[resnet_frozen_mask()] == 0).all()
    scale = np.abs(rgrad).max()
    assert np.abs(g - rgrad).max() <= 1e-4 * scale, (np.abs(g - rgrad).max(), scale)
    for name, (off, sh) in res_blob_views().items():
        k = int(np.prod(sh))
        ref = rgrad[off:off + k]
        if np.abs(ref).max() > 1e-3 * scale:
            assert np.abs(g[off:off + k] - ref).max() <= 2e-3 * np.abs(ref).max(), name
    grad2 = torch.zeros_like(grad)
    assert net.loss_grad(*d, n, grad2) == (lp, lv)
    assert torch.equal(grad, grad2)
    net.check()


def test_resnet_adam_matches_torch_and_keeps_bn_statistics(cuda):
    n = 32
    w = gz.synth_weights(G, gz.RESNET, seed=81, bias_scale=0.3)
    net = resnet(n)
    d = dev(*batch(n, seed=84))
    frozen = resnet_frozen_mask()
    cfg = gz.train_config(learning_rate=2e-3, weight_decay=1e-4)
    p = torch.tensor(w[~frozen], requires_grad=True)
    opt = torch.optim.Adam([p], lr=2e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-4)
    for _ in range(3):
        g = torch.zeros(net.weight_count(), device="cuda")
        net.loss_grad(*d, n, g)
        net.train_step(*d, n, cfg)
        p.grad = g.cpu()[torch.from_numpy(~frozen)]
        opt.step()
        now = net.save_weights()
        assert np.abs(now[~frozen] - p.detach().numpy()).max() < 1e-6
        assert np.array_equal(now[frozen], w[frozen])
    net.check()


def teacher_examples(n, seed):
    """Canonical-board examples whose targets are another ResNet's outputs."""
    boards, side = gz.synth_positions(G, n, seed=seed + 1)
    tw = gz.synth_weights(G, gz.RESNET, seed=seed, bias_scale=0.5)
    o = res_blob_views()
    p, sh = o["pol_fc"]
    tw[p:p + int(np.prod(sh))] *= 8.0  # a teacher policy far from uniform
    tpi, tv = torch_resnet(tw, boards, side)
    ex = np.zeros(n, gz.EXAMPLE_DTYPE)
    ex["board"][:, :42] = boards * side[:, None]
    ex["pi"][:, :7] = tpi
    ex["v"] = tv
    return ex


def test_resnet_training_reduces_the_loss_and_predictions_follow(cuda):
    ex = teacher_examples(512, seed=90)
    net = gz.Net(G, gz.RESNET, max_batch=512)
    net.load_weights(gz.synth_weights(G, gz.RESNET, seed=91))
    first = net.train(ex, gz.train_config(epochs=1, learning_rate=1e-3))
    last = net.train(ex, gz.train_config(epochs=8, learning_rate=1e-3, seed=9))
    assert last.steps == 9 * (512 // 64)
    tp = ex["pi"][:, :7].astype(np.float64)
    ent = float(-(tp * np.log(np.maximum(tp, 1e-30))).sum(1).mean())
    kl0, kl1 = first.policy_loss - ent, last.policy_loss - ent
    assert kl1 < kl0 and last.value_loss < first.value_loss, (kl0, kl1, first.value_loss, last.value_loss)
    assert kl1 + last.value_loss < 0.8 * (kl0 + first.value_loss), (kl0, kl1, first.value_loss, last.value_loss)
    # the tensor-core forward (fp16 operands) uses the new weights
    w = net.save_weights()
    boards, side = gz.synth_positions(G, 64, seed=92)
    pi, v = net.predict_host(boards, side)
    opi, ov = oracle.resnet_forward(w, boards, side)
    tol = max(1e-3, 1.5 * BOUNDS["fp16"])
    assert np.abs(pi - opi).max() < tol and np.abs(v - ov).max() < tol
    net.check()


def test_resnet_forward_after_a_step_follows_its_rounding_model(cuda):
    """One Adam step moves every trained weight by about lr, coherently with
    the gradient; rounded to nearest in fp16 such weights would put the
    policy 5.0e-3 from the oracle on these positions (simulated), so the
    pack kernel rounds them stochastically by a hash of their blob index
    (simulated: 8.2e-4; 1.3e-3 before the step, the tower's activation
    floor).  The tensor-core forward on the stepped weights is held to 1.5x
    the CPU rounding simulation of its formats (tests/rounding_sim.py) and
    must stay under the round-to-nearest simulation."""
    from rounding_sim import resnet_forward_rounded

    n = 8
    w = gz.synth_weights(G, gz.RESNET, seed=0x6A5A)
    boards, side = gz.synth_positions(G, n, seed=0x6A5A + 1)
    net = gz.Net(G, gz.RESNET, max_batch=n)
    net.load_weights(w)
    d = dev(boards, side, np.full((n, 7), 1.0 / 7, np.float32), np.zeros(n, np.float32))
    net.train_step(*d, n, gz.train_config(learning_rate=1e-3))
    w2 = net.save_weights()
    pi, v = net.predict_host(boards, side)
    opi, ov = oracle.resnet_forward(w2, boards, side)
    err = max(float(np.abs(pi - opi).max()), float(np.abs(v - ov).max()))
    sims = {}
    for wround in ("sr", "rn"):
        spi, sv = resnet_forward_rounded(w2, boards, side, op="fp16", wround=wround)
        sims[wround] = max(float(np.abs(spi - opi).max()), float(np.abs(sv - ov).max()))
    assert err <= 1.5 * sims["sr"] and err < sims["rn"], (err, sims)
    net.check()
