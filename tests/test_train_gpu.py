"""GAT training on the GPU: the loss and its gradient against torch autograd
on an independent fp64 restatement, Adam against torch.optim.Adam, bit-for-
bit reproducible steps, a loss that falls, the INeuralNet::train path, and
(on two GPUs) the data-parallel step with its NCCL gradient all-reduce
against one GPU stepping on the whole batch.

Tolerances: loss terms 1e-5 relative; gradient max-abs error 1e-4 of the
largest gradient entry (fp32 accumulation through 4-8 layers against fp64);
weights after Adam 1e-6 (same gradients, fp32 against fp32)."""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

import graphzero_b200 as gz
import oracle
from helpers import sharpen, torch_gat_loss

SPEC_TOL = 1e-3  # max-abs bound on policy and value against the oracle

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def batch(game, n, seed):
    boards, side = gz.synth_positions(game, n, seed=seed)
    rng = np.random.default_rng(seed)
    A = gz.game_shape(game).actions
    pi = rng.dirichlet(np.full(A, 0.5), size=n).astype(np.float32)
    v = rng.uniform(-1, 1, n).astype(np.float32)
    return boards, side, pi, v


def dev(*arrays):
    return [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in arrays]


@pytest.mark.parametrize("game,n", [(gz.TICTACTOE, 16), (gz.CONNECT4, 24), (gz.CHESS, 3)])
def test_gradient_matches_autograd(cuda, game, n):
    w = sharpen(game, gz.synth_weights(game, seed=41, bias_scale=0.3))
    net = gz.Net(game, max_batch=n)
    net.load_weights(w)
    b, s, pi, v = batch(game, n, seed=42)
    d = dev(b, s, pi, v)
    grad = torch.zeros(net.weight_count(), device="cuda")
    lp, lv = net.loss_grad(*d, n, grad)
    rlp, rlv, rgrad = torch_gat_loss(game, w, b, s, pi, v)
    assert abs(lp - rlp) <= 1e-5 * max(1.0, abs(rlp)), (lp, rlp)
    assert abs(lv - rlv) <= 1e-5 * max(1.0, abs(rlv)), (lv, rlv)
    g = grad.cpu().numpy()
    assert np.isfinite(g).all()
    scale = np.abs(rgrad).max()
    assert np.abs(g - rgrad).max() <= 1e-4 * scale, (np.abs(g - rgrad).max(), scale)
    # the weights the loss does not reach get exactly zero, the others a
    # gradient of the right size: check each layer's share separately
    from helpers import gat_blob_views
    for name, (off, sh) in gat_blob_views(game).items():
        k = int(np.prod(sh))
        ref = rgrad[off:off + k]
        if np.abs(ref).max() > 1e-3 * scale:
            assert np.abs(g[off:off + k] - ref).max() <= 2e-3 * np.abs(ref).max(), name
    # reproducible bit for bit
    grad2 = torch.zeros_like(grad)
    assert net.loss_grad(*d, n, grad2) == (lp, lv)
    assert torch.equal(grad, grad2)


def test_adam_matches_torch(cuda):
    game, n = gz.CONNECT4, 32
    w = sharpen(game, gz.synth_weights(game, seed=43, bias_scale=0.3))
    net = gz.Net(game, max_batch=n)
    net.load_weights(w)
    d = dev(*batch(game, n, seed=44))
    cfg = gz.train_config(learning_rate=2e-3, weight_decay=1e-4)
    p = torch.tensor(w, requires_grad=True)
    opt = torch.optim.Adam([p], lr=2e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-4)
    for _ in range(3):
        g = torch.zeros(net.weight_count(), device="cuda")
        net.loss_grad(*d, n, g)  # the gradient at the current weights
        net.train_step(*d, n, cfg)  # recomputes it (bit for bit) and applies Adam
        p.grad = g.cpu()
        opt.step()
        assert np.abs(net.save_weights() - p.detach().numpy()).max() < 1e-6
    net.check()


def teacher_examples(game, n, seed):
    """Canonical-board examples whose targets are another net's outputs."""
    teacher = gz.Net(game, precision=gz.PREC_FP32, max_batch=n)
    teacher.load_weights(sharpen(game, gz.synth_weights(game, seed=seed, bias_scale=0.5)))
    boards, side = gz.synth_positions(game, n, seed=seed + 1)
    tpi, tv = teacher.predict_host(boards, side)
    ex = np.zeros(n, gz.EXAMPLE_DTYPE)
    N, A = gz.game_shape(game).nodes, gz.game_shape(game).actions
    ex["board"][:, :N] = boards * side[:, None]
    ex["pi"][:, :A] = tpi
    ex["v"] = tv
    return ex


@pytest.mark.parametrize("game", [gz.TICTACTOE, gz.CONNECT4])
def test_training_reduces_the_loss_and_predictions_follow(cuda, game):
    ex = teacher_examples(game, 512, seed=50)
    net = gz.Net(game, max_batch=512)
    net.load_weights(gz.synth_weights(game, seed=51))
    first = net.train(ex, gz.train_config(epochs=1, learning_rate=2e-3))
    last = net.train(ex, gz.train_config(epochs=12, learning_rate=2e-3, seed=9))
    assert last.steps == 13 * (512 // 64)
    # the policy cross-entropy cannot fall below the targets' entropy: compare
    # the excess over it (the KL divergence to the teacher)
    A = gz.game_shape(game).actions
    tp = ex["pi"][:, :A].astype(np.float64)
    ent = float(-(tp * np.log(np.maximum(tp, 1e-30))).sum(1).mean())
    kl0, kl1 = first.policy_loss - ent, last.policy_loss - ent
    assert kl1 < 0.5 * kl0 and last.value_loss < first.value_loss, (kl0, kl1, first.value_loss, last.value_loss)
    assert kl1 + last.value_loss < 0.8 * (kl0 + first.value_loss)
    # the default forward (tensor cores where the game has them) uses the new weights
    w = net.save_weights()
    boards, side = gz.synth_positions(game, 64, seed=52)
    pi, v = net.predict_host(boards, side)
    opi, ov = oracle.gat_forward(game, w, boards, side)
    assert np.abs(pi - opi).max() < 1e-3 and np.abs(v - ov).max() < 1e-3
    net.check()


@pytest.mark.parametrize("kind", ["gat", "resnet"])
def test_ineuralnet_train_through_the_shim(cuda, kind):
    """INeuralNet::train from the reference's vtable (TrainingExample with
    float board and policy arrays), for both factories' nets."""
    import ctypes as C

    game = gz.CONNECT4
    nn = gz.create_ineuralnet(kind, gz.create_igame("connect4"))
    net_h = gz._lib.gz_shim_net(nn)
    w0 = np.empty(gz.weight_count(game, gz.RESNET if kind == "resnet" else gz.GAT), np.float32)
    gz._check(gz._lib.gz_net_save_weights(net_h, gz._ptr(w0, C.c_float), w0.size))
    ex = teacher_examples(game, 128, seed=60)

    class TE(C.Structure):
        _fields_ = [("board", C.POINTER(C.c_float)), ("pi", C.POINTER(C.c_float)), ("v", C.c_float)]

    boards = ex["board"][:, :42].astype(np.float32).copy()
    pis = ex["pi"][:, :7].astype(np.float32).copy()
    arr = (TE * len(ex))()
    for i in range(len(ex)):
        arr[i].board = boards[i].ctypes.data_as(C.POINTER(C.c_float))
        arr[i].pi = pis[i].ctypes.data_as(C.POINTER(C.c_float))
        arr[i].v = float(ex["v"][i])
    vt = C.cast(nn, C.POINTER(C.c_void_p * 9)).contents
    train = C.CFUNCTYPE(None, C.c_void_p, C.POINTER(TE), C.c_int)(vt[2])
    train(nn, arr, len(ex))
    w1 = np.empty_like(w0)
    gz._check(gz._lib.gz_net_save_weights(net_h, gz._ptr(w1, C.c_float), w1.size))
    assert np.isfinite(w1).all() and not np.array_equal(w0, w1)
    if kind == "resnet":  # BN statistics stay fixed
        from helpers import resnet_frozen_mask
        frozen = resnet_frozen_mask()
        assert np.array_equal(w1[frozen], w0[frozen])


def _free_port():
    sk = socket.socket()
    sk.bind(("127.0.0.1", 0))
    p = sk.getsockname()[1]
    sk.close()
    return p


def _dp_weights(G, kind):
    if kind == G.RESNET:
        return G.synth_weights(G.CONNECT4, G.RESNET, seed=70, bias_scale=0.3)
    return sharpen(G.CONNECT4, G.synth_weights(G.CONNECT4, seed=70, bias_scale=0.3))


def _dp_config(G, kind):
    # The ResNet has many weights whose gradient is a sum that cancels to
    # almost nothing; Adam's first steps move each weight by about lr
    # whatever its gradient's size, so a different summation order (two half
    # batches against one whole batch) can move such a weight by a different
    # fraction of lr.  With eps = 1 the update is lr * m, proportional to the
    # averaged gradient, and the comparison checks the all-reduce and the
    # averaging themselves.
    if kind == G.RESNET:
        return G.train_config(learning_rate=1e-3, eps=1.0)
    return G.train_config(learning_rate=1e-3)


def _dp_worker(rank, world, port, out, kind):
    sys.path[:0] = [str(ROOT), str(ROOT / "oracle"), str(ROOT / "tests")]
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch as T

    import graphzero_b200 as G
    from graphzero_b200 import dist as D

    T.cuda.set_device(rank)
    info = D.rank_info()
    D.init_process_group("gloo", info, timeout_s=60.0)
    game, n = G.CONNECT4, 16
    net = G.Net(game, kind, device=rank, max_batch=n)
    net.load_weights(_dp_weights(G, kind))
    uid = D.share_bytes(G.nccl_unique_id() if rank == 0 else None)
    comm = G.nccl_comm_init(uid, world, rank, rank)
    b, s, pi, v = batch(game, n * world, seed=71)
    sl = slice(rank * n, (rank + 1) * n)
    d = [T.from_numpy(np.ascontiguousarray(a[sl])).cuda(rank) for a in (b, s, pi, v)]
    cfg = _dp_config(G, kind)
    for _ in range(2):
        net.train_step(*d, n, cfg, comm=comm, world=world)
    out[rank] = net.save_weights()
    G.nccl_comm_destroy(comm)
    net.close()
    import torch.distributed as dist
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("kind", [gz.GAT, gz.RESNET])
def test_data_parallel_step_matches_one_gpu(cuda, kind):
    """Two ranks on two GPUs, each with half of the batch, gradients
    all-reduced bucket by bucket over NCCL and averaged: both end with the
    same weights as one GPU stepping on the whole batch."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    out = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_dp_worker, args=(r, 2, port, out, kind)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        if p.is_alive():
            p.kill()
            pytest.fail("rank did not finish")
    assert [p.exitcode for p in procs] == [0, 0]
    game, n = gz.CONNECT4, 16
    net = gz.Net(game, kind, max_batch=2 * n)
    net.load_weights(_dp_weights(gz, kind))
    d = dev(*batch(game, 2 * n, seed=71))
    cfg = _dp_config(gz, kind)
    w0 = net.save_weights()
    for _ in range(2):
        net.train_step(*d, 2 * n, cfg)
    w = net.save_weights()
    assert np.array_equal(out[0], out[1])
    if kind == gz.RESNET:
        upd, upd_dp = w - w0, out[0] - w0
        assert np.abs(upd).max() > 0
        assert np.abs(upd_dp - upd).max() <= 1e-3 * np.abs(upd).max(), (np.abs(upd_dp - upd).max(), np.abs(upd).max())
        return
    # the averaged gradient differs from the whole-batch one in the last bits
    # of its sums; Adam divides by sqrt(v), so an entry with a near-zero
    # gradient can move by a different fraction of the learning rate:
    # allow 1 % of lr per step (measured on two B200s: 4.3e-6)
    assert np.abs(out[0] - w).max() < 0.01 * cfg.learning_rate * 2


@pytest.mark.parametrize("prec,mode", [(gz.PREC_AUTO, "fp16"), (gz.PREC_BF16, "bf16")])
def test_tensor_core_forward_after_training_follows_its_rounding_model(cuda, prec, mode):
    """One Adam step moves every weight coherently by about lr.  Rounded to
    nearest in a 16-bit format, such weights bias the Connect4 value output
    by more than 1e-3 (simulated: fp16 2.1e-3, bf16 6.3e-3 on these
    positions); the pack kernels therefore round weights stochastically by a
    hash of their blob index (simulated: 1.4e-4 and 1.5e-4).  Checked: the
    outputs within the 1e-3 bound of the oracle, and the kernel against the
    CPU rounding simulation of its formats (tests/rounding_sim.py) on exactly
    those weights -- with fp16 within 3e-4 of the simulated outputs (fp32
    accumulation and hardware exponentials against exact arithmetic), with
    bf16 (activations stochastically rounded with other random bits than the
    simulation's) the error from the oracle within 1.5 times the
    simulation's worst over three seeds.  The fp32 kernel stays within 1e-4
    of the oracle."""
    from rounding_sim import MODES, gat_forward_rounded, simulated_error
    from helpers import torch_features

    game, n = gz.CONNECT4, 8
    w = gz.synth_weights(game, seed=0x6A5A)
    boards, side = gz.synth_positions(game, n, seed=0x6A5A + 1)
    d = dev(boards, side, np.full((n, 7), 1.0 / 7, np.float32), np.zeros(n, np.float32))
    net = gz.Net(game, precision=prec, max_batch=n)
    net.load_weights(w)
    net.train_step(*d, n, gz.train_config(learning_rate=1e-3))
    w2 = net.save_weights()
    pi, v = net.predict_host(boards, side)
    opi, ov = oracle.gat_forward(game, w2, boards, side)
    if mode == "fp16":
        rp, col = gz.game_graph(game)
        spi, sv = gat_forward_rounded(game, gz.game_shape(game), torch_features(game, boards, side).numpy(), rp, col,
                                      w2, seed=0, **MODES["connect4"][mode])
        assert np.abs(pi - spi).max() < 3e-4 and np.abs(v - sv).max() < 3e-4, (np.abs(pi - spi).max(),
                                                                              np.abs(v - sv).max())
    else:
        sim = simulated_error(game, w2, boards, side, opi, ov, **MODES["connect4"][mode])
        err = max(float(np.abs(pi - opi).max()), float(np.abs(v - ov).max()))
        assert err <= 1.5 * sim, (err, sim)
    assert np.abs(pi - opi).max() < SPEC_TOL and np.abs(v - ov).max() < SPEC_TOL, (np.abs(pi - opi).max(),
                                                                                np.abs(v - ov).max())
    n32 = gz.Net(game, precision=gz.PREC_FP32, max_batch=n)
    n32.load_weights(w2)
    f32pi, f32v = n32.predict_host(boards, side)
    assert np.abs(f32pi - opi).max() < 1e-4 and np.abs(f32v - ov).max() < 1e-4
    net.check()
