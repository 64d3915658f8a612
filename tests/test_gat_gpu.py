"""GAT leaf evaluation on the GPU against the CPU oracle, through the C ABI.

Tolerances (max-abs on policy probabilities and values): the spec's 1e-3,
except where the operand format itself cannot reach it.  Which is which
comes from the CPU rounding simulation (tests/rounding_sim.py, results in
tests/golden/rounding_bounds.json): it repeats the forward with exactly the
kernel's operand roundings on the same inputs, so its error is the floor of
that operand format.
  fp32 SIMT path                        2e-5
  fp16 tensor-core operands (AUTO)      1e-3, Glorot and sharpened heads
                                        (simulated floor 8e-4 sharpened)
  bf16 tensor-core operands, Glorot     1e-3
  bf16 on sharpened heads               1.5 x the simulated bf16 floor
                                        (bf16 keeps 8 significant bits; a
                                        30x policy head amplifies them)
"Sharpened" heads (policy x30, value x4, random biases) keep the policy far
from uniform, so the bound has teeth.
"""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

import graphzero_b200 as gz
import oracle
from helpers import chess_boards, sharpen

pytestmark = pytest.mark.gpu

SPEC_TOL = 1e-3
BOUNDS = json.loads((Path(__file__).resolve().parent / "golden" / "rounding_bounds.json").read_text())


def format_tol(key: str, mode: str) -> float:
    """The spec's bound, or 1.5 x the simulated floor of the operand format
    where that floor is above it."""
    return max(SPEC_TOL, 1.5 * BOUNDS[key][mode])


def run(net, boards, side):
    n = side.shape[0]
    d_b = torch.from_numpy(np.ascontiguousarray(boards)).cuda()
    d_s = torch.from_numpy(np.ascontiguousarray(side)).cuda()
    pi = torch.full((n, net.shape.actions), float("nan"), device="cuda")
    v = torch.full((n,), float("nan"), device="cuda")
    net.predict_batch(d_b, d_s, n, pi, v)
    torch.cuda.synchronize()
    return pi.cpu().numpy(), v.cpu().numpy()


def inputs(game, n, seed):
    return gz.synth_positions(game, n, seed=seed)  # chess: random legal playouts


CASES = [
    # game, precision, sharp, tol, batch sizes
    (gz.TICTACTOE, gz.PREC_FP32, True, 2e-5, (1, 5, 256)),
    (gz.CONNECT4, gz.PREC_FP32, True, 2e-5, (1, 3, 130)),
    (gz.CHESS, gz.PREC_FP32, False, 2e-5, (1, 3)),
]


@pytest.mark.parametrize("game,prec,sharp,tol,sizes", CASES)
def test_simt_matches_oracle(cuda, game, prec, sharp, tol, sizes):
    w = gz.synth_weights(game, seed=7, bias_scale=0.4 if sharp else 0.0)
    if sharp:
        w = sharpen(game, w)
    net = gz.Net(game, precision=prec, max_batch=512)
    net.load_weights(w)
    for n in sizes:
        boards, side = inputs(game, n, seed=100 + n)
        pi, v = run(net, boards, side)
        opi, ov = oracle.gat_forward(game, w, boards, side)
        assert np.isfinite(pi).all() and np.isfinite(v).all()
        assert np.abs(pi - opi).max() < tol, (n, np.abs(pi - opi).max())
        assert np.abs(v - ov).max() < tol, (n, np.abs(v - ov).max())


TC_CASES = [
    # precision, sharpened heads, tolerance
    (gz.PREC_AUTO, False, SPEC_TOL),
    (gz.PREC_AUTO, True, SPEC_TOL),
    (gz.PREC_FP16, True, SPEC_TOL),
    (gz.PREC_BF16, False, SPEC_TOL),
    (gz.PREC_BF16, True, format_tol("connect4-sharp", "bf16")),
]


def test_fp16_floor_is_below_the_spec_bound():
    """The fp16 operand format can meet 1e-3 on these inputs (simulated)."""
    for key in ("connect4", "connect4-sharp", "chess", "chess-sharp"):
        assert BOUNDS[key]["fp16"] < SPEC_TOL, (key, BOUNDS[key])


@pytest.mark.parametrize("prec,sharp,tol", TC_CASES)
def test_tensor_core_matches_oracle(cuda, prec, sharp, tol):
    game = gz.CONNECT4
    w = gz.synth_weights(game, seed=17, bias_scale=0.4 if sharp else 0.0)
    if sharp:
        w = sharpen(game, w)
    net = gz.Net(game, precision=prec, max_batch=4096)
    assert net.kernel_name == ("gat_tc_bf16" if prec == gz.PREC_BF16 else "gat_tc_fp16")
    net.load_weights(w)
    for n in (1, 2, 3, 4, 7, 300, 1000):
        boards, side = inputs(game, n, seed=200 + n)
        pi, v = run(net, boards, side)
        opi, ov = oracle.gat_forward(game, w, boards, side)
        assert np.isfinite(pi).all() and np.isfinite(v).all(), n
        assert np.abs(pi - opi).max() < tol, (n, np.abs(pi - opi).max())
        assert np.abs(v - ov).max() < tol, (n, np.abs(v - ov).max())
    net.check()


def test_tensor_core_full_batch(cuda):
    """The benchmark shape: 4096 positions in one launch, every row checked
    against the oracle, plus run-to-run determinism."""
    game = gz.CONNECT4
    w = gz.synth_weights(game, seed=0x6A5A)
    net = gz.Net(game, max_batch=4096)
    net.load_weights(w)
    boards, side = gz.synth_positions(game, 4096, seed=0x6A5A + 1)
    pi, v = run(net, boards, side)
    pi2, v2 = run(net, boards, side)
    assert (pi == pi2).all() and (v == v2).all()
    opi, ov = oracle.gat_forward(game, w, boards, side)
    assert np.abs(pi - opi).max() < 1e-3 and np.abs(v - ov).max() < 1e-3
    assert np.allclose(pi.sum(1), 1, atol=1e-5)
    # batch composition changes a position's result only slightly: its slot
    # in a 3-position tile changes how the gather MMA splits K, i.e. the last
    # bit of some fp32 sums, and such a bit can flip the rounding of one
    # activation by one unit of the operand format
    for s0 in (1000, 1500, 2000):
        pj, vj = run(net, boards[s0:s0 + 3], side[s0:s0 + 3])
        assert np.abs(pj - pi[s0:s0 + 3]).max() < 1e-5 and np.abs(vj - v[s0:s0 + 3]).max() < 1e-5
    net.check()


def test_empty_batch_is_a_no_op(cuda):
    net = gz.Net(gz.CONNECT4, precision=gz.PREC_FP32)
    net.predict_batch(0, 0, 0, 0, 0)


def test_host_call_matches_device_call(cuda):
    w = sharpen(gz.CONNECT4, gz.synth_weights(gz.CONNECT4, seed=3, bias_scale=0.3))
    net = gz.Net(gz.CONNECT4, max_batch=300)
    net.load_weights(w)
    boards, side = gz.synth_positions(gz.CONNECT4, 300, seed=4)
    p1, v1 = run(net, boards, side)
    p2, v2 = net.predict_host(boards, side)
    assert (p1 == p2).all() and (v1 == v2).all()
    with pytest.raises(gz.GZError):
        net.predict_host(np.zeros((301, 42), np.int8), np.ones(301, np.int8))


@pytest.mark.parametrize("game,kind,n", [(gz.CONNECT4, gz.GAT, 4096), (gz.CONNECT4, gz.GAT, 1023),
                                         (gz.CONNECT4, gz.RESNET, 2000), (gz.TICTACTOE, gz.GAT, 300),
                                         (gz.CHESS, gz.GAT, 1500)])
def test_host_call_routes_agree(cuda, game, kind, n):
    """The routes of the host call give the device call's results: pageable
    buffers through the net's staging (chess from 1024 positions in four
    overlapped pieces), page-locked buffers read and written by the forward
    kernel through their mapped addresses (Connect4, TicTacToe) or copied
    directly in pieces (chess); outputs reused via out=."""
    net = gz.Net(game, kind, max_batch=n)
    net.load_weights(gz.synth_weights(game, kind, seed=5))
    boards, side = gz.synth_positions(game, n, seed=6)
    p_dev, v_dev = run(net, boards, side)
    p1, v1 = net.predict_host(boards, side)
    pin_b = torch.empty(boards.shape, dtype=torch.int8, pin_memory=True).numpy()
    pin_s = torch.empty(side.shape, dtype=torch.int8, pin_memory=True).numpy()
    pin_b[:] = boards
    pin_s[:] = side
    pi = torch.full(p1.shape, float("nan"), pin_memory=True).numpy()
    v = torch.full(v1.shape, float("nan"), pin_memory=True).numpy()
    p2, v2 = net.predict_host(pin_b, pin_s, out=(pi, v))
    assert p2 is pi and v2 is v
    for p, vv in ((p1, v1), (p2, v2)):
        assert (p == p_dev).all() and (vv == v_dev).all()
    net.check()


def test_single_position_predict_uses_canonical_board(cuda):
    """INeuralNet::predict takes one canonical float board."""
    w = sharpen(gz.CONNECT4, gz.synth_weights(gz.CONNECT4, seed=5, bias_scale=0.3))
    net = gz.Net(gz.CONNECT4, precision=gz.PREC_FP32, max_batch=4)
    net.load_weights(w)
    boards, side = gz.synth_positions(gz.CONNECT4, 6, seed=6)
    for b, s in zip(boards, side):
        pi, v = net.predict((b * s).astype(np.float32))
        opi, ov = oracle.gat_forward(gz.CONNECT4, w, b[None], np.array([s], np.int8))
        assert np.abs(pi - opi[0]).max() < 2e-5 and abs(v - ov[0]) < 2e-5


def test_weights_round_trip(cuda):
    w = gz.synth_weights(gz.TICTACTOE, seed=9, bias_scale=0.1)
    net = gz.Net(gz.TICTACTOE)
    net.load_weights(w)
    assert (net.save_weights() == w).all()
    with pytest.raises(gz.GZError):
        net.load_weights(w[:-1])


def test_bounded_wait_reports_timeout_and_context_survives(cuda):
    """Failure detection on the GPU without a fault: a wait on a barrier that
    nothing arrives at gives up after its limit, the kernel exits, the host
    reads GZ_ERR_TIMEOUT, and the device keeps working."""
    assert gz.selftest_wait_timeout(0, 20000) == gz.ERR_TIMEOUT
    net = gz.Net(gz.CONNECT4, precision=gz.PREC_FP32, max_batch=2)
    boards, side = gz.synth_positions(gz.CONNECT4, 2, seed=3)
    pi, v = net.predict_host(boards, side)
    assert np.isfinite(pi).all() and np.isfinite(v).all()


CHESS_TC_CASES = [
    # precision, sharpened heads, tolerance (policy over 4672 moves, value)
    (gz.PREC_AUTO, False, SPEC_TOL),
    (gz.PREC_AUTO, True, SPEC_TOL),
    (gz.PREC_BF16, False, SPEC_TOL),
    (gz.PREC_BF16, True, format_tol("chess-sharp", "bf16")),
]


@pytest.mark.parametrize("prec,sharp,tol", CHESS_TC_CASES)
def test_chess_tensor_core_matches_oracle(cuda, prec, sharp, tol):
    """Chess on tensor cores (2 positions per 128-row tile, queen+knight
    graph, 4672-way policy as an MMA) against the oracle on legal positions."""
    game = gz.CHESS
    w = gz.synth_weights(game, seed=23, bias_scale=0.4 if sharp else 0.0)
    if sharp:
        w = sharpen(game, w)
    net = gz.Net(game, precision=prec, max_batch=512)
    assert net.kernel_name == ("gat_tc_bf16" if prec == gz.PREC_BF16 else "gat_tc_fp16")
    net.load_weights(w)
    for n in (1, 2, 3, 65, 300):
        boards, side = inputs(game, n, seed=300 + n)
        pi, v = run(net, boards, side)
        opi, ov = oracle.gat_forward(game, w, boards, side)
        assert np.isfinite(pi).all() and np.isfinite(v).all(), n
        assert np.abs(pi.sum(1) - 1).max() < 1e-4
        assert np.abs(pi - opi).max() < tol, (n, np.abs(pi - opi).max())
        assert np.abs(v - ov).max() < tol, (n, np.abs(v - ov).max())
    net.check()


def test_chess_direct_softmax_path(cuda, monkeypatch):
    """The chess kernel's direct numerators (one exponential per square,
    taken by rows whose score spread would push the factor products out of
    the fp32 range), forced for every row: against the oracle, and against
    the factor path (the same numerators up to fp32 rounding)."""
    game = gz.CHESS
    w = sharpen(game, gz.synth_weights(game, seed=23, bias_scale=0.4))
    net = gz.Net(game, max_batch=128)
    net.load_weights(w)
    boards, side = inputs(game, 65, seed=365)
    pi_f, v_f = run(net, boards, side)
    monkeypatch.setenv("GZ_CHESS_FACTOR_GAP", "-1")
    pi_d, v_d = run(net, boards, side)
    opi, ov = oracle.gat_forward(game, w, boards, side)
    assert np.isfinite(pi_d).all() and np.isfinite(v_d).all()
    assert np.abs(pi_d - opi).max() < SPEC_TOL and np.abs(v_d - ov).max() < SPEC_TOL
    # numerators equal up to fp32 rounding can still round to neighbouring
    # fp16 values; eight layers and the sharpened policy turn that into
    # about 1.2e-4 (measured on B200), the same size as each path's distance
    # from the oracle
    assert np.abs(pi_d - pi_f).max() < 5e-4 and np.abs(v_d - v_f).max() < 5e-4
    net.check()


def test_chess_tensor_core_full_batch(cuda):
    """The c3 shape: 8192 legal positions in one launch; determinism, batch
    invariance, and a sample of rows against the oracle."""
    game = gz.CHESS
    w = gz.synth_weights(game, seed=0x6A5A + 3)
    net = gz.Net(game, max_batch=8192)
    net.load_weights(w)
    boards, side = gz.synth_positions(game, 8192, seed=0x6A5A + 3)
    pi, v = run(net, boards, side)
    pi2, v2 = run(net, boards, side)
    assert (pi == pi2).all() and (v == v2).all()
    # the same positions in other batch slots give the same results
    perm = np.random.default_rng(3).permutation(8192)
    pi3, v3 = run(net, boards[perm], side[perm])
    assert np.abs(pi3 - pi[perm]).max() < 1e-6 and np.abs(v3 - v[perm]).max() < 1e-6
    idx = np.random.default_rng(4).choice(8192, 200, replace=False)
    opi, ov = oracle.gat_forward(game, w, boards[idx], side[idx])
    assert np.abs(pi[idx] - opi).max() < 1e-3 and np.abs(v[idx] - ov).max() < 1e-3
    net.check()
