"""Batched PUCT on the GPU against the sequential CPU oracle: identical
leaves every wave and bit-identical visit counts and value sums, given the
same leaf evaluations (Dirichlet noise off)."""
import numpy as np
import pytest
import torch

import graphzero_b200 as gz
import oracle
from helpers import sharpen

pytestmark = pytest.mark.gpu


def make(game, trees, leaves, cap, seed, precision=gz.PREC_FP32, empty_roots=0):
    w = sharpen(game, gz.synth_weights(game, seed=seed, bias_scale=0.4))
    net = gz.Net(game, precision=precision, max_batch=trees * leaves)
    net.load_weights(w)
    m = gz.Mcts(game, trees, leaves, c_puct=1.5, virtual_loss=3, node_capacity=cap, dirichlet_eps=0.0)
    o = oracle.Mcts(game, trees, leaves, c_puct=1.5, virtual_loss=3, node_capacity=cap)
    boards, side = gz.synth_positions(game, trees, seed=seed + 1)
    boards[:empty_roots] = 0  # games from the start, as in self-play
    side[:empty_roots] = 1
    m.reset_roots(torch.from_numpy(boards).cuda(), torch.from_numpy(side).cuda())
    o.set_roots(boards, side)
    return net, m, o


def wave(net, m, o, A):
    L = m.trees * m.leaves
    m.select()
    gb, gs, gt = m.copy_leaves()
    ob, os_, ot = o.select()
    assert (gb == ob).all() and (gs == os_).all() and (gt == ot).all()
    lb, ls, _ = m.leaf_buffers()
    pi = torch.empty((L, A), device="cuda")
    v = torch.empty(L, device="cuda")
    net.predict_batch(lb, ls, L, pi, v)
    m.backup(pi, v)
    torch.cuda.synchronize()
    o.backup(pi.cpu().numpy(), v.cpu().numpy())


def compare(m, o):
    gv, gw = m.root_stats()
    ov, ow = o.root_stats()
    assert (gv == ov).all()
    assert (gw.view(np.uint32) == ow.view(np.uint32)).all()  # bit-identical sums
    gn, ge = m.tree_sizes()
    on, oe = o.tree_sizes()
    assert (gn == on).all() and (ge == oe).all()


@pytest.mark.parametrize("game,trees,leaves,waves", [(gz.CONNECT4, 64, 4, 40), (gz.TICTACTOE, 48, 4, 30),
                                                     (gz.CONNECT4, 7, 1, 25)])
def test_search_is_bit_exact(cuda, game, trees, leaves, waves):
    A = gz.game_shape(game).actions
    net, m, o = make(game, trees, leaves, cap=4096, seed=21)
    for _ in range(waves):
        wave(net, m, o, A)
    compare(m, o)
    # The first wave finds every root unexpanded (all its leaves are the root);
    # every later selection passes through a root edge.
    visits, _ = m.root_stats()
    assert (visits.sum(1) == (waves - 1) * leaves).all()


def test_search_at_selfplay_shape_is_bit_exact(cuda):
    """The self-play search shape: 1024 trees, 4 leaves per tree (leaf batch
    4096), one whole move of 800 simulations (200 waves), evaluations from
    the tensor-core network (the default operand format), c_puct 1.5,
    virtual loss 3, Dirichlet noise off; half of the games at the start
    position.  The oracle, fed the same evaluations, selects the same leaves
    every wave and ends with bit-identical visit counts and value sums."""
    game, trees, leaves = gz.CONNECT4, 1024, 4
    A = gz.game_shape(game).actions
    net, m, o = make(game, trees, leaves, cap=(800 + 1) * 3, seed=51, precision=gz.PREC_AUTO, empty_roots=512)
    assert net.kernel_name == "gat_tc_fp16"
    for _ in range(800 // leaves):
        wave(net, m, o, A)
    compare(m, o)
    visits, _ = m.root_stats()
    assert (visits.sum(1) == 800 - leaves).all()
    m.check()
    net.check()


def test_search_with_moves_is_bit_exact(cuda):
    game, trees, leaves = gz.CONNECT4, 32, 4
    A = gz.game_shape(game).actions
    net, m, o = make(game, trees, leaves, cap=600, seed=33)
    acts = torch.empty(trees, dtype=torch.int32, device="cuda")
    done = torch.empty(trees, dtype=torch.int8, device="cuda")
    for move in range(12):
        for _ in range(25):
            wave(net, m, o, A)
        compare(m, o)
        m.choose(4, acts)
        torch.cuda.synchronize()
        a = acts.cpu().numpy()
        m.play(acts, 100 + 1, done)  # reserve one move's nodes
        od = o.play(a, 100 + 1)
        torch.cuda.synchronize()
        assert (done.cpu().numpy() == od).all()
    compare(m, o)
    m.check()


def test_terminal_leaves_take_game_values(cuda):
    """A position with an immediate win: the winning child is terminal and its
    value (-1 for the side to move there) is what the backup uses."""
    game = gz.CONNECT4
    b = np.zeros((1, 42), np.int8)
    b[0, [35, 36, 37]] = 1  # first player: three in the bottom row, column 3 wins
    b[0, [28, 29, 30]] = -1  # second player: stacked on top
    side = np.array([1], np.int8)
    net = gz.Net(game, precision=gz.PREC_FP32, max_batch=4)
    net.load_weights(gz.synth_weights(game, seed=1))
    m = gz.Mcts(game, 1, 4, node_capacity=512)
    m.reset_roots(torch.from_numpy(b).cuda(), torch.from_numpy(side).cuda())
    m.run(net, 400)
    visits, wsum = m.root_stats()
    assert visits[0].argmax() == 3
    assert np.isclose(wsum[0, 3], visits[0, 3])  # every visit of the win scores +1
    m.check()


def test_capacity_error_is_reported_not_faulted(cuda):
    game = gz.CONNECT4
    net = gz.Net(game, precision=gz.PREC_FP32, max_batch=16)
    m = gz.Mcts(game, 4, 4, node_capacity=8)
    boards, side = gz.synth_positions(game, 4, seed=2)
    m.reset_roots(torch.from_numpy(boards).cuda(), torch.from_numpy(side).cuda())
    m.run(net, 64)
    with pytest.raises(gz.GZError) as e:
        m.check()
    assert e.value.status == gz.ERR_CAPACITY


def test_dirichlet_noise_keeps_counts_consistent(cuda):
    game, trees = gz.CONNECT4, 32
    net = gz.Net(game, max_batch=trees * 4)
    net.load_weights(gz.synth_weights(game, seed=4))
    m = gz.Mcts(game, trees, 4, node_capacity=1024, dirichlet_alpha=1.0, dirichlet_eps=0.25, seed=9)
    boards, side = gz.synth_positions(game, trees, seed=5)
    m.reset_roots(torch.from_numpy(boards).cuda(), torch.from_numpy(side).cuda())
    m.run(net, 200)
    visits, _ = m.root_stats()
    assert (visits.sum(1) == 196).all()
    m.check()
