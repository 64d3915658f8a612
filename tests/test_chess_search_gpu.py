"""Batched PUCT on chess positions (gz_mcts_* with GZ_GAME_CHESS) against the
sequential CPU restatement of the same waves (tests/chess_search_oracle.py):
identical leaves every wave, bit-identical visit counts and value sums and
equal tree sizes given the same leaf evaluations (Dirichlet noise off),
then the same move choice, re-rooting and game-end flags."""
import numpy as np
import pytest
import torch

import graphzero_b200 as gz
from chess_search_oracle import ChessSearch

pytestmark = pytest.mark.gpu
G = gz.CHESS
A = gz.CHESS_ACTIONS


def wave(net, m, o):
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
    assert (gw.view(np.uint32) == ow.view(np.uint32)).all()
    gn, ge = m.tree_sizes()
    on, oe = o.tree_sizes()
    assert (gn == on).all() and (ge == oe).all()
    m.check()
    assert o.error == 0


@pytest.mark.parametrize("precision,bias", [(gz.PREC_AUTO, 0.4), (gz.PREC_FP32, 0.0)])
def test_chess_search_is_bit_exact(cuda, precision, bias):
    trees, leaves, cap = 6, 4, 1200
    w = gz.synth_weights(G, seed=41, bias_scale=bias)
    net = gz.Net(G, precision=precision, max_batch=trees * leaves)
    net.load_weights(w)
    m = gz.Mcts(G, trees, leaves, c_puct=1.5, virtual_loss=3, node_capacity=cap, dirichlet_eps=0.0)
    o = ChessSearch(trees, leaves, c_puct=1.5, virtual_loss=3, node_capacity=cap)
    boards, side = gz.synth_positions(G, trees, seed=42)
    m.reset_roots(torch.from_numpy(boards).cuda(), torch.from_numpy(side).cuda())
    o.set_roots(boards, side)
    for _ in range(25):
        wave(net, m, o)
    compare(m, o)
    # greedy move, re-rooting (subtree kept while 200 nodes stay free), more waves
    act = torch.zeros(trees, dtype=torch.int32, device="cuda")
    m.choose(0, act)
    ga = act.cpu().numpy()
    assert (ga == o.choose_greedy()).all()
    done = torch.zeros(trees, dtype=torch.int8, device="cuda")
    m.play(act, 200, done)
    od = o.play(ga, 200)
    assert (done.cpu().numpy() == od).all()
    for _ in range(10):
        wave(net, m, o)
    compare(m, o)


def test_chess_search_ends_games_and_restarts(cuda):
    """A root one move from mate: the search finds the mating move among its
    root edges as a terminal loss for the opponent, and playing it reports
    the game over and restarts the tree from the initial position."""
    from test_chess_rules import fen_record

    rec, s = fen_record("6k1/5ppp/8/8/8/8/5PPP/R5K1 w - - 0 1")  # Ra8#
    mate = 0 * 73 + 56  # a1 -> a8
    assert mate in gz.chess_legal_actions(rec, s)
    trees, leaves = 2, 4
    net = gz.Net(G, max_batch=trees * leaves)
    net.load_weights(gz.synth_weights(G, seed=5))
    m = gz.Mcts(G, trees, leaves, node_capacity=2000, dirichlet_eps=0.0)
    o = ChessSearch(trees, leaves, node_capacity=2000)
    boards = np.stack([rec, rec])
    side = np.array([s, s], np.int8)
    m.reset_roots(torch.from_numpy(boards).cuda(), torch.from_numpy(side).cuda())
    o.set_roots(boards, side)
    for _ in range(60):
        wave(net, m, o)
    compare(m, o)
    gv, gw = m.root_stats()
    # the mate's value to the mover is +1 per visit: W equals its visit count
    assert gv[0, mate] > 0 and gw[0, mate] == gv[0, mate]
    act = torch.full((trees,), mate, dtype=torch.int32, device="cuda")
    done = torch.zeros(trees, dtype=torch.int8, device="cuda")
    m.play(act, 100, done)
    assert (done.cpu().numpy() == 1).all() and (o.play(np.full(trees, mate), 100) == 1).all()
    m.select()
    lb, _, _ = m.copy_leaves()
    from chess_search_oracle import start_record
    assert (lb[0] == start_record()).all()  # restarted, the first leaf is the new root
