"""Arena games between two networks (gz_arena_play) on the GPU.

The fused call against the same search stepped by hand through the
primitives tests/test_mcts_gpu.py pins (fresh roots each move, both
networks' leaf evaluations, the searching side's kept per tree, argmax
moves, rules on the host): identical results.  Also the half-way swap of
who moves first (arena/arena.cu:98-102) and a Connect4 run on the
tensor-core kernel.
"""
import numpy as np
import pytest

import graphzero_b200 as gz

pytestmark = pytest.mark.gpu


def nets(game, seeds, trees, leaves, precision=gz.PREC_AUTO):
    out = []
    for sd in seeds:
        n = gz.Net(game, precision=precision, max_batch=trees * leaves)
        n.load_weights(gz.synth_weights(game, seed=sd, bias_scale=0.3))
        out.append(n)
    return out


def manual_arena(game, m, net_a, net_b, n_games, sims):
    import torch

    s = gz.game_shape(game)
    T, leaves, A, N = m.trees, m.leaves, s.actions, s.nodes
    L = T * leaves
    res = [0, 0, 0]
    acts = torch.empty(T, dtype=torch.int32, device="cuda")
    for g0 in range(0, n_games, T):
        n = min(T, n_games - g0)
        boards = np.zeros((T, N), np.int8)
        side = np.ones(T, np.int8)
        a_moves = np.array([g0 + t < n_games // 2 for t in range(T)])
        active = np.arange(T) < n
        while active.any():
            m.reset_roots(torch.from_numpy(boards).cuda(), torch.from_numpy(side).cuda())
            for _ in range((sims + leaves - 1) // leaves):
                m.select()
                lb, ls, _ = m.leaf_buffers()
                pa, va = torch.empty((L, A), device="cuda"), torch.empty(L, device="cuda")
                pb, vb = torch.empty((L, A), device="cuda"), torch.empty(L, device="cuda")
                net_a.predict_batch(lb, ls, L, pa, va)
                net_b.predict_batch(lb, ls, L, pb, vb)
                pick = torch.from_numpy(np.repeat(a_moves, leaves)).cuda()
                m.backup(torch.where(pick[:, None], pa, pb).contiguous(), torch.where(pick, va, vb).contiguous())
            m.choose(0, acts)
            torch.cuda.synchronize()
            a = acts.cpu().numpy()
            for t in np.flatnonzero(active):
                mover = int(side[t])
                nb, _ = gz.next_state(game, boards[t], mover, int(a[t]))
                won = gz.game_ended(game, nb, mover) == 1
                if won or not gz.valid_moves(game, nb).any():
                    res[2 if not won else (0 if a_moves[t] else 1)] += 1
                    active[t] = False
                    boards[t] = 0
                    side[t] = 1
                else:
                    boards[t] = nb
                    side[t] = -mover
                    a_moves[t] = not a_moves[t]
    return tuple(res)


def test_arena_matches_the_search_stepped_by_hand(cuda):
    game, trees, leaves, sims = gz.TICTACTOE, 6, 4, 24
    net_a, net_b = nets(game, (31, 32), trees, leaves, gz.PREC_FP32)
    n_games = 14  # three rounds, the last one partial; A starts games 0-6
    m = gz.Mcts(game, trees, leaves, node_capacity=(sims + leaves) * 4, dirichlet_eps=0.0)
    got = gz.arena_play(m, net_a, net_b, n_games, sims)
    want = manual_arena(game, gz.Mcts(game, trees, leaves, node_capacity=(sims + leaves) * 4, dirichlet_eps=0.0),
                        net_a, net_b, n_games, sims)
    assert got == want and sum(got) == n_games
    m.check()


def test_arena_swaps_who_moves_first(cuda):
    # one network against itself with argmax moves: every game from the
    # empty board is the same game, so the first mover's result repeats and
    # each side gets the first move in half of the games
    game, trees, leaves, sims = gz.TICTACTOE, 8, 4, 32
    (net,) = nets(game, (41,), trees, leaves, gz.PREC_FP32)
    m = gz.Mcts(game, trees, leaves, node_capacity=(sims + leaves) * 4, dirichlet_eps=0.0)
    a, b, d = gz.arena_play(m, net, net, 8, sims)
    assert a == b and a + b + d == 8 and (d == 8 or d == 0)
    assert gz.arena_play(m, net, net, 0, sims) == (0, 0, 0)


def test_arena_connect4_tensor_cores(cuda):
    game, trees, leaves, sims = gz.CONNECT4, 32, 4, 64
    net_a, net_b = nets(game, (51, 52), trees, leaves)
    m = gz.Mcts(game, trees, leaves, node_capacity=(sims + leaves) * 4, dirichlet_eps=0.0)
    r1 = gz.arena_play(m, net_a, net_b, 40, sims)
    r2 = gz.arena_play(m, net_a, net_b, 40, sims)
    assert sum(r1) == 40 and r1 == r2  # deterministic
    m.check()
