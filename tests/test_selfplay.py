"""Self-play episodes (gz_selfplay_*) and the training-example file.

GPU: the fused driver against the same search stepped by hand through the
primitives the search tests pin (run, root statistics, choose, play), with
the game rules applied on the host: identical examples, in the same order,
with the same values.
CPU: the reference's train_examples_*.bin layout (self_play/self_play.cu:
510-573), written and read back, and checked byte for byte with struct.
"""
import struct

import numpy as np
import pytest

import graphzero_b200 as gz


def examples(n, seed):
    rng = np.random.default_rng(seed)
    e = np.zeros(n, gz.EXAMPLE_DTYPE)
    e["board"][:, :42] = rng.integers(-1, 2, (n, 42))
    e["pi"][:, :7] = rng.random((n, 7), np.float32)
    e["v"] = rng.choice([-1.0, 0.0, 1.0], n)
    return e


def test_example_record_is_the_reference_struct():
    # int board[64]; float pi[64]; float v;  (self_play.cuh:56-60)
    assert gz.EXAMPLE_DTYPE.itemsize == 4 * 64 + 4 * 64 + 4


def test_example_file_layout(tmp_path):
    its = [examples(5, 1), examples(0, 2), examples(3, 3)]
    p = tmp_path / "train_examples_7.bin"
    gz.save_train_examples(p, its)
    raw = p.read_bytes()
    (h,) = struct.unpack_from("<i", raw, 0)
    assert h == 3
    off = 4
    for it in its:
        (c,) = struct.unpack_from("<i", raw, off)
        off += 4
        assert c == it.size
        for k in range(c):
            rec = struct.unpack_from("<64i64ff", raw, off)
            off += 516
            assert list(rec[:64]) == it["board"][k].tolist()
            assert np.array(rec[64:128], np.float32).tobytes() == it["pi"][k].tobytes()
            assert np.float32(rec[128]) == it["v"][k]
    assert off == len(raw)
    back = gz.load_train_examples(p)
    assert [b.size for b in back] == [5, 0, 3]
    assert all((a == b).all() for a, b in zip(its, back))


def test_example_file_errors(tmp_path):
    p = tmp_path / "t.bin"
    gz.save_train_examples(p, [examples(4, 5)])
    raw = p.read_bytes()
    (tmp_path / "short.bin").write_bytes(raw[:-10])
    with pytest.raises(gz.GZError) as e:
        gz.load_train_examples(tmp_path / "short.bin")
    assert e.value.status == gz.ERR_IO
    (tmp_path / "neg.bin").write_bytes(struct.pack("<i", -1))
    with pytest.raises(gz.GZError) as e:
        gz.load_train_examples(tmp_path / "neg.bin")
    assert e.value.status == gz.ERR_IO
    with pytest.raises(gz.GZError) as e:
        gz.load_train_examples(tmp_path / "missing.bin")
    assert e.value.status == gz.ERR_IO


def manual_selfplay(game, net, m, trees, n_games, sims, temp, leaves):
    """The driver's algorithm, one primitive at a time, rules on the host."""
    import torch

    s = gz.game_shape(game)
    N, A = s.nodes, s.actions
    boards = np.zeros((trees, N), np.int8)
    side = np.ones(trees, np.int8)
    moves = np.zeros(trees, np.int64)
    logs = [[] for _ in range(trees)]
    out, games = [], 0
    acts = torch.empty(trees, dtype=torch.int32, device="cuda")
    done = torch.empty(trees, dtype=torch.int8, device="cuda")
    while games < n_games:
        m.run(net, sims)
        visits, _ = m.root_stats()
        for t in range(trees):
            vt = visits[t]
            pi = np.zeros(A, np.float32)
            if moves[t] < temp:
                pi[:] = vt.astype(np.float32) / np.float32(vt.sum())
            else:
                pi[np.argmax(vt)] = 1.0  # the first, i.e. lowest, action on ties
            logs[t].append((boards[t] * side[t], pi, int(side[t])))
        m.choose(temp, acts)
        torch.cuda.synchronize()
        a = acts.cpu().numpy()
        ended = np.zeros(trees, bool)
        for t in range(trees):
            mover = int(side[t])
            nb, _ = gz.next_state(game, boards[t], mover, int(a[t]))
            won = gz.game_ended(game, nb, mover) == 1
            full = not gz.valid_moves(game, nb).any()
            if won or full:
                z = 1.0 if won else 0.0
                for b, pi, sd in logs[t]:
                    out.append((b, pi, z if sd == mover else -z))
                games += 1
                ended[t] = True
                logs[t] = []
                boards[t] = 0
                side[t] = 1
                moves[t] = 0
            else:
                boards[t] = nb
                side[t] = -mover
                moves[t] += 1
        m.play(acts, sims + leaves, done)
        torch.cuda.synchronize()
        assert (done.cpu().numpy().astype(bool) == ended).all()
    return out, games


@pytest.mark.gpu
@pytest.mark.parametrize("game,trees,sims,n_games", [(gz.TICTACTOE, 16, 24, 20), (gz.CONNECT4, 12, 40, 14)])
def test_selfplay_matches_the_search_stepped_by_hand(cuda, game, trees, sims, n_games):
    import torch

    leaves, temp = 4, 3
    s = gz.game_shape(game)
    net = gz.Net(game, max_batch=trees * leaves)
    net.load_weights(gz.synth_weights(game, seed=17, bias_scale=0.3))

    def search():
        m = gz.Mcts(game, trees, leaves, c_puct=1.5, virtual_loss=3, node_capacity=(sims + leaves) * 4,
                    dirichlet_eps=0.0, seed=7)
        m.reset_roots(torch.zeros((trees, s.nodes), dtype=torch.int8, device="cuda"),
                      torch.ones(trees, dtype=torch.int8, device="cuda"))
        return m

    m1 = search()
    sp = gz.SelfPlay(m1, max_examples=n_games * s.nodes + trees * s.nodes)
    sp.run(net, n_games, sims, temp)
    ex, games = sp.take()
    want, want_games = manual_selfplay(game, net, search(), trees, n_games, sims, temp, leaves)
    assert games == want_games >= n_games
    assert ex.size == len(want)
    assert (ex["board"][:, s.nodes:] == 0).all() and (ex["pi"][:, s.actions:] == 0).all()
    for k, (b, pi, v) in enumerate(want):
        assert (ex["board"][k, :s.nodes] == b).all(), k
        assert ex["pi"][k, :s.actions].tobytes() == pi.tobytes(), k
        assert ex["v"][k] == v, k
    # every game opens on the empty board, seen by the first player
    first = np.flatnonzero((ex["board"] == 0).all(1))
    assert first.size == games
    # the buffer is empty after take; the search keeps going where it stopped
    assert sp.take()[0].size == 0
    sp.run(net, 1, sims, temp)
    assert sp.take()[1] >= 1
    m1.check()


@pytest.mark.gpu
def test_selfplay_buffer_overflow_is_reported(cuda):
    import torch

    game, trees = gz.TICTACTOE, 8
    net = gz.Net(game, max_batch=trees * 4)
    m = gz.Mcts(game, trees, 4, node_capacity=256)
    m.reset_roots(torch.zeros((trees, 9), dtype=torch.int8, device="cuda"),
                  torch.ones(trees, dtype=torch.int8, device="cuda"))
    sp = gz.SelfPlay(m, max_examples=5)
    with pytest.raises(gz.GZError) as e:
        sp.run(net, 8, 16, 2)
    assert e.value.status == gz.ERR_CAPACITY
    # what the buffer keeps are whole games, each opening on the empty board
    ex, _ = sp.take()
    assert ex.size <= 5
    if ex.size:
        assert (ex["board"][0] == 0).all()
