"""Game rules on the device (graphzero_b200/csrc/rules_dev.cu) against the
host entry points: the seeded position generator must give the same bytes
for every game, and the chess legal-move kernel the same action lists in the
same order as gz_chess_legal_actions (the rules behind both are one set of
host/device functions; the host side is pinned by the perft tests)."""
import time

import numpy as np
import pytest
import torch

import graphzero_b200 as gz
from test_chess_rules import fen_record

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("game,n", [(gz.TICTACTOE, 5000), (gz.CONNECT4, 5000), (gz.CHESS, 2048)])
def test_device_positions_equal_host_positions(cuda, game, n):
    for seed, first in ((0x6A5A, 0), (7, 123457)):
        hb, hs = gz.synth_positions(game, n, seed=seed, first=first)
        db, ds = gz.synth_positions_device(game, n, seed=seed, first=first)
        torch.cuda.synchronize()
        assert np.array_equal(db.cpu().numpy(), hb) and np.array_equal(ds.cpu().numpy(), hs)


def test_device_chess_move_lists_equal_host_lists(cuda):
    boards, side = gz.synth_positions(gz.CHESS, 2048, seed=19)
    fens = ["r1r4k/1P6/8/8/8/8/8/R3K2R w KQ - 0 1",  # promotions with and without capture, castling
            "rnbqkbnr/ppp1p1pp/8/3pPp2/8/8/PPPP1PPP/RNBQKBNR w KQkq f6 0 3",  # en passant
            "r3k2r/p1ppqpb1/bn2pnp1/3PN3/1p2P3/2N2Q1p/PPPBBPPP/R3K2R w KQkq - 0 1",  # Kiwipete
            "rnb1kbnr/pppp1ppp/8/4p3/6Pq/5P2/PPPPP2P/RNBQKBNR w KQkq - 1 3"]  # checkmated: no moves
    extra = [fen_record(f) for f in fens]
    crowd = np.zeros(66, np.int8)
    crowd[:64], crowd[0], crowd[63], crowd[65] = 5, 6, -6, -1  # unreachable: more moves than the list holds
    extra.append((crowd, 1))
    boards = np.concatenate([boards, np.stack([b for b, _ in extra])])
    side = np.concatenate([side, np.array([s for _, s in extra], np.int8)])
    acts, counts = gz.chess_legal_actions_device(torch.from_numpy(boards).cuda(), torch.from_numpy(side).cuda())
    acts, counts = acts.cpu().numpy(), counts.cpu().numpy()
    for i in range(len(boards)):
        host = gz.chess_legal_actions(boards[i], int(side[i]))
        assert counts[i] == len(host), i
        assert np.array_equal(acts[i, :counts[i]], host), i
        assert (acts[i, counts[i]:] == -1).all()
    assert counts[len(boards) - 2] == 0


def test_device_chess_generator_throughput(cuda):
    """Not a bound: prints the device and host time for 8192 chess positions
    (the chess benchmark's batch) so the figure can be quoted."""
    n = 8192
    gz.synth_positions_device(gz.CHESS, 64, seed=1)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    db, _ = gz.synth_positions_device(gz.CHESS, n, seed=2)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    hb, _ = gz.synth_positions(gz.CHESS, n, seed=2)
    t2 = time.perf_counter()
    assert np.array_equal(db.cpu().numpy(), hb)
    print(f"chess positions x{n}: device {1e3 * (t1 - t0):.1f} ms, host (threads) {1e3 * (t2 - t1):.1f} ms")
