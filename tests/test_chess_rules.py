"""Chess rules behind the c3 position generator (CPU).

The move generator is checked against published perft counts (the number of
leaves of the legal move tree) of the standard test positions: the initial
position, "Kiwipete" (castling, en passant, promotions, pins) and positions
3-5 of the usual perft suite.  The synthetic positions are checked for
legality-derived invariants.
"""
import numpy as np
import pytest

import graphzero_b200 as gz

PIECES = {"p": 1, "n": 2, "b": 3, "r": 4, "q": 5, "k": 6}


def fen_record(fen: str):
    """66-byte record + side to move from a FEN string."""
    parts = fen.split()
    rec = np.zeros(66, np.int8)
    for i, row in enumerate(parts[0].split("/")):
        rank, f = 7 - i, 0
        for ch in row:
            if ch.isdigit():
                f += int(ch)
            else:
                v = PIECES[ch.lower()]
                rec[rank * 8 + f] = v if ch.isupper() else -v
                f += 1
    side = 1 if parts[1] == "w" else -1
    castle = 0
    for ch, bit in (("K", 1), ("Q", 2), ("k", 4), ("q", 8)):
        if ch in parts[2]:
            castle |= bit
    rec[64] = castle
    ep = parts[3] if len(parts) > 3 else "-"
    rec[65] = -1 if ep == "-" else (int(ep[1]) - 1) * 8 + (ord(ep[0]) - ord("a"))
    return rec, side


PERFT = [
    ("rnbqkbnr/pppppppp/8/8/8/8/PPPPPPPP/RNBQKBNR w KQkq -", [20, 400, 8902, 197281]),
    ("r3k2r/p1ppqpb1/bn2pnp1/3PN3/1p2P3/2N2Q1p/PPPBBPPP/R3K2R w KQkq -", [48, 2039, 97862]),
    ("8/2p5/3p4/KP5r/1R3p1k/8/4P1P1/8 w - -", [14, 191, 2812, 43238]),
    ("r3k2r/Pppp1ppp/1b3nbN/nP6/BBP1P3/q4N2/Pp1P2PP/R2Q1RK1 w kq -", [6, 264, 9467]),
    ("rnbq1k1r/pp1Pbppp/2p5/8/2B5/8/PPP1NnPP/RNBQK2R w KQ -", [44, 1486, 62379]),
]


@pytest.mark.parametrize("fen,counts", PERFT)
def test_perft(fen, counts):
    rec, side = fen_record(fen)
    assert gz.chess_legal_count(rec, side) == counts[0]
    for depth, want in enumerate(counts, start=1):
        assert gz.chess_perft(rec, side, depth) == want, (fen, depth)


def test_initial_record_matches_generator():
    """Index with zero plies is the initial position."""
    rec, side = fen_record(PERFT[0][0])
    boards, sides = gz.synth_positions(gz.CHESS, 400, seed=11)
    zero = [i for i in range(400) if (boards[i] == rec).all() and sides[i] == side]
    assert zero, "some playouts have k = 0 plies"


def test_synthetic_positions_are_legal_and_deterministic():
    boards, side = gz.synth_positions(gz.CHESS, 300, seed=5)
    b2, s2 = gz.synth_positions(gz.CHESS, 300, seed=5)
    assert (boards == b2).all() and (side == s2).all()
    # a sub-range of the stream equals the same indices of the full stream
    b3, s3 = gz.synth_positions(gz.CHESS, 10, seed=5, first=100)
    assert (b3 == boards[100:110]).all() and (s3 == side[100:110]).all()
    for i in range(300):
        sq = boards[i, :64]
        assert (sq == 6).sum() == 1 and (sq == -6).sum() == 1
        assert not ((sq[:8] == 1) | (sq[:8] == -1) | (sq[56:] == 1) | (sq[56:] == -1)).any()  # no pawn on a back rank
        assert 0 <= boards[i, 64] <= 15
        assert boards[i, 65] == -1 or boards[i, 65] in range(16, 24) or boards[i, 65] in range(40, 48)
        assert gz.chess_legal_count(boards[i], int(side[i])) > 0
    # the side to move varies and most playouts leave the initial position
    assert 0.3 < (side == 1).mean() < 0.7
    assert (np.abs(boards[:, :64].astype(np.int32)).sum(1) < 74).mean() > 0.5  # captures in most playouts
