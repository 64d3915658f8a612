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


def sq(name: str) -> int:
    return (int(name[1]) - 1) * 8 + (ord(name[0]) - ord("a"))


def test_action_indices_name_each_legal_move_once():
    """The legal moves of random positions map to distinct indices in the
    64 x 73 action space; valid_moves marks exactly those; each one plays
    through next_state and an unlisted index is refused."""
    boards, side = gz.synth_positions(gz.CHESS, 150, seed=11)
    for b, s in zip(boards, side):
        acts = gz.chess_legal_actions(b, int(s))
        assert len(acts) == gz.chess_legal_count(b, int(s)) > 0
        assert len(set(acts.tolist())) == len(acts)
        valid = gz.chess_valid_moves(b, int(s))
        assert valid.sum() == len(acts) and valid[acts].all()
        assert gz.chess_ended(b, int(s)) == 0
        for a in acts[:8]:
            nb, ns = gz.chess_next_state(b, int(s), int(a))
            assert ns == -int(s) and nb.shape == (66,)
        bad = int(np.flatnonzero(valid == 0)[0])
        with pytest.raises(gz.GZError):
            gz.chess_next_state(b, int(s), bad)


def test_action_layout_follows_the_reference():
    """from * 73 + destination for ordinary moves and castling; a promoting
    pawn: queen at its destination square, underpromotions at 64 + u
    (straight; the reference's 64 + piece - KNIGHT), 67 + u and 70 + u
    (capturing toward the lower / higher file)."""
    b, s = fen_record("r1r4k/1P6/8/8/8/8/8/R3K2R w KQ - 0 1")
    acts = set(gz.chess_legal_actions(b, s).tolist())
    f = sq("b7") * 73
    promo = {f + sq("b8"), f + 64, f + 65, f + 66, f + sq("a8"), f + 67, f + 68, f + 69, f + sq("c8"), f + 70, f + 71,
             f + 72}
    assert promo <= acts
    assert sq("e1") * 73 + sq("g1") in acts  # castling king side
    assert sq("e1") * 73 + sq("c1") not in acts  # queen side: c1 is attacked by the rook on c8
    nb, _ = gz.chess_next_state(b, s, f + 69)  # bxa8=R
    assert nb[sq("a8")] == 4 and nb[sq("b7")] == 0
    nb, _ = gz.chess_next_state(b, s, f + sq("c8"))  # bxc8=Q
    assert nb[sq("c8")] == 5
    nb, _ = gz.chess_next_state(b, s, sq("e1") * 73 + sq("g1"))  # O-O: rook to f1, rights cleared
    assert nb[sq("g1")] == 6 and nb[sq("f1")] == 4 and nb[sq("h1")] == 0 and (nb[64] & 3) == 0


def test_game_end():
    fools, s = fen_record("rnb1kbnr/pppp1ppp/8/4p3/6Pq/5P2/PPPPP2P/RNBQKBNR w KQkq - 1 3")
    assert gz.chess_ended(fools, s) == -1 and gz.chess_legal_count(fools, s) == 0
    stale, s = fen_record("7k/5Q2/6K1/8/8/8/8/8 b - - 0 1")
    assert gz.chess_ended(stale, s) == 2
    start, s = fen_record("rnbqkbnr/pppppppp/8/8/8/8/PPPPPPPP/RNBQKBNR w KQkq - 0 1")
    assert gz.chess_ended(start, s) == 0 and len(gz.chess_legal_actions(start, s)) == 20


def test_move_lists_stay_in_bounds_on_unreachable_records():
    """A record with far more pieces than a game can have: the pseudo-legal
    list stops at its 256-entry buffer instead of writing past it."""
    rec = np.zeros(66, np.int8)
    rec[:64] = 5  # 64 white queens
    rec[0] = 6
    rec[63] = -6
    rec[65] = -1
    assert 0 <= gz.chess_legal_count(rec, 1) <= 256
    assert len(gz.chess_legal_actions(rec, 1)) <= 256
