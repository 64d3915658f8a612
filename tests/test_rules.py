"""Game rules: the oracle's restatement against the reference's own rule
functions (compiled unmodified under oracle/_ref), the product's rules
against the oracle, and the synthetic position generator."""
import ctypes as C

import numpy as np
import pytest

import graphzero_b200 as gz
import oracle

REF = oracle.ref_rules()
needs_ref = pytest.mark.skipif(REF is None, reason="oracle/_ref not built (reference tree absent)")


def random_playouts(game, n_games, seed):
    """Yield (board, player_to_move, action) along random full games."""
    rng = np.random.default_rng(seed)
    s = oracle.shape(game)
    for _ in range(n_games):
        b = np.zeros(s["nodes"], np.int8)
        p = 1
        while True:
            legal = [a for a in range(s["actions"]) if oracle.legal(game, b, a)]
            if not legal:
                break
            a = int(rng.choice(legal))
            yield b.copy(), p, a
            oracle.apply(game, b, a, p)
            if oracle.outcome(game, b, p) != 0:
                yield b.copy(), -p, None
                break
            p = -p


def _ref_next(game, b, p, a):
    bi = b.astype(np.int32)
    out = np.zeros_like(bi)
    np_ = C.c_int()
    REF.ref_next_state(game, bi.ctypes.data_as(C.POINTER(C.c_int32)), p, a,
                       out.ctypes.data_as(C.POINTER(C.c_int32)), C.cast(C.byref(np_), C.POINTER(C.c_int32)))
    return out.astype(np.int8), np_.value


def _ref_valid(game, b):
    bi = b.astype(np.int32)
    n = 7 if game == gz.CONNECT4 else 9
    out = (C.c_uint8 * n)()
    REF.ref_valid_moves(game, bi.ctypes.data_as(C.POINTER(C.c_int32)), 1, out)
    return np.array(out, bool)


def _ref_ended(game, b, p):
    bi = b.astype(np.int32)
    return REF.ref_game_ended(game, bi.ctypes.data_as(C.POINTER(C.c_int32)), p)


@needs_ref
@pytest.mark.parametrize("game", [gz.TICTACTOE, gz.CONNECT4])
def test_oracle_rules_match_reference(game):
    s = oracle.shape(game)
    checked = 0
    for b, p, a in random_playouts(game, 300, seed=game + 1):
        valid = np.array([oracle.legal(game, b, x) for x in range(s["actions"])])
        assert (valid == _ref_valid(game, b)).all()
        for q in (1, -1):
            won = oracle.has_won(game, b, q)
            r = _ref_ended(game, b, q)
            if game == gz.CONNECT4:
                # connect4_get_game_ended reports only `player`'s own line; a
                # draw's marker is truncated to 0 by the int return type.
                assert (r == 1) == won
            else:
                # tictactoe_get_game_ended returns winner * player: +1 when
                # `player` owns the line, -1 when the opponent does.
                if won:
                    assert r == 1
                elif oracle.has_won(game, b, -q):
                    assert r == -1
                else:
                    assert r == 0
        if a is not None:
            nb = b.copy()
            oracle.apply(game, nb, a, p)
            rb, rp = _ref_next(game, b, p, a)
            assert (nb == rb).all() and rp == -p
        checked += 1
    assert checked > 1000


@needs_ref
@pytest.mark.parametrize("game", [gz.TICTACTOE, gz.CONNECT4])
def test_reference_canonical_form(game):
    s = oracle.shape(game)
    boards, side = gz.synth_positions(game, 50, seed=3)
    for b, p in zip(boards, side):
        out = np.zeros(s["nodes"], np.int32)
        REF.ref_canonical(game, b.astype(np.int32).ctypes.data_as(C.POINTER(C.c_int32)), int(p),
                          out.ctypes.data_as(C.POINTER(C.c_int32)))
        assert (out == b.astype(np.int32) * p).all()


@pytest.mark.parametrize("game", [gz.TICTACTOE, gz.CONNECT4])
def test_product_rules_match_oracle(game):
    s = oracle.shape(game)
    for b, p, a in random_playouts(game, 200, seed=game + 7):
        valid = gz.valid_moves(game, b)
        assert (valid == np.array([oracle.legal(game, b, x) for x in range(s["actions"])])).all()
        r = gz.game_ended(game, b, p)
        if oracle.has_won(game, b, p):
            assert r == 1
        elif oracle.has_won(game, b, -p):
            assert r == -1
        elif not valid.any():
            assert r == 2
        else:
            assert r == 0
        if a is not None:
            nb, np_ = gz.next_state(game, b, p, a)
            ob = b.copy()
            oracle.apply(game, ob, a, p)
            assert (nb == ob).all() and np_ == -p


def test_product_rejects_illegal_move():
    b = np.zeros(42, np.int8)
    b[[0, 7, 14, 21, 28, 35]] = [1, -1, 1, -1, 1, -1]  # column 0 full
    with pytest.raises(gz.GZError) as e:
        gz.next_state(gz.CONNECT4, b, 1, 0)
    assert e.value.status == gz.ERR_INVALID_ARG


@pytest.mark.parametrize("game", [gz.TICTACTOE, gz.CONNECT4])
def test_synth_positions_are_reachable_and_live(game):
    s = oracle.shape(game)
    boards, side = gz.synth_positions(game, 2000, seed=9)
    for b, p in zip(boards, side):
        n1, n2 = int((b == 1).sum()), int((b == -1).sum())
        assert n1 - n2 in (0, 1) and (p == 1) == (n1 == n2)
        assert not oracle.has_won(game, b, 1) and not oracle.has_won(game, b, -1)
        assert any(oracle.legal(game, b, a) for a in range(s["actions"]))
        if game == gz.CONNECT4:  # stones rest on stones
            g = b.reshape(6, 7)
            for c in range(7):
                col = g[:, c]
                filled = np.nonzero(col)[0]
                if filled.size:
                    assert (col[filled.min():] != 0).all()
    plies = (boards != 0).sum(1)
    assert plies.min() == 0 and plies.max() >= (7 if game == gz.TICTACTOE else 30)


def test_synth_positions_shard_reproducibly():
    a_b, a_s = gz.synth_positions(gz.CONNECT4, 100, seed=5)
    b_b, b_s = gz.synth_positions(gz.CONNECT4, 60, seed=5, first=40)
    assert (a_b[40:] == b_b).all() and (a_s[40:] == b_s).all()
    c_b, _ = gz.synth_positions(gz.CONNECT4, 100, seed=6)
    assert (a_b != c_b).any()
