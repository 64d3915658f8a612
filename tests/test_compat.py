"""The reference-layout shim: IGame and INeuralNet vtables built by the
library, called through their function pointers as the reference's callers
would (self_play/self_play.cu, arena/arena.cu)."""
import ctypes as C
import os

import numpy as np
import pytest

import graphzero_b200 as gz
import oracle
from helpers import sharpen
from test_rules import random_playouts


def _ints(a):
    a = np.ascontiguousarray(a, np.int32)
    return a, a.ctypes.data_as(C.POINTER(C.c_int))


@pytest.mark.parametrize("name,game", [("connect4", gz.CONNECT4), ("tictactoe", gz.TICTACTOE)])
def test_igame_vtable_matches_oracle(name, game):
    g = gz.create_igame(name)
    try:
        vt = g.contents
        s = oracle.shape(game)
        rows, cols = C.c_int(), C.c_int()
        vt.get_board_size(g, C.byref(rows), C.byref(cols))
        assert (rows.value, cols.value) == (s["rows"], s["cols"])
        assert vt.get_action_size(g) == s["actions"]
        init, pinit = _ints(np.ones(s["nodes"]))
        vt.get_init_board(g, pinit)
        assert (init == 0).all()
        for b, p, a in random_playouts(game, 60, seed=game + 40):
            bi, pb = _ints(b)
            valid = (C.c_bool * s["actions"])()
            vt.get_valid_moves(g, pb, int(p), valid)
            assert list(valid) == [oracle.legal(game, b, x) for x in range(s["actions"])]
            r = vt.get_game_ended(g, pb, int(p))
            exp = 1 if oracle.has_won(game, b, p) else -1 if oracle.has_won(game, b, -p) else 0
            assert r == exp
            can, pc = _ints(np.zeros(s["nodes"]))
            vt.get_canonical_form(g, pb, int(p), pc)
            assert (can == b * p).all()
            if a is not None:
                nb, pn = _ints(np.zeros(s["nodes"]))
                npl = C.c_int()
                vt.get_next_state(g, pb, int(p), a, pn, C.byref(npl))
                ob = b.copy()
                oracle.apply(game, ob, a, p)
                assert (nb == ob).all() and npl.value == -p
        # symmetries keep (board, pi) pairs consistent
        b = np.arange(s["nodes"]) % 3 - 1
        bi, pb = _ints(b)
        pi = np.arange(s["actions"], dtype=np.float32)
        syms = (C.c_int * 64 * 8)()
        spis = (C.c_float * 64 * 8)()
        num = C.c_int()
        vt.get_symmetries(g, pb, pi.ctypes.data_as(C.POINTER(C.c_float)), syms, spis, C.byref(num))
        assert num.value == (2 if game == gz.CONNECT4 else 8)
        for k in range(num.value):
            sb = np.array(syms[k][:s["nodes"]])
            assert sorted(sb) == sorted(b)
        buf = C.create_string_buffer(128)
        vt.string_representation(g, pb, buf, 128)
        assert buf.value.count(b"\n") == s["rows"]
    finally:
        gz.free_igame(g)


@pytest.mark.gpu
def test_ineuralnet_predict_and_checkpoint(cuda, tmp_path):
    g = gz.create_igame("connect4")
    nn = gz.create_ineuralnet("gat", g, 0)
    try:
        vt = nn.contents
        boards, side = gz.synth_positions(gz.CONNECT4, 4, seed=8)
        net_h = gz._lib.gz_shim_net(C.cast(nn, C.c_void_p))
        # the shim's net starts with the seeded generator's weights
        w = gz.synth_weights(gz.CONNECT4, seed=0x6A5A)
        for b, s in zip(boards, side):
            canon = (b * s).astype(np.float32)
            pi = np.zeros(7, np.float32)
            v = np.zeros(1, np.float32)
            vt.predict(nn, canon.ctypes.data_as(C.POINTER(C.c_float)), pi.ctypes.data_as(C.POINTER(C.c_float)),
                       v.ctypes.data_as(C.POINTER(C.c_float)))
            opi, ov = oracle.gat_forward(gz.CONNECT4, w, b[None], np.array([s], np.int8))
            assert np.abs(pi - opi[0]).max() < 1e-3 and abs(v[0] - ov[0]) < 1e-3
        # checkpoint round trip through the vtable
        vt.save_checkpoint(nn, str(tmp_path).encode(), b"ckpt.bin")
        path = tmp_path / "ckpt.bin"
        assert path.stat().st_size == 32 + 4 * gz.weight_count(gz.CONNECT4) + 8
        other = gz.Net(gz.CONNECT4)
        other.load_checkpoint(str(path))
        assert (other.save_weights() == w).all()
        # a corrupted checkpoint is rejected
        data = bytearray(path.read_bytes())
        data[100] ^= 0xFF
        bad = tmp_path / "bad.bin"
        bad.write_bytes(bytes(data))
        with pytest.raises(gz.GZError) as e:
            other.load_checkpoint(str(bad))
        assert e.value.status == gz.ERR_IO
        assert net_h
    finally:
        vt.destroy(nn)
        gz.free_igame(g)
