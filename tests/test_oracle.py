"""The CPU oracle against an independent torch restatement, its own fp64
mode, the graph geometry, and the committed golden fixtures."""
import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

import graphzero_b200 as gz
import oracle
from helpers import chess_boards, sharpen, torch_gat, torch_resnet

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("game,nnz", [(gz.TICTACTOE, 49), (gz.CONNECT4, 304), (gz.CHESS, 1856)])
def test_graph_geometry(game, nnz):
    rp, col = oracle.graph(game)
    s = oracle.shape(game)
    assert s["nnz"] == nnz and rp[-1] == nnz
    adj = np.zeros((s["nodes"], s["nodes"]), bool)
    for i in range(s["nodes"]):
        nb = col[rp[i]:rp[i + 1]]
        assert (np.diff(nb) > 0).all()  # ascending, unique
        assert i in nb  # self loop
        adj[i, nb] = True
    assert (adj == adj.T).all()  # undirected board geometry
    # the product builds the identical CSR
    rp2, col2 = gz.game_graph(game)
    assert (rp == rp2).all() and (col == col2).all()


def test_connect4_degree_matches_survey():
    rp, _ = oracle.graph(gz.CONNECT4)
    assert np.isclose(np.diff(rp).mean(), 304 / 42)


@pytest.mark.parametrize("game", [gz.TICTACTOE, gz.CONNECT4])
def test_features(game):
    boards, side = gz.synth_positions(game, 16, seed=5)
    for b, s in zip(boards, side):
        f = oracle.features(game, b, s)
        assert (f[:, :3].sum(1) == 1).all()
        assert (f[:, 1] == (b == s)).all() and (f[:, 2] == (b == -s)).all()
        assert (f[:, 3] == (s == 1)).all()


def test_chess_features():
    b, s = chess_boards(8, 1)
    for bb, ss in zip(b, s):
        f = oracle.features(gz.CHESS, bb, ss)
        assert f.shape == (64, 18)
        assert (f[:, :12].sum(1) == (bb[:64] != 0)).all()
        assert (f[:, 12] == (ss == 1)).all()
        assert (f[:, 17].sum() == (1 if bb[65] >= 0 else 0))


@pytest.mark.parametrize("game", [gz.TICTACTOE, gz.CONNECT4])
@pytest.mark.parametrize("sharp", [False, True])
def test_oracle_matches_torch_restatement(game, sharp):
    w = gz.synth_weights(game, seed=11, bias_scale=0.5 if sharp else 0.0)
    if sharp:
        w = sharpen(game, w)
    boards, side = gz.synth_positions(game, 24, seed=12)
    pi, v = oracle.gat_forward(game, w, boards, side)
    pt, vt = torch_gat(game, w, boards, side)
    assert np.abs(pi - pt).max() < 2e-5
    assert np.abs(v - vt).max() < 2e-5
    assert np.allclose(pi.sum(1), 1, atol=1e-5)


def test_oracle_chess_matches_torch_restatement():
    w = gz.synth_weights(gz.CHESS, seed=13, bias_scale=0.3)
    boards, side = chess_boards(3, 2)
    pi, v = oracle.gat_forward(gz.CHESS, w, boards, side)
    pt, vt = torch_gat(gz.CHESS, w, boards, side)
    assert pi.shape == (3, 4672)
    assert np.abs(pi - pt).max() < 1e-6 and np.abs(v - vt).max() < 2e-5


@pytest.mark.parametrize("game", [gz.TICTACTOE, gz.CONNECT4])
def test_oracle_fp32_vs_fp64(game):
    w = sharpen(game, gz.synth_weights(game, seed=21, bias_scale=0.5))
    boards, side = gz.synth_positions(game, 32, seed=22)
    p32, v32 = oracle.gat_forward(game, w, boards, side)
    p64, v64 = oracle.gat_forward(game, w, boards, side, f64=True)
    assert np.abs(p32 - p64).max() < 1e-5 and np.abs(v32 - v64).max() < 1e-5


def test_resnet_oracle_matches_torch():
    w = gz.synth_weights(gz.CONNECT4, gz.RESNET, seed=31)
    boards, side = gz.synth_positions(gz.CONNECT4, 6, seed=32)
    pi, v = oracle.resnet_forward(w, boards, side)
    pt, vt = torch_resnet(w, boards, side)
    assert np.abs(pi - pt).max() < 2e-5 and np.abs(v - vt).max() < 2e-5


def test_oracle_threads_do_not_change_results():
    w = gz.synth_weights(gz.CONNECT4, seed=41, bias_scale=0.2)
    boards, side = gz.synth_positions(gz.CONNECT4, 40, seed=42)
    a = oracle.gat_forward(gz.CONNECT4, w, boards, side, threads=1)
    b = oracle.gat_forward(gz.CONNECT4, w, boards, side, threads=7)
    assert (a[0] == b[0]).all() and (a[1] == b[1]).all()


def _sha(x: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(x).tobytes()).hexdigest()


@pytest.mark.parametrize("name", ["gat_tictactoe", "gat_connect4", "gat_connect4_sharp", "gat_chess",
                                  "resnet_connect4"])
def test_golden_fixtures(name):
    meta = json.loads((GOLDEN / f"{name}.json").read_text())
    data = np.load(GOLDEN / f"{name}.npz")
    game, kind = meta["game"], meta["kind"]
    w = gz.synth_weights(game, kind, seed=meta["weight_seed"], bias_scale=meta["bias_scale"])
    if meta.get("sharpen"):
        w = sharpen(game, w)
    assert _sha(w) == meta["weights_sha256"], "synthetic weight generator changed"
    boards, side = data["boards"], data["side"]
    if kind == gz.GAT:
        pi, v = oracle.gat_forward(game, w, boards, side)
    else:
        pi, v = oracle.resnet_forward(w, boards, side)
    assert np.abs(pi - data["pi"]).max() < 1e-5
    assert np.abs(v - data["v"]).max() < 1e-5
