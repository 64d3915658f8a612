"""The CPU rounding simulation the GPU tolerances come from: with every
rounding switched off it reproduces the oracle, and its rounding helpers
round like the hardware formats (nearest-even; stochastic rounding unbiased)."""
import numpy as np
import torch

import graphzero_b200 as gz
import oracle
from helpers import sharpen, torch_features
from rounding_sim import gat_forward_rounded, resnet_forward_rounded, round_bf16, round_fp16


def test_exact_mode_reproduces_the_oracle():
    for game, n in ((gz.CONNECT4, 12), (gz.CHESS, 3), (gz.TICTACTOE, 12)):
        w = sharpen(game, gz.synth_weights(game, seed=5, bias_scale=0.4))
        boards, side = gz.synth_positions(game, n, seed=6)
        rp, col = gz.game_graph(game)
        f = torch_features(game, boards, side).numpy()
        pi, v = gat_forward_rounded(game, gz.game_shape(game), f, rp, col, w, op="exact", gather="exact",
                                    last="fp32")
        opi, ov = oracle.gat_forward(game, w, boards, side)
        assert np.abs(pi - opi).max() < 1e-5 and np.abs(v - ov).max() < 1e-5
    w = gz.synth_weights(gz.CONNECT4, gz.RESNET, seed=31)
    boards, side = gz.synth_positions(gz.CONNECT4, 4, seed=7)
    pi, v = resnet_forward_rounded(w, boards, side, op="exact")
    opi, ov = oracle.resnet_forward(w, boards, side)
    assert np.abs(pi - opi).max() < 1e-5 and np.abs(v - ov).max() < 1e-5


def test_rounding_helpers_match_the_formats():
    x = np.random.default_rng(0).normal(size=4096).astype(np.float32) * 3
    assert (round_bf16(x, "rn") == torch.tensor(x).bfloat16().double().numpy()).all()
    assert (round_fp16(x, "rn") == x.astype(np.float16).astype(np.float64)).all()
    rng = np.random.default_rng(1)
    y = np.full(20000, 1.0 + 2.0 ** -12, np.float32)  # a quarter of an fp16 step above 1
    for f in (round_fp16, round_bf16):
        r = f(y, "sr", rng)
        lo, hi = r.min(), r.max()
        assert lo == 1.0 and hi > 1.0 and abs(r.mean() - float(y[0])) < 4 * (hi - lo) / np.sqrt(y.size)
