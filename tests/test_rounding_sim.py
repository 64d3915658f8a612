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


def test_weight_rounding_is_unbiased_and_exact_on_the_grid():
    """The pack kernels' weight rounding (hashed stochastic): values already
    in the format stay; a value between two neighbours lands on one of them,
    on the far one in proportion to its distance; zero stays zero."""
    from rounding_sim import round_weights

    idx = np.arange(40000, dtype=np.int64)
    for fmt, step in (("fp16", 2.0 ** -10), ("bf16", 2.0 ** -7)):
        y = np.full(idx.size, 1.0 + step / 4, np.float32)
        r = round_weights(y, fmt, idx)
        assert set(np.unique(r)) == {1.0, 1.0 + step}
        assert abs(r.mean() - float(y[0])) < 4 * step * np.sqrt(3 / 16 / y.size)
        neg = round_weights(-y, fmt, idx)
        assert (neg == -r).all()  # same hash, mirrored value: the mirrored choice
        g = round_fp16(np.random.default_rng(2).normal(size=4096).astype(np.float32), "rn")
        g = round_bf16(g.astype(np.float32), "rn") if fmt == "bf16" else g
        assert (round_weights(g.astype(np.float32), fmt, idx[:4096]) == g).all()
    assert (round_weights(np.zeros(8, np.float32), "fp16", idx[:8]) == 0).all()
    tiny = np.full(idx.size, 2.0 ** -26, np.float32)  # a quarter of fp16's smallest subnormal
    r = round_weights(tiny, "fp16", idx)
    assert set(np.unique(r)) == {0.0, 2.0 ** -24} and abs(r.mean() / 2.0 ** -26 - 1) < 0.05
