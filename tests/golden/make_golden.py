"""Generates the golden fixtures under tests/golden/.

The reference publishes no golden vectors and its network code does not
build, so these fixtures pin the oracle (fp64 mode) on small seeded inputs,
together with a checksum of the synthetic weights they were computed from.

    python tests/golden/make_golden.py
"""
import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path[:0] = [str(ROOT), str(ROOT / "oracle"), str(ROOT / "tests")]

import graphzero_b200 as gz  # noqa: E402
import oracle  # noqa: E402
from helpers import chess_boards, sharpen  # noqa: E402

CASES = [
    ("gat_tictactoe", gz.TICTACTOE, gz.GAT, 101, 0.3, False, 16),
    ("gat_connect4", gz.CONNECT4, gz.GAT, 102, 0.0, False, 16),
    ("gat_connect4_sharp", gz.CONNECT4, gz.GAT, 103, 0.5, True, 16),
    ("gat_chess", gz.CHESS, gz.GAT, 104, 0.3, False, 2),
    ("resnet_connect4", gz.CONNECT4, gz.RESNET, 105, 0.2, False, 4),
]


def main():
    for name, game, kind, seed, bias, sharp, n in CASES:
        w = gz.synth_weights(game, kind, seed=seed, bias_scale=bias)
        if sharp:
            w = sharpen(game, w)
        if game == gz.CHESS:
            boards, side = chess_boards(n, seed)
        else:
            boards, side = gz.synth_positions(game, n, seed=seed + 1000)
        if kind == gz.GAT:
            pi, v = oracle.gat_forward(game, w, boards, side, f64=True)
        else:
            pi, v = oracle.resnet_forward(w, boards, side, f64=True)
        np.savez_compressed(HERE / f"{name}.npz", boards=boards, side=side, pi=pi, v=v)
        meta = {"game": game, "kind": kind, "weight_seed": seed, "bias_scale": bias, "sharpen": sharp,
                "weights_sha256": hashlib.sha256(np.ascontiguousarray(w).tobytes()).hexdigest(),
                "oracle_mode": "fp64", "n": n}
        (HERE / f"{name}.json").write_text(json.dumps(meta, indent=1) + "\n")
        print(name, pi.shape, v[:3])


if __name__ == "__main__":
    main()
