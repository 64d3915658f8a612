"""bench.py's reference arm (the CPU restatement timed on the host cores):
it prints the contract's JSON line with the product arm's config block, and
never loads the product library -- its weights and positions come from the
oracle's own generator, which reproduces the product's seeded streams bit
for bit (so both arms evaluate the same workload)."""
import json
import subprocess
import sys
from pathlib import Path

import numpy as np

import graphzero_b200 as gz
import oracle

ROOT = Path(__file__).resolve().parents[1]


def test_oracle_generator_matches_product_generator():
    for game in (gz.TICTACTOE, gz.CONNECT4, gz.CHESS):
        for bias in (0.0, 0.4):
            a = gz.synth_weights(game, seed=1234, bias_scale=bias)
            b = oracle.synth_gat_weights(game, 1234, bias)
            assert (a.view(np.uint32) == b.view(np.uint32)).all()
    a = gz.synth_weights(gz.CONNECT4, gz.RESNET, seed=0x6A5A + 2000)
    b = oracle.synth_res_weights(0x6A5A + 2000)
    assert (a.view(np.uint32) == b.view(np.uint32)).all()
    for game in (gz.TICTACTOE, gz.CONNECT4):
        pb, ps = gz.synth_positions(game, 700, seed=0x6A5A + 1001, first=333)
        ob, os_ = oracle.synth_positions(game, 700, 0x6A5A + 1001, 333)
        assert (pb == ob).all() and (ps == os_).all()


PROBE = r"""
import runpy, sys
sys.argv = ["bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3"]
runpy.run_path("bench.py", run_name="__main__")
maps = open("/proc/self/maps").read()
print("PRODUCT_LOADED", int("libgraphzero_b200" in maps or "graphzero_b200" in sys.modules))
"""


def test_reference_arm_runs_without_the_product_library():
    r = subprocess.run([sys.executable, "-c", PROBE], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    lines = r.stdout.strip().splitlines()
    assert lines[-1] == "PRODUCT_LOADED 0", lines[-1]
    line = json.loads(lines[-2])
    assert line["impl"] == "reference" and line["value"] > 0 and line["unit"] == "leaf evals/s"
    sys.path.insert(0, str(ROOT))
    import bench

    assert line["config"] == bench.config_block(bench.CONFIGS["c1"], 1)
    assert line["cpu_baseline"]["kind"] == "port" and line["e2e"]["h2d_bytes_per_step"] == 0
