"""Multi-rank host logic on CPU (gloo, world size 2): per-rank shards,
one-time weight agreement, max-over-ranks timing, and a rank failure that
surfaces as an error on the surviving rank instead of a hang."""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out, mode):
    sys.path[:0] = [str(ROOT), str(ROOT / "oracle")]
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    import torch.distributed as dist

    import graphzero_b200 as gz
    from graphzero_b200 import dist as gzd

    info = gzd.rank_info()
    gzd.init_process_group("gloo", info, timeout_s=10.0)
    try:
        if mode == "shard":
            seed = gzd.shard_seed(1, info.rank)
            boards, side = gz.synth_positions(gz.CONNECT4, 64, seed=seed)
            w = gz.synth_weights(gz.CONNECT4, seed=1234 + info.rank)  # ranks disagree before the broadcast
            import torch
            t = torch.from_numpy(w)
            dist.broadcast(t, src=0)
            uid = gzd.share_bytes(bytes([7] * 128) if info.rank == 0 else None)
            slow = gzd.max_over_ranks(1.0 + info.rank)
            total = gzd.sum_over_ranks(64)
            out[info.rank] = (boards.sum(), float(t.numpy().sum()), uid == bytes([7] * 128), slow, total)
        elif mode == "failure":
            if info.rank == 1:
                raise SystemExit(3)  # leaves between steps, before the collective
            try:
                gzd.barrier()
                out[info.rank] = "no error"
            except Exception as e:  # noqa: BLE001
                out[info.rank] = "error:" + type(e).__name__
    finally:
        if dist.is_initialized() and mode == "shard":
            dist.destroy_process_group()


def _spawn(mode):
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    out = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, out, mode)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
        if p.is_alive():
            p.kill()
            pytest.fail("rank did not finish")
    return dict(out), [p.exitcode for p in procs]


def test_two_rank_sharding_and_broadcast():
    out, codes = _spawn("shard")
    assert codes == [0, 0]
    (b0, w0, u0, s0, t0), (b1, w1, u1, s1, t1) = out[0], out[1]
    assert b0 != b1  # different positions per rank
    assert w0 == w1  # identical weights after the broadcast
    assert u0 and u1
    assert s0 == s1 == 2.0  # max over ranks
    assert t0 == t1 == 128


def test_rank_failure_is_an_error_not_a_hang():
    out, codes = _spawn("failure")
    assert codes[1] == 3
    assert out.get(0, "").startswith("error:")
