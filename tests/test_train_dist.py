"""Host logic of data-parallel training on CPU (gloo, world size 2): the
per-rank batch order (gz_train_batch_indices), the gradient buckets
(gz_train_bucket_range) and the exchange gz_net_train_step performs on them
-- each bucket summed over the ranks in the fixed order heads, then layers
from the last down, then averaged -- so that every rank applies the same
update; and a rank that leaves before the exchange is an error on the
other rank, not a hang."""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch.multiprocessing as mp

import graphzero_b200 as gz

ROOT = Path(__file__).resolve().parents[1]


def test_batch_order_partitions_each_pass():
    n, world = 1000, 2
    cfg = gz.train_config(batch_size=32, seed=5)
    steps = n // (cfg.batch_size * world)
    for epoch in (0, 1):
        seen = []
        for step in range(steps):
            per_rank = [gz.train_batch_indices(n, cfg, epoch, step, r, world) for r in range(world)]
            assert not set(per_rank[0]) & set(per_rank[1])
            seen += [i for p in per_rank for i in p]
        assert len(seen) == len(set(seen)) == steps * cfg.batch_size * world
        assert all(0 <= i < n for i in seen)
    a = gz.train_batch_indices(n, cfg, 0, 0, 0, world)
    assert (a == gz.train_batch_indices(n, cfg, 0, 0, 0, world)).all()
    assert not (a == gz.train_batch_indices(n, cfg, 1, 0, 0, world)).all()
    with pytest.raises(gz.GZError):
        gz.train_batch_indices(n, cfg, 0, steps, 0, world)  # past the last full step


def test_buckets_tile_the_weight_blob():
    for game in (gz.TICTACTOE, gz.CONNECT4, gz.CHESS):
        L = gz.game_shape(game).layers
        ranges = [gz.train_bucket_range(game, k) for k in range(L + 1)]
        ends = 0
        for off, cnt in ranges:
            assert off == ends and cnt > 0
            ends += cnt
        assert ends == gz.weight_count(game)
        with pytest.raises(gz.GZError):
            gz.train_bucket_range(game, L + 1)


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
    import torch
    import torch.distributed as dist

    import graphzero_b200 as G
    from graphzero_b200 import dist as D

    info = D.rank_info()
    D.init_process_group("gloo", info, timeout_s=10.0)
    game = G.CONNECT4
    L = G.game_shape(game).layers
    # this rank's gradient: any function of its own batch
    cfg = G.train_config(batch_size=8, seed=3)
    idx = G.train_batch_indices(256, cfg, 0, 0, info.rank, info.world)
    rng = np.random.default_rng(int(idx.sum()))
    grad = rng.normal(size=G.weight_count(game)).astype(np.float32)
    try:
        if mode == "failure" and info.rank == 1:
            raise SystemExit(3)  # leaves before the exchange
        t = torch.from_numpy(grad.copy())
        for k in [L] + list(range(L - 1, -1, -1)):  # heads first, then layers from the last down
            off, cnt = G.train_bucket_range(game, k)
            dist.all_reduce(t[off:off + cnt])
        t /= info.world
        out[info.rank] = (grad, t.numpy().copy())
    except Exception as e:  # noqa: BLE001
        out[info.rank] = "error:" + type(e).__name__
    finally:
        if dist.is_initialized() and mode == "exchange":
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


def test_bucketed_exchange_gives_every_rank_the_mean_gradient():
    out, codes = _spawn("exchange")
    assert codes == [0, 0]
    (g0, m0), (g1, m1) = out[0], out[1]
    assert not np.array_equal(g0, g1)
    assert np.array_equal(m0, m1)
    assert np.allclose(m0, (g0 + g1) / 2, atol=1e-6)


def test_rank_leaving_before_the_exchange_is_an_error():
    out, codes = _spawn("failure")
    assert codes[1] == 3
    assert str(out.get(0, "")).startswith("error:")
