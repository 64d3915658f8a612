"""Host-side multi-GPU plumbing: one process per GPU, independent shards.

Leaf evaluation and self-play shard by independent positions / games with the
network replicated (the reference splits games per rank the same way,
self_play/self_play.cu:217).  The only collective is the one-time weight
broadcast from rank 0 (gz_net_broadcast, NCCL over NVLink); timing reductions
use torch.distributed.
"""
from __future__ import annotations

import os
from dataclasses import dataclass

BASE_SEED = 0x6A5A


@dataclass(frozen=True)
class RankInfo:
    rank: int
    world: int
    local_rank: int


def rank_info() -> RankInfo:
    return RankInfo(int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
                    int(os.environ.get("LOCAL_RANK", 0)))


def shard_seed(config_index: int, rank: int, base: int = BASE_SEED) -> int:
    """Per-rank input seed: base + config + rank."""
    return base + 1000 * config_index + rank


def init_process_group(backend: str, info: RankInfo, timeout_s: float = 120.0):
    import datetime

    import torch.distributed as dist

    if info.world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29533")
        kw = {}
        if backend == "nccl":
            import torch
            kw["device_id"] = torch.device("cuda", info.local_rank)
        dist.init_process_group(backend, rank=info.rank, world_size=info.world,
                                timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return info.world > 1


def max_over_ranks(x: float, device=None) -> float:
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, device=None) -> float:
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def share_bytes(payload: bytes | None, src: int = 0) -> bytes:
    """Broadcast a small byte string (e.g. an ncclUniqueId) from `src`."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        assert payload is not None
        return payload
    box = [payload]
    dist.broadcast_object_list(box, src=src)
    return box[0]


def barrier() -> None:
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        dist.barrier()
