"""Clip sharding across GPUs: the reference's chunk loop over clips (src/main.rs:195) spread over one process per
device. The path has no cross-GPU reduction, so ranks exchange nothing while they work; results are gathered on the
host at the end, and a rank that fails is reported to every rank instead of leaving the others waiting."""
from typing import Callable, List

import numpy as np


class ShardError(RuntimeError):
    pass


def shard(n: int, world: int, rank: int):
    """Contiguous shard of n clips for `rank` of `world` processes: (start, count). Shards differ by at most one
    clip and cover 0..n in rank order, so results merge by concatenation."""
    if world < 1 or not 0 <= rank < world or n < 0:
        raise ValueError("bad shard request")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def merge(parts: List[dict], keys=("tokens", "lens", "times")):
    """Concatenates per-rank result dicts (in rank order) into one."""
    return {k: np.concatenate([p[k] for p in parts], axis=0) for k in keys}


def run_sharded(work: Callable[[int, int], dict], n: int, group=None):
    """Runs work(start, count) on this rank's shard of n clips and gathers every rank's result (rank order) on all
    ranks through torch.distributed (any backend; object collectives). A rank whose work raises still takes part
    in the gather, so every rank learns of the failure and raises ShardError naming the failed ranks."""
    import torch.distributed as dist
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    start, count = shard(n, world, rank)
    try:
        out = ("ok", work(start, count))
    except Exception as e:  # reported to every rank below
        out = ("error", f"{type(e).__name__}: {e}")
    gathered = [None] * world
    dist.all_gather_object(gathered, out, group=group)
    failed = [(r, g[1]) for r, g in enumerate(gathered) if g[0] != "ok"]
    if failed:
        raise ShardError("; ".join(f"rank {r} failed: {msg}" for r, msg in failed))
    return [g[1] for g in gathered]
