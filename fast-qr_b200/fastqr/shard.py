"""Batch partitioning across GPUs of one node.

Matrices are independent, so the batch splits by contiguous ranges with no
data-path collective: rank r of G owns
``[r * ceil(B/G), min(B, (r+1) * ceil(B/G)))``.  The reference is
single-GPU (it never imports torch.distributed); this is the multi-GPU mode of
the benchmark plan.
"""
from __future__ import annotations

import os


def shard_range(batch: int, world: int, rank: int) -> tuple[int, int]:
    if world <= 0 or not 0 <= rank < world or batch < 0:
        raise ValueError("need world > 0, 0 <= rank < world, batch >= 0")
    per = -(-batch // world)
    start = min(batch, rank * per)
    stop = min(batch, start + per)
    return start, stop


def dist_env() -> tuple[int, int, int]:
    """(rank, world_size, local_rank) from the torchrun environment (1-process defaults)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def rank_inputs(config: str, seed: int, world: int, rank: int, device, batch: int | None = None,
                weak: bool = False):
    """This rank's share of a configuration's input batch.

    strong (default): the global batch is ``batch`` (default: the
    configuration's) and rank r factors its contiguous ``shard_range``.
    weak: every rank factors ``batch`` matrices of a global batch of
    ``batch * world``.
    Returns ``(A_shard, first_global_index)``.  C3 shards are exact slices of
    the global batch (structure labels are drawn over global indices); the
    other configurations draw each shard from ``seed + rank`` (the same
    distribution, without materialising the global batch on every rank).
    """
    from .inputs import CONFIGS, baseline_input

    per = batch if batch is not None else CONFIGS[config]["batch"]
    if weak:
        first, count = rank * per, per
    else:
        first, stop = shard_range(per, world, rank)
        count = stop - first
    if config == "C3":
        return baseline_input(config, seed=seed, device=device, batch=count, first=first), first
    return baseline_input(config, seed=seed + rank, device=device, batch=count), first


def max_over_ranks(value: float, device) -> float:
    """Max of a per-rank float over the default process group (identity when
    torch.distributed is not initialised)."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def all_ranks_ok(ok: bool, device) -> bool:
    """Logical AND of a per-rank verdict over the default process group."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return bool(ok)
    t = torch.tensor([0 if ok else 1], dtype=torch.int32, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return int(t.item()) == 0
