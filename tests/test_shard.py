"""Batch sharding across ranks and the multi-rank host logic (gloo, CPU)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fastqr.shard import shard_range


@pytest.mark.parametrize("batch", [0, 1, 7, 16, 256, 1024, 1001])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shards_are_contiguous_and_cover(batch, world):
    seen = []
    prev = 0
    for r in range(world):
        s, e = shard_range(batch, world, r)
        assert s == prev and s <= e
        seen.extend(range(s, e))
        prev = e
    assert seen == list(range(batch))
    per = -(-batch // world)
    assert all(shard_range(batch, world, r)[1] - shard_range(batch, world, r)[0] <= per
               for r in range(world))


def test_shard_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard_range(8, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root), str(root / "fast-qr_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from fastqr.shard import all_ranks_ok, max_over_ranks, rank_inputs
        a, first = rank_inputs("C3", seed=7, world=world, rank=rank, device="cpu", batch=8)
        t = max_over_ranks(0.5 + rank, device="cpu")
        ok = all_ranks_ok(True, device="cpu")
        bad = all_ranks_ok(rank == 0, device="cpu")
        q.put((rank, first, a.shape[0], float(a.sum()), t, ok, bad))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_sharding_and_timing():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    from fastqr.inputs import baseline_input
    full = baseline_input("C3", seed=7, device="cpu", batch=8)
    assert [o[1] for o in out] == [0, 4]
    for rank, first, b, s, t, ok, bad in out:
        assert b == 4
        assert abs(s - float(full[first:first + b].sum())) < 1e-3
        assert t == 1.5  # max over ranks
        assert ok
        assert not bad  # one failing rank fails all


def test_weak_and_strong_rank_inputs():
    """bench.py's two modes: weak (every rank a full batch of a batch x world
    global batch, drawn from seed + rank) and strong (contiguous shards of one
    batch)."""
    from fastqr.shard import rank_inputs
    a, first = rank_inputs("C2", seed=3, world=4, rank=2, device="cpu", batch=3, weak=True)
    assert (a.shape[0], first) == (3, 6)
    a, first = rank_inputs("C2", seed=3, world=4, rank=2, device="cpu", batch=10, weak=False)
    assert (a.shape[0], first) == (3, 6)  # shards of 3, 3, 3, 1
    a, first = rank_inputs("C2", seed=3, world=4, rank=3, device="cpu", batch=10, weak=False)
    assert (a.shape[0], first) == (1, 9)
