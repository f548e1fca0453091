"""The N > 1 host logic on CPU: two gloo ranks (no GPU).

* head shards partition the KV heads with no overlap, and restoring a shard equals the
  same heads of the full restore (the path needs no exchange between GPUs);
* the benchmark's max-over-ranks timing and barrier work across ranks.
"""

from __future__ import annotations

import os
import socket

import torch
import torch.multiprocessing as mp

from conftest import REPO


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out: dict) -> None:
    import sys

    sys.path.insert(0, REPO)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world),
                      RANK=str(rank), LOCAL_RANK=str(rank))
    import importlib

    import torch.distributed as dist

    bench = importlib.import_module("bench")
    oracle = importlib.import_module("oracle.speccache_oracle")
    importlib.import_module("intelligent-bell_b200")
    from speccache_b200.cache import head_shard, shard_view

    d = bench.Dist(backend="gloo")
    h, t, hd = 8, 24, 64
    sl = head_shard(h, world, rank)
    owned = torch.zeros(h, dtype=torch.int64)
    owned[sl] = 1
    dist.all_reduce(owned)  # every head owned exactly once
    # identical full data on every rank (same seed); each restores only its shard
    g = torch.Generator().manual_seed(11)
    kq = torch.randint(-127, 128, (t, h, hd), generator=g, dtype=torch.int8)
    ks = (torch.rand((t, h, 1), generator=g) * 0.05 + 1e-3).half()
    c, s = oracle.compute_rope_cos_sin_delta(333, hd, 5e5)
    part = oracle.dequant_rope_shift(shard_view(kq, h, world, rank, 1),
                                     shard_view(ks, h, world, rank, 1), c, s)
    parts = [torch.empty_like(part) for _ in range(world)]
    dist.all_gather(parts, part.contiguous())
    full = oracle.dequant_rope_shift(kq, ks, c, s)
    slowest = d.max(float(rank + 1))
    d.barrier()
    out[rank] = (owned.tolist(), bool(torch.equal(torch.cat(parts, dim=1), full)), slowest)
    d.close()


def test_two_gloo_ranks_shard_heads_without_exchange():
    world = 2
    with mp.get_context("spawn").Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world,
                           start_method="spawn")
        res = dict(out)
    assert sorted(res) == [0, 1]
    for rank in range(world):
        owned, equal, slowest = res[rank]
        assert owned == [1] * 8
        assert equal
        assert slowest == 2.0


def test_bench_spreads_ranks_over_the_visible_gpus():
    # GPUs 0-3 of the measured machines share their host link, so ranks are spread
    import importlib

    bench = importlib.import_module("bench")
    assert bench.rank_gpus(1, 8) == [0]
    assert bench.rank_gpus(2, 8) == [0, 4]
    assert bench.rank_gpus(4, 8) == [0, 2, 4, 6]
    assert bench.rank_gpus(8, 8) == list(range(8))
    assert bench.rank_gpus(3, 8) == [0, 2, 4]       # still one rank per GPU
    assert bench.rank_gpus(4, 4) == [0, 1, 2, 3]    # exactly N visible: no change
    assert bench.rank_gpus(4, 8, spread=False) == [0, 1, 2, 3]

