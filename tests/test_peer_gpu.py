"""Gather of KV-head shards onto one GPU through CUDA IPC (needs two GPUs).

Each of two processes restores its half of the heads from its own pinned slab; rank 1's
kernel stores straight into rank 0's caches over NVLink.  Rank 0 checks all heads against
the oracle, for a one-stage restore and for a scattered restore in three block stages.
"""

from __future__ import annotations

import os
import random
import socket

import pytest
import torch
import torch.multiprocessing as mp

from conftest import REPO

pytestmark = pytest.mark.gpu

H, D, THETA = 8, 128, 500000.0
# single_stage: a small restore, one launch per rank.  block_stages: 130 scattered blocks of
# 8 layers x 4 heads per rank (512 KiB of codes per block, 128 blocks per 64 MiB stage), so
# every rank restores in three stages, its kernels writing rank 0's caches from a different
# token offset per stage, the scales gathered from the mapped slab; layers 0 and 7 are checked.
_RNG = random.Random(31)
CASES = {
    "single_stage": dict(L=3, blocks=6, chunk=32, ids=[4, 0, 1, 5], shifts=[-300, 12, 12, 4000],
                         check=(0, 1, 2)),
    "block_stages": dict(L=8, blocks=140, chunk=64, ids=_RNG.sample(range(140), 130),
                         shifts=[_RNG.randint(-4000, 4000) for _ in range(130)], check=(0, 7)),
}


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _full_slabs(c):
    g = torch.Generator().manual_seed(2027)
    shape = (c["L"], c["blocks"], c["chunk"], H)
    kq = torch.randint(-127, 128, shape + (D,), generator=g, dtype=torch.int8)
    vq = torch.randint(-127, 128, shape + (D,), generator=g, dtype=torch.int8)
    ks = (torch.rand(shape + (1,), generator=g) * 0.05 + 1e-3).half()
    vs = (torch.rand(shape + (1,), generator=g) * 0.05 + 1e-3).half()
    return kq, ks, vq, vs


def _worker(rank: int, world: int, port: int, case: str, out: dict) -> None:
    import importlib
    import sys

    sys.path.insert(0, REPO)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world)
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    importlib.import_module("intelligent-bell_b200")
    from speccache_b200.cache import HeadShardGather, KVRestorePipeline, shard_view

    oracle = importlib.import_module("oracle.speccache_oracle")
    c = CASES[case]
    L, chunk, ids, shifts = c["L"], c["chunk"], c["ids"], c["shifts"]
    kq, ks, vq, vs = _full_slabs(c)
    hs = H // world
    n_tok = len(ids) * chunk
    try:
        with KVRestorePipeline(L, c["blocks"], chunk, hs, D, device=dev) as pipe:
            pipe.k_quant.copy_(shard_view(kq, H, world, rank, 3))
            pipe.k_scale.copy_(shard_view(ks, H, world, rank, 3))
            pipe.v_quant.copy_(shard_view(vq, H, world, rank, 3))
            pipe.v_scale.copy_(shard_view(vs, H, world, rank, 3))
            stages = pipe.restore_launches(len(ids))
            k_full = v_full = None
            if rank == 0:
                k_full = torch.zeros((L, n_tok, H, D), dtype=torch.bfloat16, device=dev)
                v_full = torch.zeros_like(k_full)
            gather = HeadShardGather(pipe, k_full, v_full, owner=0, rank=rank, world_size=world,
                                     num_kv_heads=H)
            gather.restore(ids, shifts, theta=THETA)
            pipe.synchronize()
            status = pipe.status()
            dist.barrier()  # every writer's stream has completed
            ok = status == 0 and stages == (1 if case == "single_stage" else 3)
            if rank == 0:
                for layer in c["check"]:
                    kr, vr = oracle.restore_blocks(kq[layer], ks[layer], vq[layer], vs[layer],
                                                   ids, shifts, THETA, torch.bfloat16)
                    kd, vd = k_full[layer].cpu(), v_full[layer].cpu()
                    ok &= bool(torch.allclose(kd.float(), kr.float(), rtol=1e-2, atol=1e-2))
                    ok &= bool(torch.equal(vd.view(torch.int16), vr.view(torch.int16)))
            dist.barrier()  # rank 1 keeps its mapping until rank 0 has checked
            gather.close()
            out[rank] = ok
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
@pytest.mark.parametrize("case", sorted(CASES))
def test_head_shards_gather_into_one_gpu(case):
    world = 2
    with mp.get_context("spawn").Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_worker, args=(world, _free_port(), case, out), nprocs=world,
                           start_method="spawn")
        res = dict(out)
    assert res == {0: True, 1: True}
