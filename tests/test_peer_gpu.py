"""Gather of KV-head shards onto one GPU through CUDA IPC (needs two GPUs).

Each of two processes restores its half of the heads from its own pinned slab; rank 1's
kernel stores straight into rank 0's caches over NVLink.  Rank 0 checks all heads against
the oracle.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from conftest import REPO

pytestmark = pytest.mark.gpu

L, BLOCKS, CHUNK, H, D, THETA = 3, 6, 32, 8, 128, 500000.0
BLOCK_IDS, SHIFTS = [4, 0, 1, 5], [-300, 12, 12, 4000]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _full_slabs():
    g = torch.Generator().manual_seed(2027)
    kq = torch.randint(-127, 128, (L, BLOCKS, CHUNK, H, D), generator=g, dtype=torch.int8)
    vq = torch.randint(-127, 128, (L, BLOCKS, CHUNK, H, D), generator=g, dtype=torch.int8)
    ks = (torch.rand((L, BLOCKS, CHUNK, H, 1), generator=g) * 0.05 + 1e-3).half()
    vs = (torch.rand((L, BLOCKS, CHUNK, H, 1), generator=g) * 0.05 + 1e-3).half()
    return kq, ks, vq, vs


def _worker(rank: int, world: int, port: int, out: dict) -> None:
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
    kq, ks, vq, vs = _full_slabs()
    hs = H // world
    n_tok = len(BLOCK_IDS) * CHUNK
    try:
        with KVRestorePipeline(L, BLOCKS, CHUNK, hs, D, device=dev) as pipe:
            pipe.k_quant.copy_(shard_view(kq, H, world, rank, 3))
            pipe.k_scale.copy_(shard_view(ks, H, world, rank, 3))
            pipe.v_quant.copy_(shard_view(vq, H, world, rank, 3))
            pipe.v_scale.copy_(shard_view(vs, H, world, rank, 3))
            k_full = v_full = None
            if rank == 0:
                k_full = torch.zeros((L, n_tok, H, D), dtype=torch.bfloat16, device=dev)
                v_full = torch.zeros_like(k_full)
            gather = HeadShardGather(pipe, k_full, v_full, owner=0, rank=rank, world_size=world,
                                     num_kv_heads=H)
            gather.restore(BLOCK_IDS, SHIFTS, theta=THETA)
            pipe.synchronize()
            status = pipe.status()
            dist.barrier()  # every writer's stream has completed
            ok = status == 0
            if rank == 0:
                for layer in range(L):
                    kr, vr = oracle.restore_blocks(kq[layer], ks[layer], vq[layer], vs[layer],
                                                   BLOCK_IDS, SHIFTS, THETA, torch.bfloat16)
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
def test_head_shards_gather_into_one_gpu():
    world = 2
    with mp.get_context("spawn").Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world,
                           start_method="spawn")
        res = dict(out)
    assert res == {0: True, 1: True}
