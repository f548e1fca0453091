"""The KV-head-sharded restore, with the shards' pipelines side by side on one GPU.

On a machine, each rank restores its own head shard from its own pinned slab
(``cache/sharding.py``).  The ranks never wait on one another, so their pipelines can run
side by side on a single GPU, which checks the sharded path where only one GPU is available:

* each of W shard pipelines (W = 2, 4, 8; 8 KV heads) restores its heads into its own
  ``[L, T, 8/W, D]`` caches, and the shards put together equal, bit for bit, the restore of
  all heads by one pipeline, and match the oracle (K within 1e-2, V bit for bit);
* each shard pipeline restores into one full ``[L, T, 8, D]`` cache through per-layer addresses
  offset by its first head, the addressing ``HeadShardGather`` uses for another GPU's mapped
  cache (there over NVLink), and the full cache equals the unsharded restore bit for bit.
"""

from __future__ import annotations

import pytest
import torch

from conftest import bits_equal

pytestmark = pytest.mark.gpu

L, BLOCKS, CHUNK, H, D, THETA = 3, 6, 32, 8, 128, 500000.0
BLOCK_IDS, SHIFTS = [4, 0, 1, 5], [-300, 12, 12, 4000]


def _full_slabs():
    g = torch.Generator().manual_seed(2031)
    kq = torch.randint(-127, 128, (L, BLOCKS, CHUNK, H, D), generator=g, dtype=torch.int8)
    vq = torch.randint(-127, 128, (L, BLOCKS, CHUNK, H, D), generator=g, dtype=torch.int8)
    ks = (torch.rand((L, BLOCKS, CHUNK, H, 1), generator=g) * 0.05 + 1e-3).half()
    vs = (torch.rand((L, BLOCKS, CHUNK, H, 1), generator=g) * 0.05 + 1e-3).half()
    return kq, ks, vq, vs


def _pipeline(scb, slabs, heads: slice, dev):
    from speccache_b200.cache import KVRestorePipeline

    pipe = KVRestorePipeline(L, BLOCKS, CHUNK, heads.stop - heads.start, D, device=dev)
    for dst, src in zip((pipe.k_quant, pipe.k_scale, pipe.v_quant, pipe.v_scale), slabs):
        dst.copy_(src[..., heads, :])
    return pipe


@pytest.mark.parametrize("world", [2, 4, 8])
def test_head_shards_side_by_side_match_the_unsharded_restore(scb, oracle, world):
    from speccache_b200.cache import head_shard

    dev = torch.device("cuda", 0)
    slabs = _full_slabs()
    n_tok = len(BLOCK_IDS) * CHUNK
    with _pipeline(scb, slabs, slice(0, H), dev) as whole:
        k_ref = torch.empty((L, n_tok, H, D), dtype=torch.bfloat16, device=dev)
        v_ref = torch.empty_like(k_ref)
        whole.restore(BLOCK_IDS, SHIFTS, k_ref, v_ref, theta=THETA)
        whole.synchronize()
        assert whole.status() == 0
    pipes = [_pipeline(scb, slabs, head_shard(H, world, r), dev) for r in range(world)]
    try:
        # (1) each shard into its own caches
        outs = []
        for pipe in pipes:
            k = torch.empty((L, n_tok, H // world, D), dtype=torch.bfloat16, device=dev)
            v = torch.empty_like(k)
            pipe.restore(BLOCK_IDS, SHIFTS, k, v, theta=THETA)
            outs.append((k, v))
        # (2) each shard into one full cache, through addresses offset by its first head
        k_full = torch.zeros((L, n_tok, H, D), dtype=torch.bfloat16, device=dev)
        v_full = torch.zeros_like(k_full)
        item = k_full.element_size()
        st = k_full.stride()
        for r, pipe in enumerate(pipes):
            first = head_shard(H, world, r).start * st[2]
            kp = [k_full.data_ptr() + (layer * st[0] + first) * item for layer in range(L)]
            vp = [v_full.data_ptr() + (layer * st[0] + first) * item for layer in range(L)]
            numel = k_full.numel() - ((L - 1) * st[0] + first)
            pipe.restore_into(BLOCK_IDS, SHIFTS, kp, vp, (st[1], st[2], 1), numel, torch.bfloat16,
                              theta=THETA)
        for pipe in pipes:
            pipe.synchronize()
            assert pipe.status() == 0
    finally:
        for pipe in pipes:
            pipe.close()
    k_cat = torch.cat([k for k, _ in outs], dim=2)
    v_cat = torch.cat([v for _, v in outs], dim=2)
    assert bits_equal(k_cat.cpu(), k_ref.cpu()) and bits_equal(v_cat.cpu(), v_ref.cpu())
    assert bits_equal(k_full.cpu(), k_ref.cpu()) and bits_equal(v_full.cpu(), v_ref.cpu())
    kq, ks, vq, vs = slabs
    for layer in range(L):
        kr, vr = oracle.restore_blocks(kq[layer], ks[layer], vq[layer], vs[layer], BLOCK_IDS,
                                       SHIFTS, THETA, torch.bfloat16)
        torch.testing.assert_close(k_ref[layer].cpu().float(), kr.float(), rtol=1e-2, atol=1e-2)
        assert bits_equal(v_ref[layer].cpu(), vr)
