"""Host-side behaviour of the pool and the cache sink (no GPU needed).

Mirrors the reference's tests: tests/test_phase2_engine.py:222-257 (pool basic operations),
the LRU capacity of test_phase2_engine.py:155-214, and tests/test_phase3_serving.py:342-355
(cache truncation and legacy round trip).
"""

from __future__ import annotations

import pytest
import torch


def _slabs(blocks, chunk, h, d):
    return (torch.zeros((blocks, chunk, h, d), dtype=torch.int8),
            torch.zeros((blocks, chunk, h, 1), dtype=torch.float16),
            torch.zeros((blocks, chunk, h, d), dtype=torch.int8),
            torch.zeros((blocks, chunk, h, 1), dtype=torch.float16))


def _chunk(oracle, chunk, h, d, seed):
    g = torch.Generator().manual_seed(seed)
    kq, ks = oracle.quantize_kv_int8(torch.randn((chunk, h, d), generator=g))
    vq, vs = oracle.quantize_kv_int8(torch.randn((chunk, h, d), generator=g))
    return kq, ks, vq, vs


def test_pool_basic_operations(scb, oracle):
    from speccache_b200.cache import PinnedKVPool

    pool = PinnedKVPool(4, 64, 4, 64, None, *_slabs(4, 64, 4, 64))
    assert pool.free_count == 4 and pool.allocated_count == 0
    bid = pool.allocate()
    assert bid in range(4) and pool.allocated_count == 1 and pool.free_count == 3
    kq, ks, vq, vs = _chunk(oracle, 64, 4, 64, 42)
    pool.write_block(bid, kq, ks, vq, vs, start_pos=256)
    assert pool.get_start_pos(bid) == 256
    r = pool.get_block_views(bid)
    for got, want in zip(r, (kq, ks, vq, vs)):
        assert torch.equal(got, want)
    pool.free(bid)
    assert pool.allocated_count == 0 and pool.free_count == 4


def test_pool_lru_eviction_and_callback(scb, oracle):
    from speccache_b200.cache import PinnedKVPool

    evicted = []
    pool = PinnedKVPool(8, 16, 2, 32, evicted.append, *_slabs(8, 16, 2, 32))
    ids = [pool.allocate(start_pos=i * 16) for i in range(10)]
    assert pool.allocated_count == 8
    assert evicted == ids[:2]  # the two oldest went first
    pool.touch(ids[2])  # now ids[3] is the least recently used
    pool.allocate()
    assert evicted[-1] == ids[3]
    pool.clear()
    assert pool.allocated_count == 0 and pool.free_count == 8


def test_pool_write_block_contract(scb, oracle):
    from speccache_b200.cache import PinnedKVPool

    pool = PinnedKVPool(2, 8, 2, 32, None, *_slabs(2, 8, 2, 32))
    kq, ks, vq, vs = _chunk(oracle, 8, 2, 32, 1)
    with pytest.raises(KeyError, match="not an allocated active block"):
        pool.write_block(0, kq, ks, vq, vs)
    b = pool.allocate()
    with pytest.raises(ValueError, match="k_q shape"):
        pool.write_block(b, kq[:4], ks, vq, vs)
    with pytest.raises(ValueError, match="must be provided"):
        pool.write_block(b, kq, None, vq, vs)
    pool.write_block(b, k_quant=kq, k_scale=ks, v_quant=vq, v_scale=vs, start_pos=3)
    assert pool.get_start_pos(b) == 3


def test_pool_coalesced_views_match_gather(scb, oracle):
    from speccache_b200.cache import PinnedKVPool

    pool = PinnedKVPool(6, 8, 2, 32, None, *_slabs(6, 8, 2, 32))
    for b in range(6):
        pool.allocate(block_id=b)
        pool.write_block(b, *_chunk(oracle, 8, 2, 32, 10 + b), start_pos=8 * b)
    for order in ([2, 3, 4], [5, 0, 3, 1], [4]):
        got = pool.get_coalesced_views(order)
        for g, slab in zip(got, (pool.k_quant, pool.k_scale, pool.v_quant, pool.v_scale)):
            assert torch.equal(g, oracle.gather_blocks(slab, order))
    e = pool.get_coalesced_views([])
    assert e[0].shape == (0, 2, 32)


def test_dynamic_cache_truncation_and_legacy(scb):
    from speccache_b200.serving import SpecDynamicCache

    cache = SpecDynamicCache()
    k, v = torch.randn(1, 2, 20, 16), torch.randn(1, 2, 20, 16)
    cache.update(k, v, layer_idx=0)
    assert cache.get_seq_length(0) == 20
    cache.truncate(15)
    assert cache.get_seq_length(0) == 15
    restored = SpecDynamicCache.from_legacy_cache(cache.to_legacy_cache())
    assert restored.get_seq_length(0) == 15
    assert torch.equal(restored[0][0], k[:, :, :15])


def test_dynamic_cache_update_appends_like_cat(scb):
    from speccache_b200.serving import SpecDynamicCache

    cache = SpecDynamicCache()
    parts = [(torch.randn(1, 4, n, 8), torch.randn(1, 4, n, 8)) for n in (5, 17, 1, 40)]
    for k, v in parts:
        out_k, out_v = cache.update(k, v, layer_idx=2)
    assert len(cache) == 3 and cache.get_seq_length(0) == 0
    assert torch.equal(out_k, torch.cat([p[0] for p in parts], dim=-2))
    assert torch.equal(out_v, torch.cat([p[1] for p in parts], dim=-2))
    cache.truncate(10)
    k2, v2 = torch.randn(1, 4, 3, 8), torch.randn(1, 4, 3, 8)
    out_k, _ = cache.update(k2, v2, layer_idx=2)
    assert torch.equal(out_k, torch.cat([torch.cat([p[0] for p in parts], dim=-2)[:, :, :10], k2], -2))
    assert cache.get_max_length() == 13
    assert [x is None for x in cache.key_cache] == [True, True, False]


def test_dynamic_cache_append_views_are_model_layout(scb):
    from speccache_b200.serving import SpecDynamicCache

    cache = SpecDynamicCache()
    cache.reserve(0, 12, batch=1, heads=3, head_dim=32, dtype=torch.float16, device=torch.device("cpu"))
    k, v = cache.append_views(0, 12)
    assert k.shape == (12, 3, 32)
    src = torch.randn(12, 3, 32).to(torch.float16)
    k.copy_(src)
    v.copy_(src * 2)
    cache.commit(0, 12)
    assert torch.equal(cache[0][0], src.permute(1, 0, 2).unsqueeze(0))
    assert torch.equal(cache[0][1], (src * 2).permute(1, 0, 2).unsqueeze(0))


def test_routing_decisions_select_reusable_blocks(scb, oracle):
    # reference speccache/cache/engine.py:449-460: only exact/semantic reuse with a block id
    from speccache_b200.cache import (ChunkRoutingDecision, ChunkRoutingStatus, PinnedKVPool,
                                      RestoreEngine, reusable)

    chunk, h, d = 16, 2, 32
    pool = PinnedKVPool(4, chunk, h, d, None, *_slabs(4, chunk, h, d))
    engine = RestoreEngine(pool=pool)
    assert (engine.chunk_size, engine.num_kv_heads, engine.head_dim) == (chunk, h, d)
    with pytest.raises(ValueError, match="must equal chunk_size"):
        engine.register_chunk(range(chunk - 1), 0, *_chunk(oracle, chunk, h, d, 1))
    ids = [engine.register_chunk(range(i * chunk, (i + 1) * chunk), 64 * i,
                                 *_chunk(oracle, chunk, h, d, 10 + i)) for i in range(3)]
    assert [pool.get_start_pos(b) for b in ids] == [0, 64, 128]
    assert pool._active_lru[ids[1]].token_ids == tuple(range(chunk, 2 * chunk))
    S = ChunkRoutingStatus
    ds = [ChunkRoutingDecision(i, 0, chunk, (), st, block_id=b, delta_p=5 * i)
          for i, (st, b) in enumerate([(S.EXACT_REUSE, ids[0]), (S.CACHE_MISS, ids[1]),
                                       (S.SEMANTIC_REUSE, ids[2]), (S.SPECULATIVE_DRAFT, ids[0]),
                                       (S.EXACT_REUSE, None)])]
    assert [d.chunk_index for d in reusable(ds)] == [0, 2]
    assert ChunkRoutingDecision(0, 0, 1, (), S.CACHE_MISS).continuation_tokens == []
    assert S("SEMANTIC_REUSE") is S.SEMANTIC_REUSE and S.EXACT_REUSE == "EXACT_REUSE"
