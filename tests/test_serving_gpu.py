"""GPU tests of the pool, injector, cache sink and offload against the oracle and the
reference's own injector outputs (golden vectors).

Mirrors tests/test_phase3_serving.py:137-235 (multi-layer shifted injection),
tests/test_phase2_engine.py:297-359 (multi-chunk pipeline parity, through the pool and through
routing decisions) and the restore half of tests/test_phase2_engine.py:57-147 (semantic shifted
hit, delta_p = -384) of the reference.
K is compared with the reference tolerance (the kernels build cos/sin from delta_p, one
fp16 ulp apart from torch's tables in rare entries), V bit for bit.
"""

from __future__ import annotations

import pytest
import torch

from conftest import as_tensor, bits_equal

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0) if torch.cuda.is_available() else None


def test_multi_layer_shifted_kv_injection(scb, oracle):
    from speccache_b200.serving import MultiLayerKVInjector, SpecDynamicCache

    layers, h, d, chunk = 4, 4, 64, 32
    inj = MultiLayerKVInjector(layers, h, d, device=DEV, max_blocks=16, chunk_size=chunk)
    p_cached, delta_p = 256, -256
    g = torch.Generator().manual_seed(123)
    c256, s256 = oracle.compute_rope_cos_sin_delta(p_cached, d)
    cf = torch.cat([c256, c256], -1)[:, None, :].float()
    sf = torch.cat([s256, s256], -1)[:, None, :].float()
    raw_k, raw_v = [], []
    for layer in range(layers):
        k = torch.randn((chunk, h, d), generator=g)
        v = torch.randn((chunk, h, d), generator=g)
        raw_k.append(k)
        raw_v.append(v)
        kq, ks = scb.quantize_kv_int8((k * cf + oracle.rotate_half(k) * sf).to(torch.float16).to(DEV))
        vq, vs = scb.quantize_kv_int8(v.to(DEV))
        pool = inj.layer_pools[layer]
        pool.allocate(block_id=0, start_pos=p_cached)
        pool.write_block(block_id=0, k_quant=kq.cpu(), k_scale=ks.cpu(), v_quant=vq.cpu(),
                         v_scale=vs.cpu(), start_pos=p_cached)
    cache = SpecDynamicCache()
    legacy = inj.reconstruct_and_inject_multi_layer(cache, block_ids=[0], delta_ps=[delta_p])
    inj.pipeline.synchronize()
    assert len(cache) == layers and len(legacy) == layers
    for layer in range(layers):
        k_c, v_c = cache[layer]
        assert k_c.shape == (1, h, chunk, d) and v_c.shape == (1, h, chunk, d)
        k_exp = raw_k[layer].to(torch.float16).permute(1, 0, 2).unsqueeze(0)
        v_exp = raw_v[layer].to(torch.float16).permute(1, 0, 2).unsqueeze(0)
        torch.testing.assert_close(v_c.float().cpu(), v_exp.float(), rtol=2e-2, atol=2e-2)
        torch.testing.assert_close(k_c.float().cpu(), k_exp.float(), rtol=3e-2, atol=3e-2)
    inj.close()


def test_injector_matches_reference_golden(scb, golden):
    from speccache_b200.serving import MultiLayerKVInjector, SpecDynamicCache

    kq_all, ks_all = as_tensor(golden["inj_kq"]), as_tensor(golden["inj_ks"])
    vq_all, vs_all = as_tensor(golden["inj_vq"]), as_tensor(golden["inj_vs"])
    layers, blocks, chunk, h, d = kq_all.shape
    block_ids = golden["inj_blocks"].tolist()
    inj = MultiLayerKVInjector(layers, h, d, device=DEV, max_blocks=blocks, chunk_size=chunk)
    inj.unified_k_quant.copy_(kq_all)
    inj.unified_k_scale.copy_(ks_all)
    inj.unified_v_quant.copy_(vq_all)
    inj.unified_v_scale.copy_(vs_all)
    for tag in ("const", "mixed"):
        cache = SpecDynamicCache()
        legacy = inj.reconstruct_and_inject_multi_layer(
            cache, block_ids, golden[f"inj_{tag}_dps"].tolist())
        inj.pipeline.synchronize()
        assert inj.pipeline.status() == 0
        for layer, (k, v) in enumerate(legacy):
            k_ref = as_tensor(golden[f"inj_{tag}_k{layer}"])
            v_ref = as_tensor(golden[f"inj_{tag}_v{layer}"])
            torch.testing.assert_close(k.cpu(), k_ref, rtol=1e-2, atol=1e-2)
            assert bits_equal(v.contiguous().cpu(), v_ref)
    inj.close()


def test_injector_appends_after_existing_tokens(scb, oracle):
    from speccache_b200.serving import MultiLayerKVInjector, SpecDynamicCache

    layers, h, d, chunk = 2, 8, 128, 16
    inj = MultiLayerKVInjector(layers, h, d, device=DEV, max_blocks=8, chunk_size=chunk,
                               out_dtype=torch.bfloat16, theta=500000.0)
    g = torch.Generator().manual_seed(4)
    inj.unified_k_quant.copy_(torch.randint(-127, 128, inj.unified_k_quant.shape, generator=g, dtype=torch.int8))
    inj.unified_v_quant.copy_(torch.randint(-127, 128, inj.unified_v_quant.shape, generator=g, dtype=torch.int8))
    inj.unified_k_scale.fill_(0.02)
    inj.unified_v_scale.fill_(0.03)
    cache = SpecDynamicCache()
    prefix = torch.randn((1, h, 5, d), generator=g).to(torch.bfloat16).to(DEV)
    for layer in range(layers):
        cache.update(prefix, prefix, layer)
    inj.reconstruct_and_inject_multi_layer(cache, [6, 1], [10, -10])
    inj.reconstruct_and_inject_multi_layer(cache, [3], [77])
    inj.pipeline.synchronize()
    for layer in range(layers):
        k, v = cache[layer]
        assert k.shape == (1, h, 5 + 3 * chunk, d)
        assert torch.equal(k[:, :, :5], prefix)
        kr, vr = oracle.restore_blocks(inj.unified_k_quant[layer], inj.unified_k_scale[layer],
                                       inj.unified_v_quant[layer], inj.unified_v_scale[layer],
                                       [6, 1, 3], [10, -10, 77], 500000.0, torch.bfloat16)
        torch.testing.assert_close(k[0, :, 5:].permute(1, 0, 2).float().cpu(), kr.float(),
                                   rtol=1e-2, atol=1e-2)
        assert bits_equal(v[0, :, 5:].permute(1, 0, 2).contiguous().cpu(), vr)
    inj.close()


def test_offload_then_restore_round_trip(scb, oracle):
    from speccache_b200.serving import MultiLayerKVInjector, SpecDynamicCache

    layers, h, d, chunk = 3, 4, 128, 32
    inj = MultiLayerKVInjector(layers, h, d, device=DEV, max_blocks=10, chunk_size=chunk)
    g = torch.Generator().manual_seed(9)
    blocks = [7, 2, 3]
    ks_, vs_ = [], []
    for _ in range(layers):
        ks_.append(torch.randn((len(blocks) * chunk, h, d), generator=g).to(torch.float16))
        vs_.append(torch.randn((len(blocks) * chunk, h, d), generator=g).to(torch.float16))
    inj.offload_multi_layer(blocks, [k.to(DEV) for k in ks_], [v.to(DEV) for v in vs_])
    cache = SpecDynamicCache()
    inj.reconstruct_and_inject_multi_layer(cache, blocks, [0, 0, 0])  # ordered after the offload
    inj.pipeline.synchronize()
    for layer in range(layers):
        kq, ks = oracle.quantize_kv_int8(ks_[layer])
        vq, vs = oracle.quantize_kv_int8(vs_[layer])
        got_kq = torch.cat([inj.unified_k_quant[layer, b] for b in blocks])
        got_ks = torch.cat([inj.unified_k_scale[layer, b] for b in blocks])
        got_vq = torch.cat([inj.unified_v_quant[layer, b] for b in blocks])
        assert torch.equal(got_kq, kq) and torch.equal(got_vq, vq)
        assert bits_equal(got_ks, ks)
        k, v = cache[layer]
        assert bits_equal(v[0].permute(1, 0, 2).contiguous().cpu(), oracle.dequant_value(vq, vs))
        c, s = oracle.compute_rope_cos_sin_delta(0, d)
        torch.testing.assert_close(k[0].permute(1, 0, 2).cpu(), oracle.dequant_rope_shift(kq, ks, c, s),
                                   rtol=0, atol=0)
    inj.close()


@pytest.mark.parametrize("n_blocks", [1, 3, 7, 12])
def test_small_restore_equals_per_layer(scb, oracle, n_blocks):
    # a restore that fits one stage: below 8 blocks one stage (one 3-D copy per run, one
    # launch), from 8 blocks on the last block in a stage of its own (12 blocks: stages of 11
    # and 1); it must write exactly what the layer-by-layer path writes, scattered and
    # consecutive blocks alike
    from speccache_b200.cache import KVRestorePipeline

    layers, blocks, chunk, h, d = 5, 12, 32, 4, 128
    g = torch.Generator().manual_seed(40 + n_blocks)
    ids = torch.randperm(blocks, generator=g)[:n_blocks].tolist()
    if n_blocks == 7:
        ids = [2, 3, 4, 9, 10, 0, 1]  # runs of consecutive ids and a jump back
    dps = torch.randint(-3000, 3000, (n_blocks,), generator=g).tolist()
    outs = []
    for per_layer in (False, True):
        with KVRestorePipeline(layers, blocks, chunk, h, d, device=DEV, per_layer=per_layer) as pipe:
            g2 = torch.Generator().manual_seed(99)
            for t in (pipe.k_quant, pipe.v_quant):
                t.copy_(torch.randint(-127, 128, tuple(t.shape), generator=g2, dtype=torch.int8))
            for t in (pipe.k_scale, pipe.v_scale):
                t.copy_((torch.rand(tuple(t.shape), generator=g2) * 0.05 + 1e-3).half())
            # model-layout outputs: [1, H, Tmax, D] per layer, separate allocations
            kc = [torch.zeros((1, h, 512, d), dtype=torch.bfloat16, device=DEV) for _ in range(layers)]
            vc = [torch.zeros_like(x) for x in kc]
            n_tok = n_blocks * chunk
            assert pipe.restore_launches(n_blocks) == (
                layers if per_layer else 2 if n_blocks >= 8 else 1)
            pipe.restore(ids, dps, [x[0, :, 16:16 + n_tok].permute(1, 0, 2) for x in kc],
                         [x[0, :, 16:16 + n_tok].permute(1, 0, 2) for x in vc], theta=5e5)
            pipe.synchronize()
            assert pipe.status() == 0
            outs.append(([x.cpu() for x in kc], [x.cpu() for x in vc]))
            if not per_layer:
                for layer in range(layers):
                    kr, vr = oracle.restore_blocks(pipe.k_quant[layer], pipe.k_scale[layer],
                                                   pipe.v_quant[layer], pipe.v_scale[layer], ids, dps,
                                                   5e5, torch.bfloat16)
                    got_v = outs[0][1][layer][0, :, 16:16 + n_tok].permute(1, 0, 2)
                    assert bits_equal(got_v.contiguous(), vr)
                    got_k = outs[0][0][layer][0, :, 16:16 + n_tok].permute(1, 0, 2)
                    torch.testing.assert_close(got_k.float(), kr.float(), rtol=1e-2, atol=1e-2)
                    assert not outs[0][0][layer][0, :, :16].any()  # nothing written before
    for layer in range(layers):
        assert bits_equal(outs[0][0][layer], outs[1][0][layer])
        assert bits_equal(outs[0][1][layer], outs[1][1][layer])


@pytest.mark.parametrize("n_slots,split", [(2, False), (1, False), (2, True)])
def test_block_stage_restore_equals_per_layer(scb, oracle, n_slots, split):
    # a restore beyond one stage (64 MiB of codes over all layers: 56 blocks here) goes in
    # block stages, here 35, 34 and 1 blocks: one 3-D copy per run of blocks within a stage (a
    # run that crosses a stage boundary is split), one launch per stage, the stages rotating
    # over two slots.  Three restores back to back (each reuses the slots and the scales), the
    # last a fully scattered list (every block its own run, in stages of 40, 39 and 1); all
    # must write exactly what the layer-by-layer path writes.  Also with one slot (each stage's
    # copy waits for the kernel of the stage before) and with each run's K and V as two 2-D
    # copies (the form a slab beyond the device's copy pitch takes).
    from speccache_b200.cache import KVRestorePipeline

    layers, blocks, chunk, h, d = 9, 80, 64, 8, 128
    g = torch.Generator().manual_seed(77)
    cases = []
    for ids, theta, dt in (
            (list(range(10, 40)) + list(range(0, 10)) + [45, 44, 43] + list(range(50, 77)), 5e5,
             torch.bfloat16),
            (list(range(79, 59, -1)) + list(range(0, 50)), 1e4, torch.float16),
            (list(range(0, 80, 2)) + list(range(79, 0, -2)), 5e5, torch.bfloat16)):
        dps = torch.randint(-3000, 3000, (len(ids),), generator=g).tolist()
        cases.append((ids, dps, theta, dt))
    outs = []
    for per_layer in (False, True):
        with KVRestorePipeline(layers, blocks, chunk, h, d, device=DEV, per_layer=per_layer,
                               n_slots=n_slots, split_kv_copies=split) as pipe:
            g2 = torch.Generator().manual_seed(101)
            for t in (pipe.k_quant, pipe.v_quant):
                t.copy_(torch.randint(-127, 128, tuple(t.shape), generator=g2, dtype=torch.int8))
            for t in (pipe.k_scale, pipe.v_scale):
                t.copy_((torch.rand(tuple(t.shape), generator=g2) * 0.05 + 1e-3).half())
            # stages of 35, 34, 1 blocks (56 fit 64 MiB of codes here), or one per layer
            assert pipe.restore_launches(70) == (layers if per_layer else 3)
            assert pipe.restore_launches(4) == (layers if per_layer else 1)  # one stage
            # the first list is 6 runs; its stages hold 2, 5 and 1 of them.  Staged: 3
            # launches + the scale gather, the metadata upload + 8 code copies; layer by
            # layer: 9 launches, the upload + 6 scale copies + 9 x 6 code copies
            assert pipe.restore_plan(cases[0][0]) == ((9, 61) if per_layer else
                                                     (4, 17) if split else (4, 9))
            assert pipe.restore_plan([3, 4, 5, 6]) == ((9, 11) if per_layer else
                                                       (1, 4) if split else (1, 3))
            # offloads: K and V quantize + the codes' and scales' scatter for 80 single runs;
            # one run: two copies (codes; scales)
            assert pipe.offload_plan(cases[2][0]) == (4, 0)
            assert pipe.offload_plan([5, 6, 7]) == (2, 2)
            res = []
            for ids, dps, theta, dt in cases:
                k = torch.zeros((layers, len(ids) * chunk, h, d), dtype=dt, device=DEV)
                v = torch.zeros_like(k)
                pipe.restore(ids, dps, k, v, theta=theta)
                res.append((k, v))
            pipe.synchronize()
            assert pipe.status() == 0
            outs.append([x.cpu() for kv in res for x in kv])
            if not per_layer:
                for layer in (0, 4, 8):
                    for (ids, dps, theta, dt), (k, v) in zip(cases, res):
                        kr, vr = oracle.restore_blocks(pipe.k_quant[layer], pipe.k_scale[layer],
                                                       pipe.v_quant[layer], pipe.v_scale[layer],
                                                       ids, dps, theta, dt)
                        assert bits_equal(v[layer].cpu(), vr)
                        torch.testing.assert_close(k[layer].cpu().float(), kr.float(), rtol=1e-2,
                                                   atol=1e-2)
    for staged, per_layer in zip(outs[0], outs[1]):
        assert bits_equal(staged, per_layer)


def stage_count(n, cap):
    """Launches of a block-stage restore of n blocks with at most cap blocks per stage: one
    stage below 8 blocks when they fit, else as few front stages of at most cap blocks as
    hold n - 1 blocks plus a last one-block stage."""
    return 1 if n <= cap and (n < 8 or cap < 2) else -(-(n - 1) // cap) + 1


@pytest.mark.parametrize("seed", range(6))
def test_block_stages_random_geometries(scb, oracle, seed):
    # restores beyond one stage, with random layer counts, block lists (runs and jumps), slot
    # counts, max_restore_blocks and output dtypes: the staged path must write the bits of the
    # layer-by-layer path, in the launches the stage rule gives, and match the oracle
    import random

    from speccache_b200.cache import KVRestorePipeline

    rng = random.Random(1000 + seed)
    layers = rng.randint(2, 12)
    chunk, h, d = rng.choice([(64, 8, 128), (32, 8, 128), (64, 4, 256), (128, 8, 64)])
    cap = (64 << 20) // (2 * layers * chunk * h * d)  # blocks per 64 MiB stage
    need = cap + 1
    blocks = need + rng.randint(5, 40)
    n = rng.randint(need, blocks)
    ids = rng.sample(range(blocks), n)
    step = rng.choice([1, 4, 16])
    ids.sort(key=lambda x: x // step)  # runs of consecutive ids and jumps
    dps = [rng.randint(-6000, 6000) for _ in ids]
    dtype = rng.choice([torch.float16, torch.bfloat16])
    n_slots, max_rb = rng.randint(1, 3), rng.randint(n, blocks)
    g = torch.Generator().manual_seed(seed)
    data, outs, launches = None, [], []
    for per_layer in (False, True):
        with KVRestorePipeline(layers, blocks, chunk, h, d, device=DEV, n_slots=n_slots,
                               max_restore_blocks=max_rb, per_layer=per_layer) as pipe:
            slabs = (pipe.k_quant, pipe.k_scale, pipe.v_quant, pipe.v_scale)
            if data is None:
                data = [torch.randint(-127, 128, tuple(x.shape), generator=g, dtype=torch.int8)
                        if x.dtype == torch.int8 else
                        (torch.rand(tuple(x.shape), generator=g) * 0.05 + 1e-3).half() for x in slabs]
            for dst, src in zip(slabs, data):
                dst.copy_(src)
            ko = torch.empty((layers, n * chunk, h, d), dtype=dtype, device=DEV)
            vo = torch.empty_like(ko)
            launches.append(pipe.restore_launches(n))
            pipe.restore(ids, dps, ko, vo, theta=5e5)
            pipe.synchronize()
            assert pipe.status() == 0
            outs.append((ko.cpu(), vo.cpu()))
    assert launches == [stage_count(n, min(cap, max_rb)), layers]
    assert bits_equal(outs[0][0], outs[1][0]) and bits_equal(outs[0][1], outs[1][1])
    layer = rng.randrange(layers)
    kr, vr = oracle.restore_blocks(data[0][layer], data[1][layer], data[2][layer], data[3][layer],
                                   ids, dps, 5e5, dtype)
    assert bits_equal(outs[0][1][layer], vr)
    torch.testing.assert_close(outs[0][0][layer].float(), kr.float(), rtol=1e-2, atol=1e-2)


def test_offload_staging_ring_and_join(scb, oracle):
    # successive offloads alternate two staging slots (the third reuses the first); join makes
    # the current stream wait for their copies on the GPU, after which the slabs hold the
    # oracle's codes and scales
    from speccache_b200.cache import KVRestorePipeline

    layers, blocks, chunk, h, d = 3, 8, 32, 4, 128
    ids = [[5, 6, 7, 1], [0, 2], [3, 4, 5, 6, 7, 0]]  # a run plus a lone block; scattered; runs
    g = torch.Generator().manual_seed(21)
    with KVRestorePipeline(layers, blocks, chunk, h, d, device=DEV) as pipe:
        xs = []
        for layer, b in enumerate(ids):
            k = torch.randn((len(b) * chunk, h, d), generator=g).to(torch.bfloat16)
            v = torch.randn((len(b) * chunk, h, d), generator=g).to(torch.bfloat16)
            xs.append((k, v))
            pipe.offload(layer, b, k.to(DEV), v.to(DEV))
        pipe.join()
        torch.cuda.current_stream().synchronize()
        for layer, b in enumerate(ids):
            for x, q_slab, s_slab in ((xs[layer][0], pipe.k_quant, pipe.k_scale),
                                      (xs[layer][1], pipe.v_quant, pipe.v_scale)):
                q_ref, s_ref = oracle.quantize_kv_int8(x)
                got_q = torch.cat([q_slab[layer, blk] for blk in b])
                got_s = torch.cat([s_slab[layer, blk] for blk in b])
                assert torch.equal(got_q, q_ref)
                assert bits_equal(got_s.reshape(s_ref.shape), s_ref)


@pytest.mark.parametrize("chunk,h,n", [(16, 2, 1500), (3, 1, 40)])
def test_scattered_offload_writes_only_its_blocks(scb, oracle, chunk, h, n):
    # an offload of a block list in several runs: the scatter kernel writes each block's codes
    # and scales into the mapped slabs (1500 blocks: two launches of at most 960 ids); with
    # 3 tokens x 1 head a block's scales are 6 bytes, not a multiple of 16, so that geometry
    # goes by copies.  Every other block of the slabs keeps its bytes, and a restore of the
    # offloaded blocks (its scales gathered from the mapped slab) matches the oracle.
    import random

    from speccache_b200.cache import KVRestorePipeline

    layers, blocks, d = 2, 2 * n + 5, 32
    rng = random.Random(n)
    ids = rng.sample(range(blocks), n)
    with KVRestorePipeline(layers, blocks, chunk, h, d, device=DEV, max_restore_blocks=n) as pipe:
        pipe.k_quant.fill_(77)
        pipe.v_quant.fill_(-66)
        pipe.k_scale.fill_(0.25)
        pipe.v_scale.fill_(-0.5)
        g = torch.Generator().manual_seed(n)
        k = torch.randn((n * chunk, h, d), generator=g).half()
        v = torch.randn((n * chunk, h, d), generator=g).half()
        pipe.offload(1, ids, k.to(DEV), v.to(DEV))
        pipe.synchronize()
        assert pipe.status() == 0
        kq, ks = oracle.quantize_kv_int8(k)
        vq, vs = oracle.quantize_kv_int8(v)
        where = torch.tensor(ids)
        assert torch.equal(pipe.k_quant[1, where].reshape(kq.shape), kq)
        assert torch.equal(pipe.v_quant[1, where].reshape(vq.shape), vq)
        assert bits_equal(pipe.k_scale[1, where].reshape(ks.shape), ks)
        assert bits_equal(pipe.v_scale[1, where].reshape(vs.shape), vs)
        rest = torch.tensor(sorted(set(range(blocks)) - set(ids)))
        assert (pipe.k_quant[1, rest] == 77).all() and (pipe.v_quant[1, rest] == -66).all()
        assert (pipe.k_scale[1, rest] == 0.25).all() and (pipe.v_scale[1, rest] == -0.5).all()
        assert (pipe.k_quant[0] == 77).all() and (pipe.v_scale[0] == -0.5).all()
        dps = [rng.randint(-4000, 4000) for _ in ids]
        ko = torch.empty((layers, n * chunk, h, d), dtype=torch.float16, device=DEV)
        vo = torch.empty_like(ko)
        pipe.restore(ids, dps, ko, vo)
        pipe.synchronize()
        assert pipe.status() == 0
        kr, vr = oracle.restore_blocks(pipe.k_quant[1], pipe.k_scale[1], pipe.v_quant[1],
                                       pipe.v_scale[1], ids, dps, 10000.0, torch.float16)
        assert bits_equal(vo[1].cpu(), vr)
        torch.testing.assert_close(ko[1].cpu().float(), kr.float(), rtol=1e-2, atol=1e-2)


def test_offload_of_a_repeated_block_keeps_the_last(scb, oracle):
    # a block named twice in one offload ends with the later chunk, as the reference's
    # block-by-block writes leave it (such a list goes by copies in list order, not by the
    # scatter kernel, which would write both at once)
    from speccache_b200.cache import KVRestorePipeline

    layers, blocks, chunk, h, d = 2, 8, 16, 2, 64
    ids = [3, 5, 3]
    with KVRestorePipeline(layers, blocks, chunk, h, d, device=DEV) as pipe:
        assert pipe.offload_plan(ids) == (2, 6)  # quantize K, V; codes + scales per run
        assert pipe.offload_plan([3, 5, 1]) == (4, 0)  # no repeat: the scatter kernels
        g = torch.Generator().manual_seed(5)
        k = torch.randn((len(ids) * chunk, h, d), generator=g).half()
        v = torch.randn((len(ids) * chunk, h, d), generator=g).half()
        pipe.offload(0, ids, k.to(DEV), v.to(DEV))
        pipe.synchronize()
        assert pipe.status() == 0
        for x, q_slab, s_slab in ((k, pipe.k_quant, pipe.k_scale), (v, pipe.v_quant, pipe.v_scale)):
            q_ref, s_ref = oracle.quantize_kv_int8(x)
            q_ref, s_ref = q_ref.view(3, chunk, h, d), s_ref.view(3, chunk, h, 1)
            assert torch.equal(q_slab[0, 3], q_ref[2]) and torch.equal(q_slab[0, 5], q_ref[1])
            assert bits_equal(s_slab[0, 3], s_ref[2]) and bits_equal(s_slab[0, 5], s_ref[1])


def test_pool_async_dma_multi_chunk_parity(scb, oracle):
    # reference tests/test_phase2_engine.py:297-359: 4 chunks with distinct shifts
    from speccache_b200.cache import PinnedKVPool

    chunk, h, d = 128, 8, 128
    pool = PinnedKVPool(8, chunk, h, d, device=DEV)
    g = torch.Generator().manual_seed(77)
    ids = []
    for i in range(4):
        kq, ks = oracle.quantize_kv_int8(torch.randn((chunk, h, d), generator=g))
        vq, vs = oracle.quantize_kv_int8(torch.randn((chunk, h, d), generator=g))
        b = pool.allocate(start_pos=512 * (i + 1))
        pool.write_block(b, kq, ks, vq, vs, start_pos=512 * (i + 1))
        ids.append(b)
    shifts = [100 * i - pool.get_start_pos(b) for i, b in enumerate(ids)]
    k, v = pool.execute_async_dma_and_rope(ids, shifts)
    kr, vr = oracle.restore_blocks(pool.k_quant, pool.k_scale, pool.v_quant, pool.v_scale, ids, shifts)
    torch.testing.assert_close(k.cpu(), kr, rtol=1e-2, atol=1e-2)
    assert bits_equal(v.cpu(), vr)
    pool.close()


def test_engine_routing_decisions_multi_chunk_parity(scb, oracle):
    # reference tests/test_phase2_engine.py:297-359 through the decision records of
    # speccache/cache/engine.py:54-67: chunk c cached at c*128, wanted at c*256; decisions
    # that are not reuse (or have no block) are skipped, empty input gives [0, H, D] fp16
    from speccache_b200.cache import ChunkRoutingDecision, ChunkRoutingStatus, RestoreEngine

    chunk, h, d, n = 64, 4, 64, 4
    S = ChunkRoutingStatus
    with RestoreEngine(chunk_size=chunk, num_kv_heads=h, head_dim=d, max_blocks=16,
                       device=DEV) as engine:
        g = torch.Generator().manual_seed(200)
        data = []
        for c in range(n):
            kq, ks = oracle.quantize_kv_int8(torch.randn((chunk, h, d), generator=g))
            vq, vs = oracle.quantize_kv_int8(torch.randn((chunk, h, d), generator=g))
            toks = list(range(c * 500, c * 500 + chunk))
            bid = engine.register_chunk(toks, c * 128, kq, ks, vq, vs)
            data.append((bid, kq, ks, vq, vs, c * 256 - c * 128))
        decisions = []
        for c, (bid, *_, dp) in enumerate(data):
            st = S.EXACT_REUSE if c % 2 == 0 else S.SEMANTIC_REUSE
            decisions.append(ChunkRoutingDecision(c, c * 256, c * 256 + chunk, (), st,
                                                  block_id=bid, cached_position=c * 128,
                                                  delta_p=dp))
            decisions.append(ChunkRoutingDecision(c, 0, chunk, (), S.CACHE_MISS))
        decisions.insert(3, ChunkRoutingDecision(9, 0, chunk, (), S.SPECULATIVE_DRAFT,
                                                 block_id=data[0][0], delta_p=7))
        k_out, v_out = engine.execute_async_dma_and_rope(decisions)
        assert k_out.shape == (n * chunk, h, d) and k_out.dtype == torch.float16
        for i, (bid, kq, ks, vq, vs, dp) in enumerate(data):
            cos, sin = oracle.compute_rope_cos_sin_delta(dp, d)
            k_ref = oracle.dequant_rope_shift(kq, ks, cos, sin)
            sl = slice(i * chunk, (i + 1) * chunk)
            torch.testing.assert_close(k_out[sl].cpu(), k_ref, rtol=1e-2, atol=1e-2)
            assert bits_equal(v_out[sl].cpu(), oracle.dequant_value(vq, vs))
        # caller-given bf16 destinations are written in place
        kd = torch.empty((n * chunk, h, d), dtype=torch.bfloat16, device=DEV)
        vd = torch.empty_like(kd)
        k2, v2 = engine.execute_async_dma_and_rope(decisions, kd, vd)
        assert k2.data_ptr() == kd.data_ptr() and v2.data_ptr() == vd.data_ptr()
        for i, (bid, kq, ks, vq, vs, dp) in enumerate(data):
            sl = slice(i * chunk, (i + 1) * chunk)
            assert bits_equal(v2[sl].cpu(), oracle.dequant_value(vq, vs, torch.bfloat16))
        misses = [x for x in decisions if x.status in (S.CACHE_MISS, S.SPECULATIVE_DRAFT)]
        e_k, e_v = engine.execute_async_dma_and_rope(misses)
        assert e_k.shape == (0, h, d) and e_v.dtype == torch.float16 and e_k.device == DEV


def test_engine_semantic_shifted_hit(scb, oracle):
    # reference tests/test_phase2_engine.py:57-147 after routing: a chunk rotated at p = 512,
    # reused at p = 128 through a SEMANTIC_REUSE decision (delta_p = -384); the routing itself
    # (radix tree, semantic index) is the reference's and gives this decision
    from speccache_b200.cache import ChunkRoutingDecision, ChunkRoutingStatus, RestoreEngine

    chunk, heads, d = 128, 8, 128
    g = torch.Generator().manual_seed(1234)
    raw_k = torch.randn((chunk, heads, d), generator=g)
    raw_v = torch.randn((chunk, heads, d), generator=g)
    c512, s512 = oracle.compute_rope_cos_sin_delta(512, d)
    cf = torch.cat([c512, c512], -1)[:, None, :].float()
    sf = torch.cat([s512, s512], -1)[:, None, :].float()
    k_rot_512 = (raw_k * cf + oracle.rotate_half(raw_k) * sf).to(torch.float16)
    kq, ks = oracle.quantize_kv_int8(k_rot_512)
    vq, vs = oracle.quantize_kv_int8(raw_v)
    with RestoreEngine(chunk_size=chunk, num_kv_heads=heads, head_dim=d, max_blocks=16,
                       device=DEV) as engine:
        bid = engine.register_chunk(range(1000, 1000 + chunk), 512, kq, ks, vq, vs)
        dec = ChunkRoutingDecision(0, 128, 128 + chunk, tuple(range(5000, 5000 + chunk)),
                                   ChunkRoutingStatus.SEMANTIC_REUSE, similarity=0.96,
                                   block_id=bid, cached_position=512, delta_p=128 - 512)
        k_out, v_out = engine.execute_async_dma_and_rope([dec])
        c, s = oracle.compute_rope_cos_sin_delta(-384, d)
        torch.testing.assert_close(k_out.cpu(), oracle.dequant_rope_shift(kq, ks, c, s),
                                   atol=1e-2, rtol=1e-2)
        assert bits_equal(v_out.cpu(), oracle.dequant_value(vq, vs))
        # and the restored keys are the raw keys rotated at the target position 128
        c128, s128 = oracle.compute_rope_cos_sin_delta(128, d)
        k_128 = raw_k * torch.cat([c128, c128], -1)[:, None, :].float() + \
            oracle.rotate_half(raw_k) * torch.cat([s128, s128], -1)[:, None, :].float()
        torch.testing.assert_close(k_out.cpu().float(), k_128, atol=5e-2, rtol=5e-2)


def test_reconstruct_layer_chunk(scb, oracle):
    from speccache_b200.serving import MultiLayerKVInjector

    inj = MultiLayerKVInjector(2, 4, 64, device=DEV, max_blocks=4, chunk_size=16)
    g = torch.Generator().manual_seed(5)
    kq, ks = oracle.quantize_kv_int8(torch.randn((16, 4, 64), generator=g))
    vq, vs = oracle.quantize_kv_int8(torch.randn((16, 4, 64), generator=g))
    inj.layer_pools[1].allocate(block_id=2, start_pos=64)
    inj.layer_pools[1].write_block(2, kq, ks, vq, vs, start_pos=64)
    k, v = inj.reconstruct_layer_chunk(1, 2, -64)
    c, s = oracle.compute_rope_cos_sin_delta(-64, 64)
    torch.cuda.synchronize()
    torch.testing.assert_close(k.cpu(), oracle.dequant_rope_shift(kq, ks, c, s), rtol=1e-2, atol=1e-2)
    assert bits_equal(v.cpu(), oracle.dequant_value(vq, vs))
    inj.close()
