"""Parity at the full sizes of the benchmark configurations (GPU).

Each test runs one configuration at its full size and checks every output element against
the oracle (layer by layer, on the host) or, for the 70B slab, every layer against the same
arithmetic in torch on the GPU plus three whole layers against the oracle:

* Llama-3-8B (32 layers x T=8192 x 8 heads x 128, theta 5e5, one shift from the seed, bf16):
  GPU quantize bit-exact; restore with the shift expanded in the kernel within the reference
  tolerance (and at least 98 % of K bit-equal); restore with the oracle's tables bit-exact;
  V bit-exact.
* Qwen-2.5-7B-like round trip (28 x 16384 x 4 x 128, 2 % outlier channels x10, theta 1e6,
  shift 2048, fp16): the same checks.
* Ragged paged batch (64 requests, lengths U[256, 8192], shifts U[0, 4096], shuffled page
  table): every request against the oracle's gather + eager restore.
* Llama-3-70B host slab (80 x 32768 x 8 x 128, 5.4 GB pinned, shift 8192): the pipeline restore
  of every layer; V bit-exact and K within tolerance against torch on the GPU for all layers,
  and layers 0, 41 and 79 against the oracle.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import bits_equal

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0) if torch.cuda.is_available() else None
SEED = 1234


def _fp16_inputs(layers, t, h, d, seed, outliers=False):
    gen = torch.Generator(device=DEV)
    gen.manual_seed(seed)
    out = []
    for _ in range(2):
        x = torch.randn((layers, t, h, d), generator=gen, device=DEV)
        if outliers:
            ch = torch.randperm(d, generator=gen, device=DEV)[: max(1, round(0.02 * d))]
            x[..., ch] *= 10.0
        out.append(x.to(torch.float16))
    return out


def _k_close(k_gpu: torch.Tensor, k_ref: torch.Tensor, min_exact: float = 0.98) -> None:
    torch.testing.assert_close(k_gpu.float(), k_ref.float(), rtol=1e-2, atol=1e-2)
    exact = (k_gpu.view(torch.int16) == k_ref.view(torch.int16)).float().mean().item()
    assert exact >= min_exact, exact


def _quantize_restore_config(scb, oracle, layers, t, h, d, theta, dp, out_dtype, outliers):
    xk, xv = _fp16_inputs(layers, t, h, d, SEED, outliers)
    q, s = [], []
    for x in (xk, xv):
        qq, ss = scb.quantize_kv_int8(x.view(layers * t, h, d))
        q.append(qq.view(layers, t, h, d))
        s.append(ss.view(layers, t, h, 1))
    kq, vq = q
    ks, vs = s
    k_out, v_out = scb.restore_layers(kq, ks, vq, vs, delta_p=dp, theta=theta,
                                      out_dtype=out_dtype)
    cos, sin = oracle.compute_rope_cos_sin_delta(dp, d, theta)
    cos_d, sin_d = cos.to(DEV), sin.to(DEV)
    k_tab = torch.empty((t, h, d), dtype=out_dtype, device=DEV)
    v_tab = torch.empty_like(k_tab)
    torch.cuda.synchronize()
    for layer in range(layers):
        kq_h, vq_h = kq[layer].cpu(), vq[layer].cpu()
        ks_h, vs_h = ks[layer].cpu(), vs[layer].cpu()
        for x, qh, sh in ((xk, kq_h, ks_h), (xv, vq_h, vs_h)):
            q_ref, s_ref = oracle.quantize_kv_int8(x[layer].cpu())
            assert torch.equal(qh, q_ref), layer
            assert bits_equal(sh, s_ref), layer
        k_ref = oracle.dequant_rope_shift(kq_h, ks_h, cos, sin, out_dtype)
        v_ref = oracle.dequant_value(vq_h, vs_h, out_dtype)
        _k_close(k_out[layer].cpu(), k_ref)
        assert bits_equal(v_out[layer].cpu(), v_ref), layer
        scb.dequant_kv_cache(kq[layer], ks[layer], vq[layer], vs[layer], cos_d, sin_d,
                             k_out=k_tab, v_out=v_tab, fp32_intermediate=False)
        assert bits_equal(k_tab.cpu(), k_ref), layer
        assert bits_equal(v_tab.cpu(), v_ref), layer


def test_llama8b_full_size(scb, oracle):
    dp = int(np.random.default_rng(SEED).integers(1, 4097))
    _quantize_restore_config(scb, oracle, 32, 8192, 8, 128, 500000.0, dp, torch.bfloat16, False)


def test_qwen_round_trip_full_size(scb, oracle):
    _quantize_restore_config(scb, oracle, 28, 16384, 4, 128, 1e6, 2048, torch.float16, True)


def test_ragged_paged_full_size(scb, oracle):
    h, d, page, n_req = 8, 128, 64, 64
    rng = np.random.default_rng(SEED)
    lens = rng.integers(256, 8193, n_req)
    dps = rng.integers(0, 4097, n_req)
    pages = [(int(n) + page - 1) // page for n in lens]
    n_pool = sum(pages)
    perm = rng.permutation(n_pool)
    table = np.zeros((n_req, max(pages)), np.int32)
    k = 0
    for r, n in enumerate(pages):
        table[r, :n] = perm[k:k + n]
        k += n
    gen = torch.Generator(device=DEV)
    gen.manual_seed(SEED)
    pool = []
    for _ in range(2):
        x = torch.randn((n_pool * page, h, d), generator=gen, device=DEV).to(torch.float16)
        q, s = scb.quantize_kv_int8(x)
        pool += [q.view(n_pool, page, h, d), s.view(n_pool, page, h, 1)]
    pkq, pks, pvq, pvs = pool
    k_out, v_out, cu = scb.restore_paged(pkq, pks, pvq, pvs, torch.from_numpy(table),
                                         lens.tolist(), dps.tolist(), theta=500000.0)
    torch.cuda.synchronize()
    assert scb.paged_status(DEV) == 0
    host = [t.cpu() for t in (pkq, pks, pvq, pvs)]
    for r in range(n_req):
        ids = table[r, :pages[r]].tolist()
        sub = [t[ids] for t in host]
        (kr, vr), = oracle.restore_paged(*sub, torch.arange(len(ids), dtype=torch.int32)[None],
                                         [int(lens[r])], [int(dps[r])], theta_base=500000.0,
                                         out_dtype=torch.bfloat16)
        a, b = int(cu[r]), int(cu[r + 1])
        _k_close(k_out[a:b].cpu(), kr)
        assert bits_equal(v_out[a:b].cpu(), vr), r


def test_llama70b_host_slab_full_size(scb, oracle):
    from speccache_b200.cache import KVRestorePipeline

    layers, t, h, d, chunk, dp, theta = 80, 32768, 8, 128, 64, 8192, 500000.0
    n_blocks = t // chunk
    gen = torch.Generator(device=DEV)
    gen.manual_seed(SEED)
    cos, sin = oracle.compute_rope_cos_sin_delta(dp, d, theta)
    cos_f = torch.cat([cos, cos], -1).float().to(DEV)[:, None, :]
    sin_f = torch.cat([sin, sin], -1).float().to(DEV)[:, None, :]
    with KVRestorePipeline(layers, n_blocks, chunk, h, d, device=DEV, n_slots=3) as pipe:
        for layer in range(layers):
            for q_slab, s_slab in ((pipe.k_quant, pipe.k_scale), (pipe.v_quant, pipe.v_scale)):
                x = torch.randn((t, h, d), generator=gen, device=DEV).to(torch.float16)
                qd, sd = scb.quantize_kv_int8(x)
                q_slab[layer].view(t, h, d).copy_(qd.cpu())
                s_slab[layer].view(t, h, 1).copy_(sd.cpu())
        k_out = torch.empty((layers, t, h, d), dtype=torch.bfloat16, device=DEV)
        v_out = torch.empty_like(k_out)
        pipe.restore(list(range(n_blocks)), [dp] * n_blocks, list(k_out), list(v_out), theta=theta)
        pipe.synchronize()
        assert pipe.status() == 0
        for layer in range(layers):
            kq = pipe.k_quant[layer].view(t, h, d).to(DEV)
            ks = pipe.k_scale[layer].view(t, h, 1).to(DEV)
            vq = pipe.v_quant[layer].view(t, h, d).to(DEV)
            vs = pipe.v_scale[layer].view(t, h, 1).to(DEV)
            # the eager arithmetic in torch on the GPU (fp16 intermediate, fp32 rotation)
            v_ref = (vq.float() * vs.float()).to(torch.bfloat16)
            x = (kq.float() * ks.float()).half().float()
            rot = torch.cat([-x[..., d // 2:], x[..., :d // 2]], -1)
            k_ref = (x * cos_f + rot * sin_f).to(torch.bfloat16)
            assert torch.equal(v_out[layer].view(torch.int16), v_ref.view(torch.int16)), layer
            torch.testing.assert_close(k_out[layer].float(), k_ref.float(), rtol=1e-2, atol=1e-2)
            if layer in (0, 41, 79):
                k_h, v_h = oracle.restore_blocks(
                    pipe.k_quant[layer], pipe.k_scale[layer], pipe.v_quant[layer],
                    pipe.v_scale[layer], list(range(n_blocks)), [dp] * n_blocks, theta,
                    torch.bfloat16)
                _k_close(k_out[layer].cpu(), k_h)
                assert bits_equal(v_out[layer].cpu(), v_h), layer
