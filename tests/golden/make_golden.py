"""Generate golden vectors for the KV-restore path by running the reference itself.

Usage (in a container that has the reference checked out; it is not needed on the
GPU machine, which only reads the committed ``.npz`` output)::

    python tests/golden/make_golden.py --reference <reference source tree>

The reference package is imported from its source tree.  Each case records the
inputs and the reference's outputs; ``tests/test_oracle_golden.py`` checks the
oracle against them bit for bit, and the GPU tests check the CUDA kernels against
both.  Fixtures are small (a few hundred KB in total).

Reference functions exercised (``path:line`` in the reference project):

* speccache/kernels/reference.py:122-165  compute_rope_cos_sin_delta
* speccache/kernels/reference.py:179-205  quantize_kv_int8
* speccache/kernels/reference.py:212-276  pytorch_eager_dequant_rope_shift
* speccache/kernels/reference.py:283-307  dequant_value_ref
* speccache/cache/pinned_pool.py:392-464  PinnedKVPool.get_coalesced_views
* speccache/serving/kv_injector.py:392-498 MultiLayerKVInjector.reconstruct_and_inject_multi_layer (CPU path)
* speccache/serving/kv_injector.py:246-322 MultiLayerKVInjector.apply_rope_shift, inject_layer_kv,
  inject_multi_layer (CPU path)
"""

from __future__ import annotations

import argparse
import importlib.util
import logging
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _load_reference_kernels(ref_root: str):
    """Import speccache/kernels/reference.py alone (it only depends on torch)."""
    path = os.path.join(ref_root, "speccache", "kernels", "reference.py")
    spec = importlib.util.spec_from_file_location("_sc_ref_kernels", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _t2n(x: torch.Tensor) -> np.ndarray:
    """Tensor -> numpy; fp16/bf16 are stored as their raw 16-bit patterns."""
    x = x.detach().cpu().contiguous()
    if x.dtype == torch.bfloat16:
        return x.view(torch.int16).numpy().view(np.uint16)
    if x.dtype == torch.float16:
        return x.numpy().view(np.uint16)
    return x.numpy()


def make_quantize(ref, out: dict) -> None:
    # The reference's own known-answer test (tests/test_correctness.py:80-88).
    x = torch.tensor([[[-127.0, 0.0, 63.5, 127.0]]], dtype=torch.float32)
    q, s = ref.quantize_kv_int8(x)
    out["q_kat_x"], out["q_kat_q"], out["q_kat_s"] = _t2n(x), _t2n(q), _t2n(s)

    cases = []
    g = torch.Generator().manual_seed(7)
    # fp32 N(0,1), odd token count
    cases.append(("f32", torch.randn((17, 4, 64), generator=g, dtype=torch.float32)))
    # fp16 N(0,1) with 2% outlier channels x10 (the Qwen-like round-trip config)
    x16 = torch.randn((33, 4, 128), generator=g, dtype=torch.float32)
    ch = torch.randperm(128, generator=g)[:3]
    x16[..., ch] *= 10.0
    cases.append(("f16", x16.to(torch.float16)))
    # bf16 input
    cases.append(("bf16", torch.randn((9, 2, 64), generator=g).to(torch.bfloat16)))
    # rows that are all zero, tiny (subnormal scale), ties at .5 and huge values
    xe = torch.zeros((6, 2, 32), dtype=torch.float32)
    xe[1] = 1e-7
    xe[2, :, :] = torch.arange(32, dtype=torch.float32) - 15.5  # .5 ties
    xe[3, 0, :] = 65504.0
    xe[3, 1, :] = -3.0e-5
    xe[4] = torch.linspace(-1.0, 1.0, 32)
    xe[5, :, 0] = 127.0
    xe[5, :, 1:] = torch.arange(31, dtype=torch.float32) + 0.5
    cases.append(("edge_f32", xe))
    # fp16 ties: values k + 0.5 with scale exactly 1 (amax 127)
    xt = torch.zeros((4, 1, 16), dtype=torch.float32)
    xt[:, :, 0] = 127.0
    xt[:, :, 1:] = torch.tensor([0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 63.5, 64.5, -63.5,
                                 -64.5, 125.5, 126.5, -126.5, 3.5, 4.5])
    cases.append(("ties_f16", xt.to(torch.float16)))

    names = []
    for name, x in cases:
        q, s = ref.quantize_kv_int8(x)
        out[f"q_{name}_x"], out[f"q_{name}_q"], out[f"q_{name}_s"] = _t2n(x), _t2n(q), _t2n(s)
        out[f"q_{name}_xdtype"] = np.array(str(x.dtype).replace("torch.", ""))
        names.append(name)
    out["q_cases"] = np.array(names)


def make_tables(ref, out: dict) -> None:
    dps = [-123456, -9000, -512, -350, -1, 0, 1, 12, 15, 27, 42, 250, 600, 1024, 2048,
           3000, 4095, 8192, 32768, 123457]
    out["tab_dps"] = np.array(dps, dtype=np.int64)
    for d in (64, 128):
        for theta in (10000.0, 500000.0, 1000000.0):
            c, s = ref.compute_rope_cos_sin_delta(torch.tensor(dps), d, theta_base=theta)
            key = f"tab_d{d}_th{int(theta)}"
            out[key + "_cos"], out[key + "_sin"] = _t2n(c), _t2n(s)


def make_shift(ref, out: dict) -> None:
    cases = [
        # (name, T, H, D, dp, theta, per_token)
        ("t17_h4_d64_m512", 17, 4, 64, -512, 10000.0, False),
        ("t33_h8_d128_p1024", 33, 8, 128, 1024, 10000.0, False),
        ("t16_h2_d128_th5e5", 16, 2, 128, 3000, 500000.0, False),
        ("t24_h4_d128_th1e6", 24, 4, 128, 2048, 1000000.0, False),
        ("t20_h3_d64_pertok", 20, 3, 64, None, 10000.0, True),
        ("t5_h1_d32_zero", 5, 1, 32, 0, 10000.0, False),
    ]
    names = []
    for idx, (name, t, h, d, dp, theta, per_tok) in enumerate(cases):
        torch.manual_seed(42 + idx)
        raw = torch.randn((t, h, d), dtype=torch.float32)
        kq, ks = ref.quantize_kv_int8(raw)
        if per_tok:
            dps = torch.randint(-4096, 4096, (t,))
            c, s = ref.compute_rope_cos_sin_delta(dps, d, theta_base=theta)
        else:
            c, s = ref.compute_rope_cos_sin_delta(torch.tensor([dp]), d, theta_base=theta)
            dps = torch.tensor([dp])
        k = ref.pytorch_eager_dequant_rope_shift(kq, ks, c, s)
        if dp is not None and theta == 10000.0:
            # the delta_p convenience path must agree with the explicit-table path
            k2 = ref.pytorch_eager_dequant_rope_shift(kq, ks, delta_p=dp)
            assert torch.equal(k, k2)
        torch.manual_seed(1337 + idx)
        rawv = torch.randn((t, h, d), dtype=torch.float32)
        vq, vs = ref.quantize_kv_int8(rawv)
        v = ref.dequant_value_ref(vq, vs)
        p = f"sh_{name}_"
        out[p + "kq"], out[p + "ks"], out[p + "cos"], out[p + "sin"] = (
            _t2n(kq), _t2n(ks), _t2n(c), _t2n(s))
        out[p + "dps"] = dps.numpy().astype(np.int64)
        out[p + "theta"] = np.array(theta)
        out[p + "k"], out[p + "vq"], out[p + "vs"], out[p + "v"] = (
            _t2n(k), _t2n(vq), _t2n(vs), _t2n(v))
        names.append(name)
    out["sh_cases"] = np.array(names)


def make_pool_and_injector(ref_root: str, out: dict) -> None:
    """PinnedKVPool gather + MultiLayerKVInjector CPU restore, run by the reference."""
    sys.path.insert(0, ref_root)
    logging.disable(logging.CRITICAL)
    from speccache.cache.pinned_pool import PinnedKVPool  # noqa: E402
    from speccache.serving.kv_injector import MultiLayerKVInjector, SpecDynamicCache  # noqa: E402

    ref = _load_reference_kernels(ref_root)
    chunk, h, d, blocks = 8, 2, 64, 6
    pool = PinnedKVPool(max_blocks=blocks, chunk_size=chunk, num_heads=h, head_dim=d)
    g = torch.Generator().manual_seed(5)
    for b in range(blocks):
        pool.allocate(block_id=b, start_pos=b * chunk)
        kq, ks = ref.quantize_kv_int8(torch.randn((chunk, h, d), generator=g))
        vq, vs = ref.quantize_kv_int8(torch.randn((chunk, h, d), generator=g))
        pool.write_block(b, kq, ks, vq, vs, start_pos=b * chunk)
    order = [4, 1, 5, 2]
    gk, gks, gv, gvs = pool.get_coalesced_views(order)
    out["pool_kq"], out["pool_ks"] = _t2n(pool.k_quant), _t2n(pool.k_scale)
    out["pool_vq"], out["pool_vs"] = _t2n(pool.v_quant), _t2n(pool.v_scale)
    out["pool_order"] = np.array(order, dtype=np.int32)
    out["pool_gk"], out["pool_gks"], out["pool_gv"], out["pool_gvs"] = (
        _t2n(gk), _t2n(gks), _t2n(gv), _t2n(gvs))

    layers = 2
    inj = MultiLayerKVInjector(layers, h, d, device=torch.device("cpu"), max_blocks=blocks,
                               chunk_size=chunk)
    for layer in range(layers):
        for b in range(blocks):
            inj.layer_pools[layer].allocate(block_id=b, start_pos=b * chunk)
            kq, ks = ref.quantize_kv_int8(torch.randn((chunk, h, d), generator=g))
            vq, vs = ref.quantize_kv_int8(torch.randn((chunk, h, d), generator=g))
            inj.layer_pools[layer].write_block(b, kq, ks, vq, vs, start_pos=b * chunk)
    for tag, dps in (("const", [-256, -256, -256]), ("mixed", [-256, 100, 4000])):
        cache = SpecDynamicCache()
        legacy = inj.reconstruct_and_inject_multi_layer(cache, [3, 0, 5], dps)
        for layer, (k, v) in enumerate(legacy):
            out[f"inj_{tag}_k{layer}"], out[f"inj_{tag}_v{layer}"] = _t2n(k), _t2n(v)
        out[f"inj_{tag}_dps"] = np.array(dps, dtype=np.int64)
    out["inj_blocks"] = np.array([3, 0, 5], dtype=np.int32)
    out["inj_kq"], out["inj_ks"] = _t2n(inj.unified_k_quant), _t2n(inj.unified_k_scale)
    out["inj_vq"], out["inj_vs"] = _t2n(inj.unified_v_quant), _t2n(inj.unified_v_scale)


def make_key_shift_and_inject(ref_root: str, out: dict) -> None:
    """RoPE shift of dequantised keys and the cache injection built on it, run by the reference."""
    sys.path.insert(0, ref_root)
    logging.disable(logging.CRITICAL)
    from speccache.serving.kv_injector import MultiLayerKVInjector, SpecDynamicCache  # noqa: E402

    g = torch.Generator().manual_seed(11)
    cases = [("f16_d64", torch.float16, 24, 3, 64, [-384, 1, 4095, 70000]),
             ("f16_d128", torch.float16, 17, 2, 128, [-8192, 513]),
             ("bf16_d128", torch.bfloat16, 9, 4, 128, [2048])]
    for tag, dtype, t, h, d, dps in cases:
        inj = MultiLayerKVInjector(1, h, d, device=torch.device("cpu"), max_blocks=1, chunk_size=8)
        k = (torch.randn((t, h, d), generator=g) * 4).to(dtype)
        out[f"ks_{tag}_k"] = _t2n(k)
        out[f"ks_{tag}_dps"] = np.array(dps, dtype=np.int64)
        for i, dp in enumerate(dps):
            out[f"ks_{tag}_out{i}"] = _t2n(inj.apply_rope_shift(k, dp))
        # the model layout [1, H, T, D] is shifted in the same layout
        out[f"ks_{tag}_out4d"] = _t2n(inj.apply_rope_shift(inj.format_to_model_layout(k), dps[0]))
    # injection: two appends to one layer (the second shifted), then a multi-layer injection
    h, d, t = 2, 64, 12
    inj = MultiLayerKVInjector(2, h, d, device=torch.device("cpu"), max_blocks=1, chunk_size=8)
    ks = [torch.randn((t, h, d), generator=g).half() for _ in range(4)]
    vs = [torch.randn((t, h, d), generator=g).half() for _ in range(4)]
    cache = SpecDynamicCache()
    inj.inject_layer_kv(cache, 0, ks[0], vs[0])
    inj.inject_layer_kv(cache, 0, ks[1], vs[1], delta_p=-700)
    out["inj1_k"], out["inj1_v"] = _t2n(cache[0][0]), _t2n(cache[0][1])
    cache = SpecDynamicCache()
    inj.inject_multi_layer(cache, ks[2:], vs[2:], delta_p=300)
    for layer in range(2):
        out[f"injm_k{layer}"], out[f"injm_v{layer}"] = _t2n(cache[layer][0]), _t2n(cache[layer][1])
    for i in range(4):
        out[f"inj_in_k{i}"], out[f"inj_in_v{i}"] = _t2n(ks[i]), _t2n(vs[i])


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SPECCACHE_REFERENCE"),
                    help="the reference project's source tree (or set SPECCACHE_REFERENCE)")
    ap.add_argument("--out", default=os.path.join(HERE, "golden_path1.npz"))
    args = ap.parse_args()
    if not args.reference:
        ap.error("give the reference's source tree with --reference or SPECCACHE_REFERENCE")
    torch.set_num_threads(1)
    ref = _load_reference_kernels(args.reference)
    out: dict = {}
    make_quantize(ref, out)
    make_tables(ref, out)
    make_shift(ref, out)
    make_pool_and_injector(args.reference, out)
    make_key_shift_and_inject(args.reference, out)
    np.savez_compressed(args.out, **out)
    print(f"wrote {args.out}: {len(out)} arrays, {os.path.getsize(args.out)} bytes")


if __name__ == "__main__":
    main()
