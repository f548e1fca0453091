"""Pin the CPU oracle to the reference: every golden vector must match bit for bit.

The fixtures were produced by running the reference's own functions
(tests/golden/make_golden.py).  These tests run on CPU only.
"""

from __future__ import annotations

import torch

from conftest import as_tensor, bits_equal


def test_quantize_known_answer(golden, oracle):
    # reference tests/test_correctness.py:80-88: 63.5 -> 64 (half to even), scale fp16 1.0
    x = as_tensor(golden["q_kat_x"])
    q, s = oracle.quantize_kv_int8(x)
    assert torch.equal(q, torch.tensor([[[-127, 0, 64, 127]]], dtype=torch.int8))
    assert s.dtype == torch.float16 and s.shape == (1, 1, 1) and float(s) == 1.0
    assert torch.equal(q, as_tensor(golden["q_kat_q"]))
    assert bits_equal(s, as_tensor(golden["q_kat_s"]))


def test_quantize_cases_bit_exact(golden, oracle):
    for name in golden["q_cases"]:
        name = str(name)
        xd = str(golden[f"q_{name}_xdtype"])
        x = as_tensor(golden[f"q_{name}_x"], xd)
        q, s = oracle.quantize_kv_int8(x)
        assert torch.equal(q, as_tensor(golden[f"q_{name}_q"])), name
        assert bits_equal(s, as_tensor(golden[f"q_{name}_s"])), name


def test_rope_tables_bit_exact(golden, oracle):
    dps = golden["tab_dps"]
    for d in (64, 128):
        for theta in (10000.0, 500000.0, 1000000.0):
            key = f"tab_d{d}_th{int(theta)}"
            c, s = oracle.compute_rope_cos_sin_delta(torch.from_numpy(dps), d, theta)
            assert bits_equal(c, as_tensor(golden[key + "_cos"])), key
            assert bits_equal(s, as_tensor(golden[key + "_sin"])), key


def test_dequant_shift_and_value_bit_exact(golden, oracle):
    for name in golden["sh_cases"]:
        p = f"sh_{name}_"
        kq, ks = as_tensor(golden[p + "kq"]), as_tensor(golden[p + "ks"])
        c, s = as_tensor(golden[p + "cos"]), as_tensor(golden[p + "sin"])
        k = oracle.dequant_rope_shift(kq, ks, c, s)
        assert bits_equal(k, as_tensor(golden[p + "k"])), name
        # the tables themselves come from the oracle's table function too
        dps = golden[p + "dps"]
        c2, s2 = oracle.compute_rope_cos_sin_delta(
            torch.from_numpy(dps), kq.shape[-1], float(golden[p + "theta"]))
        assert bits_equal(c2, c) and bits_equal(s2, s), name
        v = oracle.dequant_value(as_tensor(golden[p + "vq"]), as_tensor(golden[p + "vs"]))
        assert bits_equal(v, as_tensor(golden[p + "v"])), name


def test_gather_blocks_matches_pool(golden, oracle):
    order = golden["pool_order"].tolist()
    for slab, ref in (("pool_kq", "pool_gk"), ("pool_ks", "pool_gks"),
                      ("pool_vq", "pool_gv"), ("pool_vs", "pool_gvs")):
        got = oracle.gather_blocks(as_tensor(golden[slab]), order)
        assert bits_equal(got, as_tensor(golden[ref])), slab


def test_multi_layer_injector_restore(golden, oracle):
    blocks = golden["inj_blocks"].tolist()
    kq_all, ks_all = as_tensor(golden["inj_kq"]), as_tensor(golden["inj_ks"])
    vq_all, vs_all = as_tensor(golden["inj_vq"]), as_tensor(golden["inj_vs"])
    for tag in ("const", "mixed"):
        dps = golden[f"inj_{tag}_dps"].tolist()
        for layer in range(kq_all.shape[0]):
            k, v = oracle.restore_blocks(kq_all[layer], ks_all[layer], vq_all[layer],
                                         vs_all[layer], blocks, dps)
            assert bits_equal(oracle.to_model_layout(k), as_tensor(golden[f"inj_{tag}_k{layer}"]))
            assert bits_equal(oracle.to_model_layout(v), as_tensor(golden[f"inj_{tag}_v{layer}"]))


def test_restore_paged_equals_per_request_blocks(oracle):
    # The ragged restore is the block restore applied per request, cut to seq_len.
    g = torch.Generator().manual_seed(3)
    n_pages, page, h, d = 10, 4, 2, 32
    pkq = torch.randint(-127, 128, (n_pages, page, h, d), generator=g, dtype=torch.int8)
    pks = (torch.rand((n_pages, page, h, 1), generator=g) * 0.05 + 1e-3).to(torch.float16)
    pvq = torch.randint(-127, 128, (n_pages, page, h, d), generator=g, dtype=torch.int8)
    pvs = (torch.rand((n_pages, page, h, 1), generator=g) * 0.05 + 1e-3).to(torch.float16)
    table = torch.tensor([[7, 2, 9], [0, 5, 0], [3, 0, 0]], dtype=torch.int32)
    lens, dps = [11, 5, 4], [100, -7, 0]
    got = oracle.restore_paged(pkq, pks, pvq, pvs, table, lens, dps)
    for r, (k, v) in enumerate(got):
        n = (lens[r] + page - 1) // page
        kb, vb = oracle.restore_blocks(pkq, pks, pvq, pvs, table[r, :n].tolist(), [dps[r]] * n)
        assert bits_equal(k, kb[: lens[r]]) and bits_equal(v, vb[: lens[r]])


KEY_SHIFT_CASES = ("f16_d64", "f16_d128", "bf16_d128")


def test_key_shift_matches_reference(golden, oracle):
    # MultiLayerKVInjector.apply_rope_shift (kv_injector.py:246-283), both layouts
    for tag in KEY_SHIFT_CASES:
        dt = "bfloat16" if tag.startswith("bf16") else "float16"
        k = as_tensor(golden[f"ks_{tag}_k"], dt)
        dps = golden[f"ks_{tag}_dps"].tolist()
        for i, dp in enumerate(dps):
            assert bits_equal(oracle.apply_rope_shift(k, dp), as_tensor(golden[f"ks_{tag}_out{i}"], dt))
        k4 = oracle.to_model_layout(k)
        assert bits_equal(oracle.apply_rope_shift(k4, dps[0]), as_tensor(golden[f"ks_{tag}_out4d"], dt))
        assert oracle.apply_rope_shift(k, 0) is k


def test_injection_matches_reference(golden, oracle):
    # inject_layer_kv / inject_multi_layer (kv_injector.py:285-322): model layout, shift, append
    ks = [as_tensor(golden[f"inj_in_k{i}"]) for i in range(4)]
    vs = [as_tensor(golden[f"inj_in_v{i}"]) for i in range(4)]
    k1 = torch.cat([oracle.to_model_layout(ks[0]),
                    oracle.apply_rope_shift(oracle.to_model_layout(ks[1]), -700)], dim=-2)
    v1 = torch.cat([oracle.to_model_layout(vs[0]), oracle.to_model_layout(vs[1])], dim=-2)
    assert bits_equal(k1, as_tensor(golden["inj1_k"])) and bits_equal(v1, as_tensor(golden["inj1_v"]))
    for layer in range(2):
        k = oracle.apply_rope_shift(oracle.to_model_layout(ks[2 + layer]), 300)
        assert bits_equal(k, as_tensor(golden[f"injm_k{layer}"]))
        assert bits_equal(oracle.to_model_layout(vs[2 + layer]), as_tensor(golden[f"injm_v{layer}"]))
