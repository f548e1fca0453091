"""GPU parity of the restore kernels against the CPU oracle and the reference's goldens.

Tolerances: where the cos/sin tables are given, K is compared bit for bit with the
reference's torch arithmetic of the same kind: the eager one (fp16-rounded dequant, fp32
rotation) for the ``*_ref`` names and ``fp32_intermediate=False``, the fp32-intermediate one
(the Triton kernel's, and what Inductor compiles the eager code to) for the Triton-named
wrappers' default and the ``*_compiled`` names; V always bit for bit.  Where the kernel builds cos/sin itself from delta_p, each table entry may differ
from torch's by one fp16 ulp in rare cases (torch's float32 cos/sin is not correctly
rounded), so K is checked with the reference's own tolerance, rtol = atol = 1e-2
(reference tests/test_correctness.py:169), plus an exact-match fraction.
"""

from __future__ import annotations

import pytest
import torch

from conftest import as_tensor, bits_equal

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0) if torch.cuda.is_available() else None


def _quantized(oracle, t, h, d, seed, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    raw = torch.randn((t, h, d), generator=g, dtype=torch.float32).to(dtype)
    return oracle.quantize_kv_int8(raw)


# Every key entry point of the reference's kernels/__init__.py:3-21, with the arithmetic of
# the function it replaces: True = fp16 intermediate (eager), False = fp32 intermediate.
KEY_NAMES = [
    ("pytorch_eager_dequant_rope_shift", True),
    ("dequant_and_rope_key_ref", True),
    ("pytorch_compiled_dequant_rope_shift", False),
    ("dequant_and_rope_key_compiled", False),
    ("triton_fused_k_dequant_rope_shift", False),
    ("dequant_and_rope_key", False),
]
VALUE_NAMES = ["dequant_value", "dequant_value_ref", "dequant_value_compiled"]


@pytest.mark.parametrize("t", [1, 17, 128, 511, 2048, 4096])
@pytest.mark.parametrize("h", [4, 8, 32])
@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("delta_p", [-512, 0, 1024])
def test_k_shift_grid_every_name_bitwise(scb, oracle, t, h, d, delta_p):
    # the reference's 108-case grid (tests/test_correctness.py:142-169), for every key and
    # value name the reference exports
    kq, ks = _quantized(oracle, t, h, d, 42)
    vq, vs = _quantized(oracle, t, h, d, 43)
    cos, sin = oracle.compute_rope_cos_sin_delta(delta_p, d)
    refs = {x16: oracle.dequant_rope_shift(kq, ks, cos, sin, fp16_intermediate=x16)
            for x16 in (True, False)}
    v_ref = oracle.dequant_value(vq, vs)
    kd, sd, cd, snd = kq.to(DEV), ks.to(DEV), cos.to(DEV), sin.to(DEV)
    outs = {name: getattr(scb, name)(kd, sd, cd, snd) for name, _ in KEY_NAMES}
    v_outs = {name: getattr(scb, name)(vq.to(DEV), vs.to(DEV)) for name in VALUE_NAMES}
    torch.cuda.synchronize()
    for name, x16 in KEY_NAMES:
        out = outs[name].cpu()
        assert out.dtype == torch.float16 and out.shape == (t, h, d), name
        torch.testing.assert_close(out, refs[x16], rtol=1e-2, atol=1e-2)
        assert bits_equal(out, refs[x16]), name
    for name in VALUE_NAMES:
        assert bits_equal(v_outs[name].cpu(), v_ref), name


def test_reference_names_reject_cpu_tensors(scb, oracle):
    kq, ks = _quantized(oracle, 4, 2, 64, 1)
    cos, sin = oracle.compute_rope_cos_sin_delta(3, 64)
    for name, _ in KEY_NAMES:
        with pytest.raises(RuntimeError):
            getattr(scb, name)(kq, ks, cos, sin)
    for name in VALUE_NAMES:
        with pytest.raises(RuntimeError):
            getattr(scb, name)(kq, ks)


def test_reference_names_with_delta_p_and_out(scb, oracle):
    # the delta_p form (theta 10000, as the reference) and a preallocated out, per name
    t, h, d, dp = 300, 8, 128, 777
    kq, ks = _quantized(oracle, t, h, d, 8)
    cos, sin = oracle.compute_rope_cos_sin_delta(dp, d)
    for name, x16 in KEY_NAMES:
        ref = oracle.dequant_rope_shift(kq, ks, cos, sin, fp16_intermediate=x16)
        pre = torch.empty((t, h, d), dtype=torch.float16, device=DEV)
        ret = getattr(scb, name)(kq.to(DEV), ks.to(DEV), out=pre, delta_p=dp)
        torch.cuda.synchronize()
        assert ret.data_ptr() == pre.data_ptr(), name
        torch.testing.assert_close(ret.cpu(), ref, rtol=1e-2, atol=1e-2)
        same = (ret.cpu().view(torch.int16) == ref.view(torch.int16)).float().mean().item()
        assert same > 0.99, (name, same)


def test_golden_vectors(scb, golden):
    for name in golden["sh_cases"]:
        p = f"sh_{name}_"
        kq, ks = as_tensor(golden[p + "kq"]).to(DEV), as_tensor(golden[p + "ks"]).to(DEV)
        cos, sin = as_tensor(golden[p + "cos"]).to(DEV), as_tensor(golden[p + "sin"]).to(DEV)
        vq, vs = as_tensor(golden[p + "vq"]).to(DEV), as_tensor(golden[p + "vs"]).to(DEV)
        k, v = scb.dequant_kv_cache(kq, ks, vq, vs, cos, sin, fp32_intermediate=False)
        torch.cuda.synchronize()
        assert bits_equal(k.cpu(), as_tensor(golden[p + "k"])), name
        assert bits_equal(v.cpu(), as_tensor(golden[p + "v"])), name


@pytest.mark.parametrize("theta", [10000.0, 500000.0, 1000000.0])
@pytest.mark.parametrize("delta_p", [-4096, -350, 1, 2048, 4095, 8192, 32768])
def test_delta_p_path_in_kernel_tables(scb, oracle, theta, delta_p):
    t, h, d = 257, 8, 128
    kq, ks = _quantized(oracle, t, h, d, 7)
    cos, sin = oracle.compute_rope_cos_sin_delta(delta_p, d, theta)
    ref = oracle.dequant_rope_shift(kq, ks, cos, sin, fp16_intermediate=False)
    out = scb.triton_fused_k_dequant_rope_shift(kq.to(DEV), ks.to(DEV), delta_p=delta_p, theta=theta)
    torch.cuda.synchronize()
    torch.testing.assert_close(out.cpu(), ref, rtol=1e-2, atol=1e-2)
    same = (out.cpu().view(torch.int16) == ref.view(torch.int16)).float().mean().item()
    assert same > 0.99, same


def test_delta_p_device_scalar_and_per_token(scb, oracle):
    t, h, d = 100, 4, 64
    kq, ks = _quantized(oracle, t, h, d, 11)
    cos, sin = oracle.compute_rope_cos_sin_delta(-77, d)
    ref = oracle.dequant_rope_shift(kq, ks, cos, sin, fp16_intermediate=False)
    out = scb.triton_fused_k_dequant_rope_shift(kq.to(DEV), ks.to(DEV),
                                                delta_p=torch.tensor([-77], device=DEV))
    torch.testing.assert_close(out.cpu(), ref, rtol=1e-2, atol=1e-2)
    dps = torch.randint(-3000, 3000, (t,), generator=torch.Generator().manual_seed(1))
    cos_t, sin_t = oracle.compute_rope_cos_sin_delta(dps, d)
    ref_t = oracle.dequant_rope_shift(kq, ks, cos_t, sin_t, fp16_intermediate=False)
    out_t = scb.triton_fused_k_dequant_rope_shift(kq.to(DEV), ks.to(DEV), delta_p=dps)
    torch.cuda.synchronize()
    torch.testing.assert_close(out_t.cpu(), ref_t, rtol=1e-2, atol=1e-2)


def test_rope_table_kernel(scb, oracle, golden):
    dps = torch.from_numpy(golden["tab_dps"])
    for d in (64, 128):
        for theta in (10000.0, 500000.0, 1000000.0):
            key = f"tab_d{d}_th{int(theta)}"
            c, s = scb.compute_rope_cos_sin_delta(dps, d, theta, device=DEV)
            torch.cuda.synchronize()
            for got, want in ((c.cpu(), as_tensor(golden[key + "_cos"])),
                              (s.cpu(), as_tensor(golden[key + "_sin"]))):
                diff = (got.float() - want.float()).abs()
                assert diff.max().item() <= 2 ** -10, key  # at most one fp16 ulp near 1
                assert (diff == 0).float().mean().item() > 0.99, key
    c32, _ = scb.compute_rope_cos_sin_delta(torch.arange(-5, 5), 128, device=DEV, dtype=torch.float32)
    ref32 = torch.cos(torch.arange(-5, 5, dtype=torch.float32)[:, None] * oracle.inv_freq(128)[None])
    torch.testing.assert_close(c32.cpu(), ref32, rtol=0, atol=2e-7)


def test_value_and_bf16_outputs(scb, oracle):
    t, h, d = 333, 8, 128
    kq, ks = _quantized(oracle, t, h, d, 3)
    vq, vs = _quantized(oracle, t, h, d, 4)
    cos, sin = oracle.compute_rope_cos_sin_delta(555, d, 500000.0)
    k, v = scb.dequant_kv_cache(kq.to(DEV), ks.to(DEV), vq.to(DEV), vs.to(DEV), cos.to(DEV),
                                sin.to(DEV), out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert k.dtype == torch.bfloat16 and v.dtype == torch.bfloat16
    assert bits_equal(k.cpu(), oracle.dequant_rope_shift(kq, ks, cos, sin, torch.bfloat16,
                                                         fp16_intermediate=False))
    assert bits_equal(v.cpu(), oracle.dequant_value(vq, vs, torch.bfloat16))
    v16 = scb.dequant_value(vq.to(DEV), vs.to(DEV))
    torch.cuda.synchronize()
    assert bits_equal(v16.cpu(), oracle.dequant_value(vq, vs))


def test_fp32_intermediate_mode(scb, oracle):
    t, h, d = 64, 8, 128
    kq, ks = _quantized(oracle, t, h, d, 5)
    cos, sin = oracle.compute_rope_cos_sin_delta(900, d)
    ref = oracle.dequant_rope_shift(kq, ks, cos, sin, fp16_intermediate=False)
    out = scb.triton_fused_k_dequant_rope_shift(kq.to(DEV), ks.to(DEV), cos.to(DEV), sin.to(DEV),
                                                fp32_intermediate=True)
    torch.cuda.synchronize()
    torch.testing.assert_close(out.cpu(), ref, rtol=1e-3, atol=1e-3)
    assert bits_equal(out.cpu(), ref)  # products and sum rounded as torch rounds them
    # bf16 outputs and float32 scales (an extension the reference's wrappers do not take,
    # reached through the launcher under them), same arithmetic
    from importlib import import_module

    launch = import_module("intelligent-bell_b200.kernels.restore")._launch
    ks32 = ks.to(torch.float32)
    ref32 = oracle.dequant_rope_shift(kq, ks32, cos, sin, torch.bfloat16, fp16_intermediate=False)
    out32 = torch.empty((t, h, d), dtype=torch.bfloat16, device=DEV)
    launch(1, t, h, d, kq.to(DEV), ks32.to(DEV), None, None, cos.to(DEV), sin.to(DEV), 0.0, None,
           1e4, out32, None, True)
    torch.cuda.synchronize()
    assert bits_equal(out32.cpu(), ref32)


def test_preallocated_out_is_written_in_place(scb, oracle):
    # reference tests/test_correctness.py:238-256
    t, h, d = 64, 8, 128
    kq, ks = _quantized(oracle, t, h, d, 42)
    cos, sin = oracle.compute_rope_cos_sin_delta(12, d)
    pre = torch.empty((t, h, d), dtype=torch.float16, device=DEV)
    ret = scb.triton_fused_k_dequant_rope_shift(kq.to(DEV), ks.to(DEV), cos.to(DEV), sin.to(DEV),
                                                out=pre)
    assert ret.data_ptr() == pre.data_ptr()
    torch.cuda.synchronize()
    assert bits_equal(ret.cpu(), oracle.dequant_rope_shift(kq, ks, cos, sin, fp16_intermediate=False))


@pytest.mark.parametrize("force_generic", [False, True])
def test_strided_views_and_multi_layer(scb, oracle, force_generic):
    n_l, t, h, d, dp, theta = 3, 77, 4, 128, 321, 500000.0
    codes = [_quantized(oracle, t, h, d, 100 + i) for i in range(2 * n_l)]
    kq = torch.stack([c[0] for c in codes[:n_l]])
    ks = torch.stack([c[1] for c in codes[:n_l]])
    vq = torch.stack([c[0] for c in codes[n_l:]])
    vs = torch.stack([c[1] for c in codes[n_l:]])
    # outputs written straight into model-layout caches [L, 1, H, Tmax, D]
    t_max = 96
    k_cache = torch.zeros((n_l, 1, h, t_max, d), dtype=torch.bfloat16, device=DEV)
    v_cache = torch.zeros_like(k_cache)
    k_view = k_cache[:, 0, :, :t, :].permute(0, 2, 1, 3)
    v_view = v_cache[:, 0, :, :t, :].permute(0, 2, 1, 3)
    scb.restore_layers(kq.to(DEV), ks.to(DEV), vq.to(DEV), vs.to(DEV), delta_p=dp, theta=theta,
                       k_out=k_view, v_out=v_view, force_generic=force_generic)
    torch.cuda.synchronize()
    cos, sin = oracle.compute_rope_cos_sin_delta(dp, d, theta)
    for layer in range(n_l):
        k_ref = oracle.dequant_rope_shift(kq[layer], ks[layer], cos, sin, torch.bfloat16)
        v_ref = oracle.dequant_value(vq[layer], vs[layer], torch.bfloat16)
        torch.testing.assert_close(k_cache[layer, 0, :, :t].permute(1, 0, 2).cpu().float(),
                                   k_ref.float(), rtol=1e-2, atol=1e-2)
        assert bits_equal(v_cache[layer, 0, :, :t].permute(1, 0, 2).contiguous().cpu(), v_ref)
    assert k_cache[:, :, :, t:].abs().sum().item() == 0  # nothing written past T


def test_generic_path_odd_strides(scb, oracle):
    # a dim stride of 2 (every other byte of a wider buffer) forces the generic kernel;
    # head_dim 96 with head-major storage goes through the vector path with 3 slices/row
    t, h, d = 19, 3, 96
    kq, ks = _quantized(oracle, t, h, d, 9)
    vq, vs = _quantized(oracle, t, h, d, 10)
    wide = torch.zeros((t, h, 2 * d), dtype=torch.int8)
    wide[..., ::2] = kq
    kq_strided = wide.to(DEV)[..., ::2]
    kq_hm = kq.permute(1, 0, 2).contiguous().to(DEV).permute(1, 0, 2)
    cos, sin = oracle.compute_rope_cos_sin_delta(-99, d)
    k_ref = oracle.dequant_rope_shift(kq, ks, cos, sin)
    k_ref32 = oracle.dequant_rope_shift(kq, ks, cos, sin, fp16_intermediate=False)
    for k_in in (kq_strided, kq_hm):
        for fp32 in (False, True):
            k, v = scb.dequant_kv_cache(k_in, ks.to(DEV), vq.to(DEV), vs.to(DEV), cos.to(DEV),
                                        sin.to(DEV), fp32_intermediate=fp32)
            torch.cuda.synchronize()
            assert bits_equal(k.cpu(), k_ref32 if fp32 else k_ref)
            assert bits_equal(v.cpu(), oracle.dequant_value(vq, vs))
    # odd head_dim is rejected like the reference; head_dim 34 (even, not a multiple of 32)
    # runs on the generic kernel
    kq34, ks34 = _quantized(oracle, 5, 2, 34, 12)
    c34, s34 = oracle.compute_rope_cos_sin_delta(7, 34)
    k34 = scb.triton_fused_k_dequant_rope_shift(kq34.to(DEV), ks34.to(DEV), c34.to(DEV), s34.to(DEV))
    e34 = scb.pytorch_eager_dequant_rope_shift(kq34.to(DEV), ks34.to(DEV), c34.to(DEV), s34.to(DEV))
    torch.cuda.synchronize()
    assert bits_equal(k34.cpu(), oracle.dequant_rope_shift(kq34, ks34, c34, s34,
                                                           fp16_intermediate=False))
    assert bits_equal(e34.cpu(), oracle.dequant_rope_shift(kq34, ks34, c34, s34))


@pytest.mark.parametrize("fp32", [False, True])
def test_zero_shift_is_plain_dequant(scb, oracle, fp32):
    # reference tests/test_correctness.py:91-106: a shift of 0 equals the plain dequant (here
    # bit for bit: cos 1 and sin 0 are exact, so the rotation returns x unchanged), through the
    # tables and through the shift expanded in the kernel
    t, h, d = 16, 4, 64
    kq, ks = _quantized(oracle, t, h, d, 61)
    direct = oracle.dequant_value(kq, ks)
    cos, sin = scb.compute_rope_cos_sin_delta(torch.tensor([0]), d, device=DEV)
    torch.cuda.synchronize()
    assert torch.equal(cos.cpu(), torch.ones_like(cos.cpu())) and torch.equal(sin.cpu(), torch.zeros_like(sin.cpu()))
    a = scb.triton_fused_k_dequant_rope_shift(kq.to(DEV), ks.to(DEV), cos, sin, fp32_intermediate=fp32)
    b = scb.triton_fused_k_dequant_rope_shift(kq.to(DEV), ks.to(DEV), delta_p=0, fp32_intermediate=fp32)
    torch.cuda.synchronize()
    assert bits_equal(a.cpu(), direct) and bits_equal(b.cpu(), direct)


def test_rotational_composition(scb, oracle):
    # reference tests/test_correctness.py:109-140: R(15 + 27) == R(27) R(15), the second
    # rotation by the key-shift kernel on the first one's fp16 output (reference tolerance 1e-3)
    t, h, d = 8, 2, 64
    kq, ks = _quantized(oracle, t, h, d, 62)
    direct = scb.pytorch_eager_dequant_rope_shift(kq.to(DEV), ks.to(DEV), delta_p=42)
    step1 = scb.pytorch_eager_dequant_rope_shift(kq.to(DEV), ks.to(DEV), delta_p=15)
    composed = scb.rope_shift_keys(step1, 27)
    torch.cuda.synchronize()
    torch.testing.assert_close(composed.cpu(), direct.cpu(), rtol=1e-3, atol=1e-3)


def test_end_to_end_rotational_equivalence(scb, oracle):
    # reference tests/test_correctness.py:172-235 with the quantize twin on the GPU
    g = torch.Generator().manual_seed(999)
    t, h, d = 256, 8, 128
    raw = torch.randn((t, h, d), generator=g).to(torch.float16)
    c600, s600 = oracle.compute_rope_cos_sin_delta(600, d)
    c250, s250 = oracle.compute_rope_cos_sin_delta(250, d)

    def rot(x, c, s):
        cf = torch.cat([c, c], -1)[:, None, :].float()
        sf = torch.cat([s, s], -1)[:, None, :].float()
        xf = x.float()
        return (xf * cf + oracle.rotate_half(xf) * sf).to(torch.float16)

    kq, ks = scb.quantize_kv_int8(rot(raw, c600, s600).to(DEV))
    shifted = scb.triton_fused_k_dequant_rope_shift(kq, ks, delta_p=-350)
    q250, s250_ = oracle.quantize_kv_int8(rot(raw, c250, s250))
    direct = oracle.dequant_value(q250, s250_)
    torch.cuda.synchronize()
    torch.testing.assert_close(shifted.cpu(), direct, rtol=5e-2, atol=5e-2)
    sim = torch.nn.functional.cosine_similarity(shifted.cpu().float().view(-1, d),
                                                direct.float().view(-1, d), dim=-1)
    assert sim.min().item() > 0.99


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape", [(1, 1, 128), (17, 4, 64), (513, 8, 128), (33, 2, 32), (5, 3, 96)])
def test_quantize_bit_exact(scb, oracle, dtype, shape):
    g = torch.Generator().manual_seed(sum(shape))
    x = torch.randn(shape, generator=g, dtype=torch.float32)
    x[..., : max(1, shape[-1] // 50)] *= 10.0  # outlier channels
    x[0, 0] = 0.0  # all-zero row -> eps scale
    x = x.to(dtype)
    q, s = scb.quantize_kv_int8(x.to(DEV))
    q_ref, s_ref = oracle.quantize_kv_int8(x)
    torch.cuda.synchronize()
    assert torch.equal(q.cpu(), q_ref)
    assert bits_equal(s.cpu(), s_ref)


def test_quantize_golden_and_strided(scb, oracle, golden):
    for name in golden["q_cases"]:
        name = str(name)
        x = as_tensor(golden[f"q_{name}_x"], str(golden[f"q_{name}_xdtype"]))
        q, s = scb.quantize_kv_int8(x.to(DEV))
        torch.cuda.synchronize()
        assert torch.equal(q.cpu(), as_tensor(golden[f"q_{name}_q"])), name
        assert bits_equal(s.cpu(), as_tensor(golden[f"q_{name}_s"])), name
    # head-major (non-contiguous) input: strided rows on the vector kernel
    x = torch.randn((40, 6, 128), generator=torch.Generator().manual_seed(2)).to(torch.float16)
    xs = x.permute(1, 0, 2).contiguous().to(DEV).permute(1, 0, 2)
    q, s = scb.quantize_kv_int8(xs)
    q_ref, s_ref = oracle.quantize_kv_int8(x)
    torch.cuda.synchronize()
    assert torch.equal(q.cpu(), q_ref) and bits_equal(s.cpu(), s_ref)


def _paged_case(oracle, n_req, page, h, d, seed, max_len):
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(1, max_len + 1, (n_req,), generator=g).tolist()
    lens[0] = max_len  # one request fills its pages exactly when max_len % page == 0
    pages_per = [(n + page - 1) // page for n in lens]
    n_pool = sum(pages_per) + 3
    pool_kq = torch.randint(-127, 128, (n_pool, page, h, d), generator=g, dtype=torch.int8)
    pool_vq = torch.randint(-127, 128, (n_pool, page, h, d), generator=g, dtype=torch.int8)
    pool_ks = (torch.rand((n_pool, page, h, 1), generator=g) * 0.05 + 1e-3).to(torch.float16)
    pool_vs = (torch.rand((n_pool, page, h, 1), generator=g) * 0.05 + 1e-3).to(torch.float16)
    perm = torch.randperm(n_pool, generator=g)
    max_pages = max(pages_per)
    table = torch.zeros((n_req, max_pages), dtype=torch.int32)
    k = 0
    for r, n in enumerate(pages_per):
        table[r, :n] = perm[k:k + n].to(torch.int32)
        k += n
    dps = torch.randint(0, 4097, (n_req,), generator=g).tolist()
    return pool_kq, pool_ks, pool_vq, pool_vs, table, lens, dps


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.bfloat16])
def test_paged_ragged_restore(scb, oracle, out_dtype):
    pkq, pks, pvq, pvs, table, lens, dps = _paged_case(oracle, 9, 64, 8, 128, 1, 700)
    theta = 500000.0
    k, v, cu = scb.restore_paged(pkq.to(DEV), pks.to(DEV), pvq.to(DEV), pvs.to(DEV), table, lens,
                                 dps, theta=theta, out_dtype=out_dtype)
    torch.cuda.synchronize()
    assert scb.paged_status(DEV) == 0
    ref = oracle.restore_paged(pkq, pks, pvq, pvs, table, lens, dps, theta, out_dtype=out_dtype)
    for r, (kr, vr) in enumerate(ref):
        kg = k[cu[r]:cu[r + 1]].cpu()
        vg = v[cu[r]:cu[r + 1]].cpu()
        torch.testing.assert_close(kg.float(), kr.float(), rtol=1e-2, atol=1e-2)
        assert bits_equal(vg, vr)


@pytest.mark.parametrize("case", ["empty_requests", "single_token", "head_dim_96", "odd_rows",
                                  "head_dim_256", "k_only", "v_only"])
def test_paged_edge_cases(scb, oracle, case):
    # requests of length 0 between others, one-token requests, rounds that do not divide a
    # page (head_dim 96: 42 rows per round), page * heads odd, head_dim 256, K or V alone
    h, d, page = {"head_dim_96": (3, 96, 16), "odd_rows": (3, 64, 5), "head_dim_256": (2, 256, 32)}.get(
        case, (4, 64, 16))
    pkq, pks, pvq, pvs, table, lens, dps = _paged_case(oracle, 6, page, h, d, 17, 60)
    if case == "empty_requests":
        lens[1] = lens[3] = lens[5] = 0
    if case == "single_token":
        lens = [1] * len(lens)
    pools = [pkq, pks, pvq, pvs]
    if case == "k_only":
        pools = [pkq, pks, None, None]
    if case == "v_only":
        pools = [None, None, pvq, pvs]
    k, v, cu = scb.restore_paged(*[x.to(DEV) if x is not None else None for x in pools], table,
                                 lens, dps, out_dtype=torch.float16)
    torch.cuda.synchronize()
    assert scb.paged_status(DEV) == 0
    ref = oracle.restore_paged(pkq, pks, pvq, pvs, table, lens, dps)
    for r, (kr, vr) in enumerate(ref):
        if k is not None:
            torch.testing.assert_close(k[cu[r]:cu[r + 1]].cpu(), kr, rtol=1e-2, atol=1e-2)
        if v is not None:
            assert bits_equal(v[cu[r]:cu[r + 1]].cpu(), vr)


def test_paged_many_requests(scb, oracle):
    # 1100 requests, a third of them empty
    pkq, pks, pvq, pvs, table, lens, dps = _paged_case(oracle, 1100, 8, 2, 64, 29, 30)
    g = torch.Generator().manual_seed(5)
    for r in torch.randperm(1100, generator=g)[:300].tolist():
        lens[r] = 0
    k, v, cu = scb.restore_paged(pkq.to(DEV), pks.to(DEV), pvq.to(DEV), pvs.to(DEV), table, lens,
                                 dps, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert scb.paged_status(DEV) == 0
    ref = oracle.restore_paged(pkq, pks, pvq, pvs, table, lens, dps, out_dtype=torch.bfloat16)
    for r in range(0, 1100, 7):
        torch.testing.assert_close(k[cu[r]:cu[r + 1]].cpu().float(), ref[r][0].float(),
                                   rtol=1e-2, atol=1e-2)
        assert bits_equal(v[cu[r]:cu[r + 1]].cpu(), ref[r][1])


def test_paged_per_page_shifts_bitwise_with_tables(scb, oracle):
    # per-page shifts (the pipeline's mode); compare against per-block oracle restore
    pkq, pks, pvq, pvs, table, lens, _ = _paged_case(oracle, 1, 16, 4, 64, 2, 16 * 7)
    n = (lens[0] + 15) // 16
    dps = [int(x) for x in torch.randint(-2000, 2000, (n,), generator=torch.Generator().manual_seed(3))]
    k, v, cu = scb.restore_paged(pkq.to(DEV), pks.to(DEV), pvq.to(DEV), pvs.to(DEV), table, lens,
                                 torch.tensor(dps, dtype=torch.float32).view(1, -1),
                                 delta_p_per_page=True, out_dtype=torch.float16)
    torch.cuda.synchronize()
    kr, vr = oracle.restore_blocks(pkq, pks, pvq, pvs, table[0, :n].tolist(), dps)
    torch.testing.assert_close(k.cpu(), kr[: lens[0]], rtol=1e-2, atol=1e-2)
    assert bits_equal(v.cpu(), vr[: lens[0]])


def test_paged_bad_entries_are_flagged_not_faulted(scb, oracle):
    pkq, pks, pvq, pvs, table, lens, dps = _paged_case(oracle, 3, 16, 2, 64, 4, 40)
    bad = table.clone()
    bad[1, 0] = 10_000  # page id outside the pool
    k, v, cu = scb.restore_paged(pkq.to(DEV), pks.to(DEV), pvq.to(DEV), pvs.to(DEV), bad, lens, dps,
                                 out_dtype=torch.float16)
    torch.cuda.synchronize()
    assert scb.paged_status(DEV) & scb._lib.SC_STATUS_BAD_PAGE_ID
    # the good requests are restored all the same
    ref = oracle.restore_paged(pkq, pks, pvq, pvs, table, lens, dps)
    assert bits_equal(v[cu[0]:cu[1]].cpu(), ref[0][1])
    assert bits_equal(v[cu[2]:cu[3]].cpu(), ref[2][1])
    # device-side lengths beyond the table, and offsets outside the output
    lens_dev = torch.tensor([lens[0], 16 * table.shape[1] + 1, lens[2]], dtype=torch.int32, device=DEV)
    out = torch.zeros((sum(lens) + 64, 2, 64), dtype=torch.float16, device=DEV)
    offs = torch.tensor([0, 0, 10**9], dtype=torch.int64)
    scb.restore_paged(pkq.to(DEV), pks.to(DEV), pvq.to(DEV), pvs.to(DEV), table, lens_dev, dps,
                      k_out=out, v_out=out.clone(), out_offsets=offs)
    torch.cuda.synchronize()
    bits = scb.paged_status(DEV)
    assert bits & scb._lib.SC_STATUS_BAD_SEQ_LEN and bits & scb._lib.SC_STATUS_BAD_OUT_OFFSET
    assert scb.paged_status(DEV) == 0  # reading cleared it


def test_pipeline_restore_into_one_tensor_per_side(scb, oracle):
    # outputs given as one [L, T, H, D] tensor per side instead of a list of layer views
    from speccache_b200.cache import KVRestorePipeline

    n_l, n_blocks, chunk, h, d = 4, 8, 32, 2, 128
    g = torch.Generator().manual_seed(31)
    with KVRestorePipeline(n_l, n_blocks, chunk, h, d, device=DEV) as pipe:
        pipe.k_quant.copy_(torch.randint(-127, 128, pipe.k_quant.shape, generator=g, dtype=torch.int8))
        pipe.v_quant.copy_(torch.randint(-127, 128, pipe.v_quant.shape, generator=g, dtype=torch.int8))
        pipe.k_scale.fill_(0.01)
        pipe.v_scale.fill_(0.02)
        blocks, dps = [6, 7, 1], [5, 5, -40]
        k4 = torch.empty((n_l, 3 * chunk, h, d), dtype=torch.bfloat16, device=DEV)
        v4 = torch.empty_like(k4)
        pipe.restore(blocks, dps, k4, v4)
        k_l = [torch.empty((3 * chunk, h, d), dtype=torch.bfloat16, device=DEV) for _ in range(n_l)]
        v_l = [torch.empty_like(x) for x in k_l]
        pipe.restore(blocks, dps, k_l, v_l)
        pipe.synchronize(timeout=30.0)
        for layer in range(n_l):
            assert bits_equal(k4[layer].cpu(), k_l[layer].cpu())
            assert bits_equal(v4[layer].cpu(), v_l[layer].cpu())
        with pytest.raises(ValueError, match="sharing one layout"):
            pipe.restore(blocks, dps, k4[:, :-1], v4[:, :-1])
        with pytest.raises(ValueError, match="sharing one layout"):
            pipe.restore(blocks, dps, k_l[:-1], v_l[:-1])


def test_pipeline_restore_matches_oracle(scb, oracle):
    from speccache_b200.cache import KVRestorePipeline

    n_l, n_blocks, chunk, h, d, theta = 3, 12, 32, 4, 128, 500000.0
    g = torch.Generator().manual_seed(8)
    with KVRestorePipeline(n_l, n_blocks, chunk, h, d, device=DEV, max_restore_blocks=8,
                           n_slots=2) as pipe:
        pipe.k_quant.copy_(torch.randint(-127, 128, pipe.k_quant.shape, generator=g, dtype=torch.int8))
        pipe.v_quant.copy_(torch.randint(-127, 128, pipe.v_quant.shape, generator=g, dtype=torch.int8))
        pipe.k_scale.copy_((torch.rand(pipe.k_scale.shape, generator=g) * 0.05 + 1e-3).half())
        pipe.v_scale.copy_((torch.rand(pipe.v_scale.shape, generator=g) * 0.05 + 1e-3).half())
        for blocks, dps in (([3, 4, 5, 0, 11, 7], [-256] * 6), ([9, 2, 10, 1], [100, -7, 4000, 0])):
            n_tok = len(blocks) * chunk
            k_out = [torch.empty((n_tok, h, d), dtype=torch.float16, device=DEV) for _ in range(n_l)]
            v_out = [torch.empty_like(x) for x in k_out]
            pipe.restore(blocks, dps, k_out, v_out, theta=theta)
            pipe.synchronize(timeout=30.0)
            assert pipe.status() == 0
            for layer in range(n_l):
                kr, vr = oracle.restore_blocks(pipe.k_quant[layer], pipe.k_scale[layer],
                                               pipe.v_quant[layer], pipe.v_scale[layer], blocks,
                                               dps, theta)
                torch.testing.assert_close(k_out[layer].cpu(), kr, rtol=1e-2, atol=1e-2)
                assert bits_equal(v_out[layer].cpu(), vr)


@pytest.mark.parametrize("per_layer", [False, True])
def test_pipeline_back_to_back_restores_reuse_slots(scb, oracle, per_layer):
    from speccache_b200.cache import KVRestorePipeline

    n_l, n_blocks, chunk, h, d = 5, 6, 64, 8, 128
    g = torch.Generator().manual_seed(12)
    with KVRestorePipeline(n_l, n_blocks, chunk, h, d, device=DEV, n_slots=2,
                           per_layer=per_layer) as pipe:
        pipe.k_quant.copy_(torch.randint(-127, 128, pipe.k_quant.shape, generator=g, dtype=torch.int8))
        pipe.v_quant.copy_(torch.randint(-127, 128, pipe.v_quant.shape, generator=g, dtype=torch.int8))
        pipe.k_scale.fill_(0.01)
        pipe.v_scale.fill_(0.02)
        outs = []
        for rep in range(4):  # enqueue four restores without waiting in between
            blocks = [(rep + i) % n_blocks for i in range(n_blocks)]
            k_out = [torch.empty((n_blocks * chunk, h, d), dtype=torch.bfloat16, device=DEV)
                     for _ in range(n_l)]
            v_out = [torch.empty_like(x) for x in k_out]
            pipe.restore(blocks, [rep * 10] * n_blocks, k_out, v_out)
            outs.append((blocks, rep * 10, k_out, v_out))
        pipe.synchronize(timeout=30.0)
        for blocks, dp, k_out, v_out in outs:
            for layer in range(n_l):
                kr, vr = oracle.restore_blocks(pipe.k_quant[layer], pipe.k_scale[layer],
                                               pipe.v_quant[layer], pipe.v_scale[layer], blocks,
                                               [dp] * len(blocks), out_dtype=torch.bfloat16)
                torch.testing.assert_close(k_out[layer].cpu().float(), kr.float(), rtol=1e-2, atol=1e-2)
                assert bits_equal(v_out[layer].cpu(), vr)


def test_validation_on_device(scb):
    k = torch.zeros((4, 2, 64), dtype=torch.int8, device=DEV)
    s = torch.ones((4, 2, 1), dtype=torch.float16, device=DEV)
    with pytest.raises(ValueError, match="k_scale must have shape"):
        scb.triton_fused_k_dequant_rope_shift(k, s[:3], delta_p=1)
    with pytest.raises(TypeError, match="out tensor must be torch.float16"):
        scb.triton_fused_k_dequant_rope_shift(k, s, delta_p=1,
                                              out=torch.empty((4, 2, 64), device=DEV))
    with pytest.raises(ValueError, match="must have shape"):
        scb.dequant_value(k, s, out=torch.empty((4, 2, 63), dtype=torch.float16, device=DEV))


@pytest.mark.parametrize("rows", [4096, 65536])
def test_quantize_ties_and_near_ties_bit_exact(scb, oracle, rows):
    # Rows whose scale is an exact fp16 value s (one element is 127*s) and whose other
    # elements are (k + 0.5) * s exactly, or one float32 ulp either side: the quotients land
    # on or next to half-integers, where the kernel must fall back to the IEEE division.
    g = torch.Generator().manual_seed(rows)
    d = 128
    s16 = (torch.rand((rows, 1), generator=g) * 0.999 + 0.001).to(torch.float16).to(torch.float32)
    k = torch.randint(-127, 127, (rows, d), generator=g).to(torch.float32)
    x = (k + 0.5) * s16
    which = torch.randint(0, 3, (rows, d), generator=g)
    x = torch.where(which == 1, torch.nextafter(x, torch.full_like(x, float("inf"))), x)
    x = torch.where(which == 2, torch.nextafter(x, torch.full_like(x, float("-inf"))), x)
    x[:, 0] = 127.0 * s16[:, 0]
    x = x.view(rows // 4, 4, d)
    q, s = scb.quantize_kv_int8(x.to(DEV))
    q_ref, s_ref = oracle.quantize_kv_int8(x)
    torch.cuda.synchronize()
    assert bits_equal(s.cpu(), s_ref)
    assert torch.equal(q.cpu(), q_ref)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_quantize_exact_ties_16bit_inputs(scb, oracle, dtype):
    # 16-bit inputs with fp16 scales take the two-product rule (no tie test).  Rows whose
    # scale is s = m * 2^e (m odd, few bits, so (2k + 1) * m fits the input's significand)
    # with one element 127 * s and the others (k + 1/2) * s or k * s: every half-integer
    # quotient is exact and must round half to even, in both directions of the
    # reciprocal's rounding error (m = 1: exact reciprocal; m = 3, 5, 7: inexact).
    g = torch.Generator().manual_seed(5)
    rows, d = 8192, 128
    ms = torch.tensor([1.0, 3.0, 5.0, 7.0] if dtype == torch.float16 else [1.0])
    m = ms[torch.randint(0, ms.numel(), (rows, 1), generator=g)]
    e = torch.randint(-12, -1, (rows, 1), generator=g).to(torch.float32)
    s = m * torch.pow(2.0, e)
    k = torch.randint(-127, 127, (rows, d), generator=g).to(torch.float32)
    half = torch.randint(0, 4, (rows, d), generator=g) > 0
    x = torch.where(half, (k + 0.5) * s, k * s)
    x[:, 0] = 127.0 * s[:, 0] * torch.where(torch.rand(rows, generator=g) < 0.5, -1.0, 1.0)
    x16 = x.to(dtype)
    assert torch.equal(x16.to(torch.float32), x)  # every element exactly representable
    x16 = x16.view(rows // 8, 8, d)
    q, sc = scb.quantize_kv_int8(x16.to(DEV))
    q_ref, s_ref = oracle.quantize_kv_int8(x16)
    torch.cuda.synchronize()
    assert bits_equal(sc.cpu(), s_ref)
    assert torch.equal(sc.cpu().to(torch.float32).view(rows, 1), s)
    assert torch.equal(q.cpu(), q_ref)


def test_fp32_scales_dense_and_quantize(scb, oracle):
    # float32 scales (an extension): x = fp16(fp32(q * s)) exactly as the reference's
    # arithmetic would do with float32 scales; quantize with float32 scale output skips the
    # fp16 rounding of the scale.
    t, h, d = 50, 4, 128
    g = torch.Generator().manual_seed(21)
    kq = torch.randint(-127, 128, (t, h, d), generator=g, dtype=torch.int8)
    ks32 = torch.rand((t, h, 1), generator=g) * 0.05 + 1e-4
    vq = torch.randint(-127, 128, (t, h, d), generator=g, dtype=torch.int8)
    vs32 = torch.rand((t, h, 1), generator=g) * 0.05 + 1e-4
    cos, sin = oracle.compute_rope_cos_sin_delta(77, d)
    # the reference-named wrappers keep its fp16-scale contract; restore_layers takes both
    k = scb.restore_layers(kq[None].to(DEV), ks32[None].to(DEV), vq[None].to(DEV), vs32[None].to(DEV),
                           delta_p=77, out_dtype=torch.float16)
    torch.cuda.synchronize()
    k_ref = oracle.dequant_rope_shift(kq, ks32, cos, sin)
    torch.testing.assert_close(k[0][0].cpu(), k_ref, rtol=1e-2, atol=1e-2)
    assert bits_equal(k[1][0].cpu(), oracle.dequant_value(vq, vs32))
    x = torch.randn((t, h, d), generator=g)
    q, s = scb.quantize_kv_int8(x.to(DEV), scale_dtype=torch.float32)
    torch.cuda.synchronize()
    s_ref = torch.clamp(x.abs().amax(-1, keepdim=True) / 127.0, min=1e-5)
    q_ref = torch.clamp(torch.round(x / s_ref), -127, 127).to(torch.int8)
    assert s.dtype == torch.float32 and bits_equal(s.cpu(), s_ref)
    assert torch.equal(q.cpu(), q_ref)
    # eps = 0 with float32 scales: rows of subnormal values get subnormal scales (whose
    # reciprocal overflows float32), handled by the exact division
    xs = torch.randn((t, h, d), generator=g) * 1e-39
    xs[3, 1] = 0.0
    q, s = scb.quantize_kv_int8(xs.to(DEV), eps=0.0, scale_dtype=torch.float32)
    torch.cuda.synchronize()
    s_ref = torch.clamp(xs.abs().amax(-1, keepdim=True) / 127.0, min=0.0)
    with torch.no_grad():
        q_ref = torch.clamp(torch.round(xs / s_ref), -127, 127).nan_to_num(0.0).to(torch.int8)
    assert bits_equal(s.cpu(), s_ref)
    nz = s_ref.expand_as(xs) != 0  # the all-zero row divides 0 by 0 (outside the contract)
    assert torch.equal(q.cpu()[nz], q_ref[nz])


def test_paged_fp32_intermediate_and_fp16(scb, oracle):
    pkq, pks, pvq, pvs, table, lens, dps = _paged_case(oracle, 5, 32, 4, 64, 31, 150)
    cos_ref = [oracle.compute_rope_cos_sin_delta(dp, 64) for dp in dps]
    k, v, cu = scb.restore_paged(pkq.to(DEV), pks.to(DEV), pvq.to(DEV), pvs.to(DEV), table, lens,
                                 dps, out_dtype=torch.float16, fp32_intermediate=True)
    torch.cuda.synchronize()
    for r in range(len(lens)):
        n = (lens[r] + 31) // 32
        ids = table[r, :n].tolist()
        kq = oracle.gather_blocks(pkq, ids)[: lens[r]]
        ks = oracle.gather_blocks(pks, ids)[: lens[r]]
        ref = oracle.dequant_rope_shift(kq, ks, *cos_ref[r], fp16_intermediate=False)
        torch.testing.assert_close(k[cu[r]:cu[r + 1]].cpu(), ref, rtol=1e-2, atol=1e-2)


def test_empty_inputs_are_no_ops(scb):
    k = torch.zeros((0, 8, 128), dtype=torch.int8, device=DEV)
    s = torch.zeros((0, 8, 1), dtype=torch.float16, device=DEV)
    out = scb.triton_fused_k_dequant_rope_shift(k, s, delta_p=5)
    v = scb.dequant_value(k, s)
    q, sc = scb.quantize_kv_int8(torch.zeros((0, 8, 128), device=DEV))
    torch.cuda.synchronize()
    assert out.shape == (0, 8, 128) and v.shape == (0, 8, 128) and q.shape == (0, 8, 128)
    kp, vp, cu = scb.restore_paged(torch.zeros((2, 16, 2, 64), dtype=torch.int8, device=DEV),
                                   torch.ones((2, 16, 2, 1), dtype=torch.float16, device=DEV),
                                   None, None, torch.zeros((3, 2), dtype=torch.int32),
                                   [0, 0, 0], [1, 2, 3])
    torch.cuda.synchronize()
    assert kp.shape == (0, 2, 64) and vp is None and cu.tolist() == [0, 0, 0, 0]


def test_concurrent_host_threads_on_separate_streams(scb, oracle):
    import threading

    t, h, d = 2048, 8, 128
    g = torch.Generator().manual_seed(33)
    cases = []
    for i in range(4):
        kq, ks = oracle.quantize_kv_int8(torch.randn((t, h, d), generator=g))
        cases.append((kq, ks, 100 * i - 150))
    results = [None] * len(cases)
    errors = []

    def work(i):
        try:
            kq, ks, dp = cases[i]
            stream = torch.cuda.Stream(device=DEV)
            with torch.cuda.stream(stream):
                kd, sd = kq.to(DEV, non_blocking=False), ks.to(DEV, non_blocking=False)
                outs = [scb.triton_fused_k_dequant_rope_shift(kd, sd, delta_p=dp + k)
                        for k in range(8)]
            stream.synchronize()
            results[i] = [o.cpu() for o in outs]
        except Exception as exc:  # pragma: no cover - reported below
            errors.append(exc)

    threads = [threading.Thread(target=work, args=(i,)) for i in range(len(cases))]
    for th in threads:
        th.start()
    for th in threads:
        th.join()
    assert not errors, errors
    for i, (kq, ks, dp) in enumerate(cases):
        for k in range(8):
            c, s = oracle.compute_rope_cos_sin_delta(dp + k, d)
            ref = oracle.dequant_rope_shift(kq, ks, c, s, fp16_intermediate=False)
            torch.testing.assert_close(results[i][k], ref, rtol=1e-2, atol=1e-2)
