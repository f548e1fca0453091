"""The restore entry point for callers that cannot allocate device memory.

``sc_dequant_rope_kv_token_shifts_noalloc`` serves callers that cannot call cudaMalloc,
for example an engine that has reserved the GPU's memory for its own pools, or a request
path that must not risk the device synchronisation cudaMalloc/cudaFree can cause.  It
keeps the per-token cos/sin tables in a fixed array inside the library instead of
buffers the caller allocates.

This test calls it through the C ABI three times in a row, each call smaller (in
n_tokens x head_dim/2, the table entries it uses) than the one before and with a different
head_dim, so that stale table rows left by an earlier call would show if they were read.
Each call is checked two ways:

* against the oracle on the oracle's per-token tables: K within the suite's restore
  tolerance (rtol = atol = 1e-2) with at least 98 % of K bit-equal (the tables come from
  double-precision cos/sin, torch's float32 cos/sin differs from them by one fp16 ulp in
  rare entries), V bit for bit;
* against the regular entry point (``sc_dequant_rope_kv`` given tables built by
  ``sc_rope_cos_sin_delta`` into allocated buffers): bit for bit, since both run the same
  arithmetic on the same tables.

The calls cover 3-D and 4-D (two layers sharing the per-token tables) layouts, V present
or absent, fp16 and fp32 scales, both output dtypes and both arithmetics (fp16 or fp32
intermediate).  A call beyond the fixed capacity, and a call with a bad argument, are
refused.  The file name makes pytest collect it last.
"""

from __future__ import annotations

import pytest
import torch

from conftest import bits_equal

pytestmark = pytest.mark.gpu

MAX_ENTRIES = 1 << 20  # n_tokens * head_dim / 2 the fixed tables hold

# (n_layers, tokens, heads, head_dim, theta, out dtype, scale dtype, with V, fp32 intermediate)
CALLS = [
    (1, 4096, 8, 128, 500000.0, torch.bfloat16, torch.float16, True, False),  # 262,144 entries
    (2, 777, 4, 64, 10000.0, torch.float16, torch.float16, True, True),       # 24,864 entries
    (1, 150, 3, 128, 1000000.0, torch.float16, torch.float32, False, False),  # 9,600 entries
]


def _codes(oracle, g, layers, t, h, d, scale_dtype):
    qs, ss = [], []
    for _ in range(layers):
        q, s = oracle.quantize_kv_int8(torch.randn((t, h, d), generator=g))
        qs.append(q)
        ss.append(s.to(scale_dtype))
    return torch.stack(qs), torch.stack(ss)


def _st(scb, t: torch.Tensor, n: int):
    """[layer, token, head(, dim)] strides of a 4-D tensor, first n of them."""
    return scb._lib.strides(*t.stride()[:n])


def _call(scb, entry, kq, ks, vq, vs, dps, theta, k_out, v_out, fp32, tables=None):
    """One call of either entry point on [L, T, H, D] tensors (V may be None)."""
    lib = scb._lib.load()
    n_l, t, h, d = kq.shape
    flags = scb._lib.SC_FLAG_FP32_INTERMEDIATE if fp32 else 0
    v_args = ((vq.data_ptr(), _st(scb, vq, 4), vs.data_ptr(), _st(scb, vs, 3)) if vq is not None
              else (None, None, None, None))
    vo_args = (v_out.data_ptr(), _st(scb, v_out, 4)) if v_out is not None else (None, None)
    common_k = (n_l, t, h, d, kq.data_ptr(), _st(scb, kq, 4), ks.data_ptr(), _st(scb, ks, 3))
    scale_code = scb._lib.DTYPE_CODE[ks.dtype]
    stream = scb._lib.stream_handle(kq.device)
    if entry == "noalloc":
        return lib.sc_dequant_rope_kv_token_shifts_noalloc(
            *common_k, *v_args, scale_code, dps.data_ptr(), float(theta),
            scb._lib.inv_freq_ptr(d, theta), k_out.data_ptr(), _st(scb, k_out, 4), *vo_args,
            scb._lib.DTYPE_CODE[k_out.dtype], flags, stream)
    cos, sin = tables
    return lib.sc_dequant_rope_kv(
        *common_k, *v_args, scale_code, cos.data_ptr(), sin.data_ptr(),
        scb._lib.strides(cos.stride(0), cos.stride(1)), 0.0, None, float(theta), None,
        k_out.data_ptr(), _st(scb, k_out, 4), *vo_args, scb._lib.DTYPE_CODE[k_out.dtype], flags,
        stream)


def test_noalloc_three_calls_against_oracle_and_regular_path(scb, oracle):
    dev = torch.device("cuda", 0)
    lib = scb._lib.load()
    g = torch.Generator().manual_seed(2024)
    prev_entries = None
    for call, (n_l, t, h, d, theta, out_dtype, scale_dtype, with_v, fp32) in enumerate(CALLS):
        entries = t * d // 2
        assert prev_entries is None or entries < prev_entries  # each call smaller than the last
        prev_entries = entries
        kq, ks = _codes(oracle, g, n_l, t, h, d, scale_dtype)
        vq, vs = _codes(oracle, g, n_l, t, h, d, scale_dtype) if with_v else (None, None)
        dps = torch.randint(-8192, 8192, (t,), generator=g).to(torch.float32)
        kq_d, ks_d, dps_d = kq.to(dev), ks.to(dev), dps.to(dev)
        vq_d, vs_d = (vq.to(dev), vs.to(dev)) if with_v else (None, None)
        shape = (n_l, t, h, d)
        k_new = torch.empty(shape, dtype=out_dtype, device=dev)
        v_new = torch.empty(shape, dtype=out_dtype, device=dev) if with_v else None
        rc = _call(scb, "noalloc", kq_d, ks_d, vq_d, vs_d, dps_d, theta, k_new, v_new, fp32)
        assert rc == 0, lib.sc_last_error().decode()

        # the regular entry point on allocated tables
        cos_d, sin_d = scb.compute_rope_cos_sin_delta(dps_d, d, theta, device=dev)
        k_reg = torch.empty_like(k_new)
        v_reg = torch.empty_like(v_new) if with_v else None
        rc = _call(scb, "regular", kq_d, ks_d, vq_d, vs_d, dps_d, theta, k_reg, v_reg, fp32,
                   tables=(cos_d, sin_d))
        assert rc == 0, lib.sc_last_error().decode()
        torch.cuda.synchronize()
        assert bits_equal(k_new.cpu(), k_reg.cpu()), f"call {call}: K differs from the regular path"
        if with_v:
            assert bits_equal(v_new.cpu(), v_reg.cpu()), f"call {call}: V differs from the regular path"

        # the oracle on its own per-token tables
        cos, sin = oracle.compute_rope_cos_sin_delta(dps, d, theta)
        k_host = k_new.cpu()
        for layer in range(n_l):
            k_ref = oracle.dequant_rope_shift(kq[layer], ks[layer], cos, sin, out_dtype,
                                              fp16_intermediate=not fp32)
            torch.testing.assert_close(k_host[layer].float(), k_ref.float(), rtol=1e-2, atol=1e-2)
            same = (k_host[layer].view(torch.int16) == k_ref.view(torch.int16)).float().mean().item()
            assert same >= 0.98, (call, layer, same)
            if with_v:
                assert bits_equal(v_new[layer].cpu(), oracle.dequant_value(vq[layer], vs[layer], out_dtype)), \
                    (call, layer)


def test_noalloc_refuses_calls_beyond_capacity_and_bad_arguments(scb):
    dev = torch.device("cuda", 0)
    lib = scb._lib.load()
    d = 128
    t = MAX_ENTRIES // (d // 2) + 1
    kq = torch.zeros((1, t, 1, d), dtype=torch.int8, device=dev)
    ks = torch.ones((1, t, 1, 1), dtype=torch.float16, device=dev)
    dps = torch.zeros(t, dtype=torch.float32, device=dev)
    out = torch.empty((1, t, 1, d), dtype=torch.float16, device=dev)
    rc = _call(scb, "noalloc", kq, ks, None, None, dps, 10000.0, out, None, False)
    assert rc == scb._lib.SC_ERR_INVALID_ARGUMENT
    assert "capacity" in lib.sc_last_error().decode()
    # an unsupported output dtype is refused before anything is launched
    small = (slice(None), slice(0, 8))
    bad_out = torch.empty((1, 8, 1, d), dtype=torch.float32, device=dev)
    rc = _call(scb, "noalloc", kq[small], ks[small], None, None, dps[:8], 10000.0, bad_out, None, False)
    assert rc == scb._lib.SC_ERR_INVALID_DTYPE
    torch.cuda.synchronize()
