"""The restore entry point for callers that cannot allocate device memory.

``sc_dequant_rope_kv_token_shifts_noalloc`` serves callers that cannot call cudaMalloc,
for example an engine that has reserved the GPU's memory for its own pools, or a request
path that must not risk the device synchronisation cudaMalloc/cudaFree can cause.  It
keeps the per-token cos/sin tables in a fixed array inside the library instead of
buffers the caller allocates.  This test calls it through the C ABI twice in a row and
checks each result against the regular path (tables built into allocated tensors, then
the fused restore), with the suite's restore tolerance (rtol = atol = 1e-2) and bit for
bit, since both paths run the same arithmetic.  It also checks that a call beyond the
fixed capacity is refused.  The file name makes pytest collect it last.
"""

from __future__ import annotations

import pytest
import torch

from conftest import bits_equal

pytestmark = pytest.mark.gpu

MAX_ENTRIES = 1 << 20  # n_tokens * head_dim / 2 the fixed tables hold


def _call_noalloc(scb, kq, ks, vq, vs, dps, theta, k_out, v_out):
    lib = scb._lib.load()
    st = scb._lib.strides
    t, h, d = kq.shape
    return lib.sc_dequant_rope_kv_token_shifts_noalloc(
        1, t, h, d,
        kq.data_ptr(), st(0, *kq.stride()), ks.data_ptr(), st(0, ks.stride(0), ks.stride(1)),
        vq.data_ptr(), st(0, *vq.stride()), vs.data_ptr(), st(0, vs.stride(0), vs.stride(1)),
        scb._lib.SC_DTYPE_F16, dps.data_ptr(), float(theta), scb._lib.inv_freq_ptr(d, theta),
        k_out.data_ptr(), st(0, *k_out.stride()), v_out.data_ptr(), st(0, *v_out.stride()),
        scb._lib.DTYPE_CODE[k_out.dtype], 0, scb._lib.stream_handle(kq.device))


def test_noalloc_matches_regular_path_two_calls(scb, oracle):
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(2024)
    for call, (t, h, d, theta, out_dtype) in enumerate(
            [(1000, 8, 128, 500000.0, torch.bfloat16), (777, 4, 64, 10000.0, torch.float16)]):
        kq, ks = oracle.quantize_kv_int8(torch.randn((t, h, d), generator=g))
        vq, vs = oracle.quantize_kv_int8(torch.randn((t, h, d), generator=g))
        kq, ks, vq, vs = kq.to(dev), ks.to(dev), vq.to(dev), vs.to(dev)
        dps = torch.randint(-8192, 8192, (t,), generator=g).to(torch.float32).to(dev)
        k_new = torch.empty((t, h, d), dtype=out_dtype, device=dev)
        v_new = torch.empty_like(k_new)
        rc = _call_noalloc(scb, kq, ks, vq, vs, dps, theta, k_new, v_new)
        assert rc == 0, scb._lib.load().sc_last_error().decode()
        k_ref, v_ref = scb.dequant_kv_cache(kq, ks, vq, vs, delta_p=dps, theta=theta,
                                            out_dtype=out_dtype)
        torch.cuda.synchronize()
        torch.testing.assert_close(k_new.float(), k_ref.float(), rtol=1e-2, atol=1e-2)
        torch.testing.assert_close(v_new.float(), v_ref.float(), rtol=1e-2, atol=1e-2)
        assert bits_equal(k_new.cpu(), k_ref.cpu()), f"call {call}: K differs"
        assert bits_equal(v_new.cpu(), v_ref.cpu()), f"call {call}: V differs"


def test_noalloc_refuses_calls_beyond_capacity(scb):
    dev = torch.device("cuda", 0)
    d = 128
    t = MAX_ENTRIES // (d // 2) + 1
    kq = torch.zeros((t, 1, d), dtype=torch.int8, device=dev)
    ks = torch.ones((t, 1, 1), dtype=torch.float16, device=dev)
    dps = torch.zeros(t, dtype=torch.float32, device=dev)
    out = torch.empty((t, 1, d), dtype=torch.float16, device=dev)
    rc = _call_noalloc(scb, kq, ks, kq, ks, dps, 10000.0, out, out.clone())
    assert rc == scb._lib.SC_ERR_INVALID_ARGUMENT
    assert "capacity" in scb._lib.load().sc_last_error().decode()
