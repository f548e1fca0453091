"""Property-based parity on random geometries, layouts, dtypes and shifts (hypothesis).

* dense restore with the reference's tables: bit-exact with the oracle for K and V, for any
  token count, head count, even head_dim (vector and generic kernels), output dtype and
  output layout (contiguous or model layout [H, T, D] viewed as [T, H, D]);
* dense restore with the shift expanded in the kernel: within the reference tolerance;
* quantize: bit-exact codes and scales for random shapes, dtypes, magnitudes and layouts;
* paged restore: V bit-exact and K within tolerance for random ragged batches, and the same
  bits whether the page table, lengths and shifts come as host lists or device tensors.
"""

from __future__ import annotations

import pytest
import torch
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

from conftest import bits_equal

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0) if torch.cuda.is_available() else None
SETTINGS = settings(max_examples=60, deadline=None, derandomize=True,
                    suppress_health_check=[HealthCheck.function_scoped_fixture])

head_dims = st.sampled_from([2, 8, 34, 64, 96, 128, 160, 256])
out_dtypes = st.sampled_from([torch.float16, torch.bfloat16])


def _codes(g, shape):
    q = torch.randint(-127, 128, shape, generator=g, dtype=torch.int8)
    s = (torch.rand(shape[:-1] + (1,), generator=g) * 0.1 + 1e-4).to(torch.float16)
    return q, s


@SETTINGS
@given(t=st.integers(1, 300), h=st.integers(1, 12), d=head_dims, dp=st.integers(-70000, 70000),
       theta=st.sampled_from([10000.0, 500000.0, 1e6]), out_dtype=out_dtypes,
       model_layout=st.booleans(), per_token=st.booleans(), fp32=st.booleans(),
       seed=st.integers(0, 2**31 - 1))
def test_dense_restore_matches_oracle(scb, oracle, t, h, d, dp, theta, out_dtype, model_layout,
                                      per_token, fp32, seed):
    g = torch.Generator().manual_seed(seed)
    kq, ks = _codes(g, (t, h, d))
    vq, vs = _codes(g, (t, h, d))
    dps = torch.randint(-5000, 5000, (t,), generator=g) if per_token else dp
    cos, sin = oracle.compute_rope_cos_sin_delta(dps, d, theta)
    if model_layout:
        k_buf = torch.empty((h, t + 3, d), dtype=out_dtype, device=DEV)
        v_buf = torch.empty_like(k_buf)
        k_out, v_out = k_buf[:, :t].permute(1, 0, 2), v_buf[:, :t].permute(1, 0, 2)
    else:
        k_out = torch.empty((t, h, d), dtype=out_dtype, device=DEV)
        v_out = torch.empty_like(k_out)
    scb.dequant_kv_cache(kq.to(DEV), ks.to(DEV), vq.to(DEV), vs.to(DEV), cos.to(DEV), sin.to(DEV),
                         k_out=k_out, v_out=v_out, fp32_intermediate=fp32)
    torch.cuda.synchronize()
    assert bits_equal(k_out.cpu().contiguous(),
                      oracle.dequant_rope_shift(kq, ks, cos, sin, out_dtype, fp16_intermediate=not fp32))
    assert bits_equal(v_out.cpu().contiguous(), oracle.dequant_value(vq, vs, out_dtype))


@SETTINGS
@given(t=st.integers(1, 200), h=st.integers(1, 8), d=st.sampled_from([32, 64, 128, 256]),
       dp=st.integers(-40000, 40000), theta=st.sampled_from([10000.0, 500000.0, 1e6]),
       seed=st.integers(0, 2**31 - 1))
def test_in_kernel_shift_within_tolerance(scb, oracle, t, h, d, dp, theta, seed):
    g = torch.Generator().manual_seed(seed)
    kq, ks = _codes(g, (t, h, d))
    out = scb.triton_fused_k_dequant_rope_shift(kq.to(DEV), ks.to(DEV), delta_p=dp, theta=theta)
    cos, sin = oracle.compute_rope_cos_sin_delta(dp, d, theta)
    torch.cuda.synchronize()
    torch.testing.assert_close(out.cpu(), oracle.dequant_rope_shift(kq, ks, cos, sin,
                                                                    fp16_intermediate=False),
                               rtol=1e-2, atol=1e-2)


@SETTINGS
@given(t=st.integers(1, 300), h=st.integers(1, 10), d=st.sampled_from([16, 32, 48, 64, 96, 128, 256]),
       dtype=st.sampled_from([torch.float16, torch.bfloat16, torch.float32]),
       mag=st.sampled_from([1e-4, 1e-2, 1.0, 30.0, 2000.0]), head_major=st.booleans(),
       seed=st.integers(0, 2**31 - 1))
def test_quantize_matches_oracle(scb, oracle, t, h, d, dtype, mag, head_major, seed):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn((t, h, d), generator=g) * mag).to(dtype)
    if t > 1:
        x[0] = 0  # zero rows take the eps scale
    xd = x.permute(1, 0, 2).contiguous().to(DEV).permute(1, 0, 2) if head_major else x.to(DEV)
    q, s = scb.quantize_kv_int8(xd)
    q_ref, s_ref = oracle.quantize_kv_int8(x)
    torch.cuda.synchronize()
    assert torch.equal(q.cpu(), q_ref)
    assert bits_equal(s.cpu(), s_ref)


@SETTINGS
@given(n_req=st.integers(1, 7), page=st.sampled_from([8, 16, 64]), h=st.integers(1, 8),
       d=st.sampled_from([32, 64, 128]), max_len=st.integers(1, 300), out_dtype=out_dtypes,
       seed=st.integers(0, 2**31 - 1))
def test_paged_matches_oracle(scb, oracle, n_req, page, h, d, max_len, out_dtype, seed):
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(1, max_len + 1, (n_req,), generator=g).tolist()
    pages = [(n + page - 1) // page for n in lens]
    n_pool = sum(pages) + 1
    pkq, pks = _codes(g, (n_pool, page, h, d))
    pvq, pvs = _codes(g, (n_pool, page, h, d))
    perm = torch.randperm(n_pool, generator=g)
    table = torch.zeros((n_req, max(pages)), dtype=torch.int32)
    k = 0
    for r, n in enumerate(pages):
        table[r, :n] = perm[k:k + n].to(torch.int32)
        k += n
    dps = torch.randint(-4096, 4097, (n_req,), generator=g).tolist()
    kk, vv, cu = scb.restore_paged(pkq.to(DEV), pks.to(DEV), pvq.to(DEV), pvs.to(DEV), table, lens,
                                   dps, out_dtype=out_dtype)
    torch.cuda.synchronize()
    assert scb.paged_status(DEV) == 0
    # the same call with every argument already on the device gives the same bits
    kd, vd = torch.empty_like(kk), torch.empty_like(vv)
    offs = (cu[:-1] * kk.stride(0)).to(DEV)
    scb.restore_paged(pkq.to(DEV), pks.to(DEV), pvq.to(DEV), pvs.to(DEV), table.to(DEV),
                      torch.tensor(lens, dtype=torch.int32, device=DEV),
                      torch.tensor(dps, dtype=torch.float32, device=DEV), out_dtype=out_dtype,
                      k_out=kd, v_out=vd, out_offsets=offs)
    torch.cuda.synchronize()
    assert bits_equal(kd.cpu(), kk.cpu()) and bits_equal(vd.cpu(), vv.cpu())
    ref = oracle.restore_paged(pkq, pks, pvq, pvs, table, lens, dps, out_dtype=out_dtype)
    for r, (kr, vr) in enumerate(ref):
        torch.testing.assert_close(kk[cu[r]:cu[r + 1]].cpu().float(), kr.float(), rtol=1e-2, atol=1e-2)
        assert bits_equal(vv[cu[r]:cu[r + 1]].cpu(), vr)
