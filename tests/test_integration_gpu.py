"""The ctypes binding of the C ABI that a maintainer adds to the reference's own wrappers
(``include/b200_abi.py``), imported and checked against the oracle.

The stub replaces the key kernel launch of the reference's Triton wrapper
(speccache/kernels/triton_rope_kv.py:320-343): fp16 tables ([1, D/2] broadcast or [T, D/2]
per token), fp16 output, bit-exact with the reference's torch arithmetic given the tables
(fp32 intermediate by default, the Triton kernel's; fp16 intermediate on request, the eager
function's).
"""

from __future__ import annotations

import importlib.util
import os

import pytest
import torch

from conftest import REPO, bits_equal

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0) if torch.cuda.is_available() else None


def _load_stub(scb):
    os.environ["SPECCACHE_B200_LIB"] = scb._lib.LIB_PATH
    spec = importlib.util.spec_from_file_location("b200_abi", os.path.join(REPO, "include", "b200_abi.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_ctypes_stub(scb, oracle):
    stub = _load_stub(scb).fused_k_dequant_rope_shift
    g = torch.Generator().manual_seed(77)
    t, h, d = 200, 8, 128
    kq = torch.randint(-127, 128, (t, h, d), generator=g, dtype=torch.int8)
    ks = (torch.rand((t, h, 1), generator=g) * 0.05 + 1e-3).half()
    for dps in ([-384], torch.randint(-4096, 4097, (t,), generator=g).tolist()):
        cos, sin = oracle.compute_rope_cos_sin_delta(dps, d)
        for fp32 in (True, False):
            out = torch.empty((t, h, d), dtype=torch.float16, device=DEV)
            got = stub(kq.to(DEV), ks.to(DEV), cos.to(DEV), sin.to(DEV), out, fp32_intermediate=fp32)
            torch.cuda.synchronize()
            assert got.data_ptr() == out.data_ptr()
            assert bits_equal(out.cpu(), oracle.dequant_rope_shift(kq, ks, cos, sin,
                                                                   fp16_intermediate=not fp32))
    # an argument error comes back as the library's message
    cos, sin = oracle.compute_rope_cos_sin_delta(5, 64)
    with pytest.raises(RuntimeError, match="head_dim"):
        stub(torch.zeros((4, 2, 63), dtype=torch.int8, device=DEV),
             torch.ones((4, 2, 1), dtype=torch.float16, device=DEV), cos.to(DEV), sin.to(DEV),
             torch.empty((4, 2, 63), dtype=torch.float16, device=DEV))
