"""The ctypes binding that INTEGRATION.md shows, executed as written (only the library path
substituted) and checked against the oracle, so the documented stub stays correct.

The stub replaces the key kernel launch of the reference's Triton wrapper
(speccache/kernels/triton_rope_kv.py:320-343): fp16 tables ([1, D/2] broadcast or [T, D/2]
per token), fp16 output, bit-exact with the reference's eager arithmetic given the tables.
"""

from __future__ import annotations

import os
import re

import pytest
import torch

from conftest import REPO, bits_equal

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0) if torch.cuda.is_available() else None


def _doc_block(marker: str) -> str:
    with open(os.path.join(REPO, "INTEGRATION.md")) as f:
        text = f.read()
    blocks = re.findall(r"```python\n(.*?)```", text, re.S)
    return next(b for b in blocks if marker in b)


def test_ctypes_stub_from_the_integration_guide(scb, oracle):
    code = _doc_block("speccache/kernels/b200_abi.py")
    assert "/path/to/libspeccache_b200.so" in code
    code = code.replace("/path/to/libspeccache_b200.so", scb._lib.LIB_PATH)
    ns: dict = {}
    exec(compile(code, "INTEGRATION.md (b200_abi.py)", "exec"), ns)
    stub = ns["fused_k_dequant_rope_shift"]

    g = torch.Generator().manual_seed(77)
    t, h, d = 200, 8, 128
    kq = torch.randint(-127, 128, (t, h, d), generator=g, dtype=torch.int8)
    ks = (torch.rand((t, h, 1), generator=g) * 0.05 + 1e-3).half()
    for dps in ([-384], torch.randint(-4096, 4097, (t,), generator=g).tolist()):
        cos, sin = oracle.compute_rope_cos_sin_delta(dps, d)
        out = torch.empty((t, h, d), dtype=torch.float16, device=DEV)
        got = stub(kq.to(DEV), ks.to(DEV), cos.to(DEV), sin.to(DEV), out)
        torch.cuda.synchronize()
        assert got.data_ptr() == out.data_ptr()
        assert bits_equal(out.cpu(), oracle.dequant_rope_shift(kq, ks, cos, sin))
    # an argument error comes back as the library's message
    cos, sin = oracle.compute_rope_cos_sin_delta(5, 64)
    with pytest.raises(RuntimeError, match="head_dim"):
        stub(torch.zeros((4, 2, 63), dtype=torch.int8, device=DEV),
             torch.ones((4, 2, 1), dtype=torch.float16, device=DEV), cos.to(DEV), sin.to(DEV),
             torch.empty((4, 2, 63), dtype=torch.float16, device=DEV))
