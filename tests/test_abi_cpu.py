"""The C ABI and the host-side contract, on a machine without a GPU.

* the library loads and exports every function ``include/speccache_b200.h`` declares;
* argument errors are reported before any CUDA call, with the reference's exception
  types and messages (speccache/kernels/reference.py:13-119);
* the operators refuse CPU tensors instead of falling back to a CPU path.
"""

from __future__ import annotations

import ctypes
import os
import re

import pytest
import torch

from conftest import REPO

HEADER = os.path.join(REPO, "include", "speccache_b200.h")


def declared_functions() -> list[str]:
    with open(HEADER) as f:
        text = f.read()
    return sorted(set(re.findall(r"^SC_API\s+[\w\s\*]+?\b(sc_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_abi():
    names = declared_functions()
    assert "sc_dequant_rope_kv" in names and "sc_quantize_int8" in names
    assert "sc_restore_paged" in names and "sc_pipeline_restore" in names
    assert len(names) >= 12


def test_library_exports_every_declared_symbol(scb):
    lib = scb._lib.load()
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in the header but not exported"
    assert set(declared_functions()) == set(scb._lib.exported_symbols())
    assert lib.sc_abi_version() == 1


def _err(lib) -> str:
    return lib.sc_last_error().decode()


def test_dense_rejects_bad_arguments_before_cuda(scb):
    lib = scb._lib.load()
    st = scb._lib.strides
    s4, s3 = st(0, 8 * 63, 63, 1), st(0, 8, 1)
    # odd head_dim
    rc = lib.sc_dequant_rope_kv(1, 4, 8, 63, 1, s4, 1, s3, None, None, None, None, 0,
                                None, None, None, 0.0, None, 1e4, None, 1, s4, None, None,
                                0, 0, None)
    assert rc == scb._lib.SC_ERR_INVALID_ARGUMENT and "head_dim must be even" in _err(lib)
    # bad output dtype
    s4 = st(0, 8 * 64, 64, 1)
    rc = lib.sc_dequant_rope_kv(1, 4, 8, 64, 1, s4, 1, s3, None, None, None, None, 0,
                                None, None, None, 0.0, None, 1e4, None, 1, s4, None, None,
                                2, 0, None)
    assert rc == scb._lib.SC_ERR_INVALID_DTYPE
    # neither K nor V
    rc = lib.sc_dequant_rope_kv(1, 4, 8, 64, None, None, None, None, None, None, None, None, 0,
                                None, None, None, 0.0, None, 1e4, None, None, None, None, None,
                                0, 0, None)
    assert rc == scb._lib.SC_ERR_INVALID_ARGUMENT
    # cos without sin
    rc = lib.sc_dequant_rope_kv(1, 4, 8, 64, 1, s4, 1, s3, None, None, None, None, 0,
                                1, None, st(0, 1), 0.0, None, 1e4, None, 1, s4, None, None,
                                0, 0, None)
    assert rc == scb._lib.SC_ERR_INVALID_ARGUMENT
    # empty work is a successful no-op
    rc = lib.sc_dequant_rope_kv(1, 0, 8, 64, 1, s4, 1, s3, None, None, None, None, 0,
                                None, None, None, 0.0, None, 1e4, None, 1, s4, None, None,
                                0, 0, None)
    assert rc == 0 and _err(lib) == ""


def test_quantize_and_tables_reject_bad_arguments(scb):
    lib = scb._lib.load()
    st = scb._lib.strides
    rc = lib.sc_quantize_int8(4, 2, 64, 1, 7, st(128, 64, 1), 1e-5, 1, st(128, 64, 1), 1, 0,
                              st(2, 1), 0, None)
    assert rc == scb._lib.SC_ERR_INVALID_DTYPE
    rc = lib.sc_rope_cos_sin_delta(1, 4, 63, 1e4, None, 1, 1, 0, None)
    assert rc == scb._lib.SC_ERR_INVALID_ARGUMENT
    rc = lib.sc_rope_cos_sin_delta(1, 4, 64, 1e4, None, 1, 1, 9, None)
    assert rc == scb._lib.SC_ERR_INVALID_DTYPE
    assert lib.sc_rope_cos_sin_delta(None, 0, 64, 1e4, None, None, None, 0, None) == 0


def test_paged_rejects_bad_arguments(scb):
    lib = scb._lib.load()
    st = scb._lib.strides
    def call(head_dim=128, strides=(1024, 128, 1), status=16, table_stride=4):
        return lib.sc_restore_paged(2, 4, 64, 8, head_dim, 10, 16, 16, 16, 16, 16, table_stride,
                                    16, 16, 0, 1e4, None, 16, 16, 16, st(*strides), 1 << 20,
                                    0, status, 0, None)

    assert call(head_dim=48) == scb._lib.SC_ERR_UNSUPPORTED
    assert call(strides=(1024, 128, 2)) == scb._lib.SC_ERR_INVALID_ARGUMENT
    assert call(status=None) == scb._lib.SC_ERR_INVALID_ARGUMENT
    assert call(table_stride=3) == scb._lib.SC_ERR_INVALID_ARGUMENT


def test_sizes_whose_products_overflow_are_rejected_before_cuda(scb):
    # sizes whose products do not fit in 64 bits are refused, not wrapped: 8 x 2^61 rows once
    # wrapped to 0 rows and the call returned success without doing anything
    lib = scb._lib.load()
    st = scb._lib.strides
    bad = scb._lib.SC_ERR_INVALID_ARGUMENT
    s4, s3 = st(0, 8 * 64, 64, 1), st(0, 8, 1)
    rc = lib.sc_dequant_rope_kv(8, 2 ** 61, 1, 64, 16, s4, 16, s3, None, None, None, None, 0,
                                None, None, None, 0.0, None, 1e4, None, 16, s4, None, None,
                                0, 0, None)
    assert rc == bad and "rows" in _err(lib)
    rc = lib.sc_quantize_int8(2 ** 62, 8, 64, 16, 0, st(512, 64, 1), 1e-5, 16, st(512, 64, 1),
                              16, 0, st(8, 1), 0, None)
    assert rc == bad and "rows" in _err(lib)
    rc = lib.sc_rope_shift_keys(2 ** 62, 8, 64, 16, 0, st(512, 64, 1), None, None, None, 5.0,
                                1e4, None, 16, 0, st(512, 64, 1), None)
    assert rc == bad
    rc = lib.sc_rope_cos_sin_delta(16, 2 ** 62, 64, 1e4, None, 16, 16, 0, None)
    assert rc == bad
    rc = lib.sc_restore_paged(2 ** 31 - 1, 2 ** 31 - 1, 64, 8, 128, 10, 16, 16, 16, 16, 16,
                              2 ** 31 - 1, 16, 16, 0, 1e4, None, 16, 16, 16, st(1024, 128, 1),
                              1 << 20, 0, 16, 0, None)
    assert rc == bad
    rc = lib.sc_dequant_rope_kv_token_shifts_noalloc(1, 2 ** 62, 8, 128, 16, s4, 16, s3, None,
                                                     None, None, None, 0, 16, 1e4, None, 16, s4,
                                                     None, None, 0, 0, None)
    assert rc == bad and "capacity" in _err(lib)
    h = ctypes.c_void_p()
    rc = lib.sc_pipeline_create(0, 2, 2 ** 40, 64, 8, 128, 8, 2, 0, ctypes.byref(h))
    assert rc == bad and "too large" in _err(lib) and h.value is None


def test_pipeline_rejects_bad_geometry(scb):
    lib = scb._lib.load()
    h = ctypes.c_void_p()
    rc = lib.sc_pipeline_create(0, 0, 8, 64, 8, 128, 8, 2, 0, ctypes.byref(h))
    assert rc == scb._lib.SC_ERR_INVALID_ARGUMENT and h.value is None
    rc = lib.sc_pipeline_create(0, 2, 8, 64, 8, 100, 8, 2, 0, ctypes.byref(h))
    assert rc == scb._lib.SC_ERR_UNSUPPORTED
    assert lib.sc_pipeline_destroy(None) == 0
    assert lib.sc_pipeline_restore(None, None, None, 0, 1e4, None, None, None, None, 0, 0,
                                   None) == scb._lib.SC_ERR_INVALID_ARGUMENT


def test_validation_messages_match_reference(scb):
    # reference tests/test_correctness.py:277-292
    with pytest.raises(ValueError, match="head_dim must be even"):
        k = torch.zeros((4, 2, 63), dtype=torch.int8)
        s = torch.ones((4, 2, 1), dtype=torch.float16)
        c = torch.ones((1, 31), dtype=torch.float16)
        scb.validate_key_inputs(k, s, c, c)
    with pytest.raises(TypeError, match="must be torch.int8"):
        k = torch.zeros((4, 2, 64), dtype=torch.float16)
        s = torch.ones((4, 2, 1), dtype=torch.float16)
        c = torch.ones((1, 32), dtype=torch.float16)
        scb.validate_key_inputs(k, s, c, c)
    with pytest.raises(ValueError, match="cos_delta must have shape"):
        k = torch.zeros((4, 2, 64), dtype=torch.int8)
        s = torch.ones((4, 2, 1), dtype=torch.float16)
        c = torch.ones((3, 32), dtype=torch.float16)
        scb.validate_key_inputs(k, s, c, c)
    with pytest.raises(TypeError, match="v_scale must be torch.float16"):
        scb.validate_value_inputs(torch.zeros((4, 2, 64), dtype=torch.int8),
                                  torch.ones((4, 2, 1), dtype=torch.float32))
    with pytest.raises(ValueError, match="Either \\(cos_delta, sin_delta\\)"):
        scb.triton_fused_k_dequant_rope_shift(torch.zeros((4, 2, 64), dtype=torch.int8),
                                              torch.ones((4, 2, 1), dtype=torch.float16))


def test_operators_refuse_cpu_tensors(scb):
    k = torch.zeros((4, 2, 64), dtype=torch.int8)
    s = torch.ones((4, 2, 1), dtype=torch.float16)
    for call in (
        lambda: scb.triton_fused_k_dequant_rope_shift(k, s, delta_p=3),
        lambda: scb.dequant_value(k, s),
        lambda: scb.quantize_kv_int8(torch.zeros((4, 2, 64))),
        lambda: scb.compute_rope_cos_sin_delta(torch.tensor([3]), 64),
    ):
        with pytest.raises(RuntimeError, match="CUDA device"):
            call()


# The fifteen public names of the reference's kernels package
# (speccache/kernels/__init__.py:23-38).
REFERENCE_KERNEL_NAMES = [
    "compute_rope_cos_sin_delta", "dequant_and_rope_key", "dequant_and_rope_key_compiled",
    "dequant_and_rope_key_ref", "dequant_kv_cache", "dequant_value", "dequant_value_compiled",
    "dequant_value_ref", "fused_k_dequant_rope_shift_kernel", "pytorch_compiled_dequant_rope_shift",
    "pytorch_eager_dequant_rope_shift", "quantize_kv_int8", "quantize_symmetric_int8",
    "rotate_half", "triton_fused_k_dequant_rope_shift",
]


def test_every_reference_kernel_name_is_exported(scb):
    for name in REFERENCE_KERNEL_NAMES:
        assert name in scb.__all__ and name in scb.kernels.__all__, name
        assert getattr(scb, name) is getattr(scb.kernels, name), name


def test_reference_eager_and_compiled_names_refuse_cpu_tensors(scb):
    k = torch.zeros((4, 2, 64), dtype=torch.int8)
    s = torch.ones((4, 2, 1), dtype=torch.float16)
    for name in ("pytorch_eager_dequant_rope_shift", "dequant_and_rope_key_ref",
                 "pytorch_compiled_dequant_rope_shift", "dequant_and_rope_key_compiled",
                 "dequant_and_rope_key"):
        with pytest.raises(RuntimeError, match="CUDA device"):
            getattr(scb, name)(k, s, delta_p=3)
    for name in ("dequant_value_ref", "dequant_value_compiled"):
        with pytest.raises(RuntimeError, match="CUDA device"):
            getattr(scb, name)(k, s)


def test_kernel_handle_explains_itself(scb):
    kern = scb.fused_k_dequant_rope_shift_kernel
    assert "sc_dequant_rope_kv" in repr(kern)
    with pytest.raises(TypeError, match="sc_dequant_rope_kv"):
        kern[(1, 1)]
    with pytest.raises(TypeError, match="triton_fused_k_dequant_rope_shift"):
        kern(1, 2, 3)


def test_ctypes_stub_matches_the_header(scb):
    # include/b200_abi.py declares sc_dequant_rope_kv with as many arguments as the header
    import importlib.util

    os.environ["SPECCACHE_B200_LIB"] = scb._lib.LIB_PATH
    spec = importlib.util.spec_from_file_location("b200_abi", os.path.join(REPO, "include", "b200_abi.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    with open(HEADER) as f:
        text = f.read()
    decl = re.search(r"SC_API int32_t sc_dequant_rope_kv\((.*?)\);", text, re.S).group(1)
    assert len(mod._lib.sc_dequant_rope_kv.argtypes) == decl.count(",") + 1
    assert mod.SC_FLAG_FP32_INTERMEDIATE == scb._lib.SC_FLAG_FP32_INTERMEDIATE


def test_rotate_half_convention(scb):
    x = torch.tensor([[[1.0, 2.0, 3.0, 4.0]]])
    assert torch.equal(scb.rotate_half(x), torch.tensor([[[-3.0, -4.0, 1.0, 2.0]]]))


def test_fastdiv_magic_numbers():
    # Host restatement of make_fastdiv/fdiv in csrc/sc_common.cuh, exhaustive over edge
    # numerators for the divisor range the kernels use (heads, tokens).
    def make(d):
        l = 0
        while (1 << l) < d:
            l += 1
        m = ((1 << 32) * ((1 << l) - d)) // d + 1
        return m & 0xFFFFFFFF, l

    for d in list(range(1, 300)) + [4095, 4096, 8191, 8192, 16384, 32768, 65535, 2**20 + 7]:
        m, s = make(d)
        for n in list(range(0, 3000)) + [2**31 - 1, 2**31 - 2, 2**30, 123456789, d * 1000 - 1]:
            t = (n * m) >> 32
            assert (t + n) >> s == n // d, (d, n)
