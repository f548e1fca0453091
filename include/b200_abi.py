"""ctypes binding of the C ABI (``include/speccache_b200.h``) for the reference's own wrappers.

A maintainer who keeps the reference's Python wrappers and replaces only the Triton kernel
launch copies this file next to ``speccache/kernels/triton_rope_kv.py`` (as
``speccache/kernels/b200_abi.py``) and calls ``fused_k_dequant_rope_shift`` where the wrapper
launches ``fused_k_dequant_rope_shift_kernel[grid](...)`` (triton_rope_kv.py:320-343).

The library is found through the environment variable ``SPECCACHE_B200_LIB`` (the path of
``libspeccache_b200.so``), or next to this file's repository when it is used in place.
Argument types follow the header's declaration of ``sc_dequant_rope_kv``.
"""

import ctypes
import os

import torch

_DEFAULT = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                        "intelligent-bell_b200", "libspeccache_b200.so")
_lib = ctypes.CDLL(os.environ.get("SPECCACHE_B200_LIB", _DEFAULT))
_vp, _i32, _i64, _u32, _f64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_uint32, ctypes.c_double
_lib.sc_dequant_rope_kv.restype = _i32
_lib.sc_dequant_rope_kv.argtypes = [_i32, _i64, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                    _i32, _vp, _vp, _vp, _f64, _vp, _f64, _vp, _vp, _vp, _vp, _vp,
                                    _i32, _u32, _vp]
_lib.sc_last_error.restype = ctypes.c_char_p

SC_FLAG_FP32_INTERMEDIATE = 1  # q*s kept in fp32 before the rotation (the Triton kernel's arithmetic)


def _s(*v):
    return (ctypes.c_int64 * len(v))(*v)


def fused_k_dequant_rope_shift(k_quant, k_scale, cos_delta, sin_delta, out, fp32_intermediate=True):
    """Drop-in for the kernel launch at triton_rope_kv.py:320-343 (fp16 tables, fp16 out).

    ``fp32_intermediate=True`` (default) is the Triton kernel's arithmetic; False rounds
    ``q*s`` to fp16 first, as the reference's eager function does (reference.py:257).
    """
    t, h, d = k_quant.shape
    cs_t = 0 if cos_delta.shape[0] == 1 else cos_delta.stride(0)
    rc = _lib.sc_dequant_rope_kv(
        1, t, h, d,
        k_quant.data_ptr(), _s(0, *k_quant.stride()), k_scale.data_ptr(), _s(0, k_scale.stride(0), k_scale.stride(1)),
        None, None, None, None, 0,
        cos_delta.data_ptr(), sin_delta.data_ptr(), _s(cs_t, cos_delta.stride(1)),
        0.0, None, 10000.0, None,
        out.data_ptr(), _s(0, *out.stride()), None, None,
        0, SC_FLAG_FP32_INTERMEDIATE if fp32_intermediate else 0,
        torch.cuda.current_stream().cuda_stream)
    if rc != 0:
        raise RuntimeError(_lib.sc_last_error().decode())
    return out
