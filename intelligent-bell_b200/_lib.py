"""ctypes binding of ``libspeccache_b200.so`` (the C ABI in include/speccache_b200.h).

There is no fallback: if the library is missing or a CUDA device is absent, the
operators raise.  Status codes map onto the exception types the reference raises for
the same conditions (speccache/kernels/reference.py:13-119, triton_rope_kv.py:287-290):
SC_ERR_INVALID_ARGUMENT -> ValueError, SC_ERR_INVALID_DTYPE -> TypeError, everything
else -> RuntimeError.
"""

from __future__ import annotations

import ctypes
import os
import threading

import numpy as np
import torch

from ._build import LIB_PATH

SC_OK = 0
SC_ERR_INVALID_ARGUMENT = 1
SC_ERR_INVALID_DTYPE = 2
SC_ERR_CUDA = 3
SC_ERR_OUT_OF_RANGE = 4
SC_ERR_TIMEOUT = 5
SC_ERR_HOST_ALLOC = 6
SC_ERR_UNSUPPORTED = 7

SC_DTYPE_F16 = 0
SC_DTYPE_BF16 = 1
SC_DTYPE_F32 = 2

SC_FLAG_FP32_INTERMEDIATE = 0x1
SC_FLAG_FORCE_GENERIC = 0x2

SC_STATUS_BAD_PAGE_ID = 0x1
SC_STATUS_BAD_SEQ_LEN = 0x2
SC_STATUS_BAD_OUT_OFFSET = 0x4

SC_PIPE_NUMA_LOCAL = 0x1
SC_PIPE_WRITE_COMBINED = 0x2
SC_PIPE_PER_LAYER = 0x4
SC_PIPE_SPLIT_KV_COPIES = 0x8

SC_IPC_HANDLE_BYTES = 64

DTYPE_CODE = {torch.float16: SC_DTYPE_F16, torch.bfloat16: SC_DTYPE_BF16, torch.float32: SC_DTYPE_F32}

# Every symbol the header declares, with its ctypes signature.
_vp, _i32, _i64, _u32, _f32, _f64 = (ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64,
                                     ctypes.c_uint32, ctypes.c_float, ctypes.c_double)
_SIGNATURES = {
    "sc_last_error": (ctypes.c_char_p, []),
    "sc_abi_version": (_i32, []),
    "sc_preload_kernels": (_i32, []),
    "sc_rope_cos_sin_delta": (_i32, [_vp, _i64, _i32, _f64, _vp, _vp, _vp, _i32, _vp]),
    "sc_dequant_rope_kv": (_i32, [_i32, _i64, _i32, _i32,
                                  _vp, _vp, _vp, _vp,   # k_quant, kq_strides, k_scale, ks_strides
                                  _vp, _vp, _vp, _vp,   # v_quant, vq_strides, v_scale, vs_strides
                                  _i32,                 # scale_dtype
                                  _vp, _vp, _vp,        # cos, sin, cs_strides
                                  _f64, _vp, _f64, _vp,  # delta_p, delta_p_dev, theta, inv_freq
                                  _vp, _vp, _vp, _vp,   # k_out, ko_strides, v_out, vo_strides
                                  _i32, _u32, _vp]),
    "sc_dequant_rope_kv_token_shifts_noalloc": (_i32, [_i32, _i64, _i32, _i32,
                                                       _vp, _vp, _vp, _vp,  # K codes/scales
                                                       _vp, _vp, _vp, _vp,  # V codes/scales
                                                       _i32, _vp, _f64, _vp,  # dtype, shifts
                                                       _vp, _vp, _vp, _vp,  # outputs
                                                       _i32, _u32, _vp]),
    "sc_rope_shift_keys": (_i32, [_i64, _i32, _i32, _vp, _i32, _vp, _vp, _vp, _vp, _f64, _f64,
                                  _vp, _vp, _i32, _vp, _vp]),
    "sc_quantize_int8": (_i32, [_i64, _i32, _i32, _vp, _i32, _vp, _f32, _vp, _vp, _vp, _i32,
                                _vp, _u32, _vp]),
    "sc_restore_paged": (_i32, [_i32, _i32, _i32, _i32, _i32, _i64,
                                _vp, _vp, _vp, _vp,     # pools
                                _vp, _i64, _vp,         # page_table, stride, seq_lens
                                _vp, _i32, _f64, _vp,   # delta_p, per_page, theta, inv_freq
                                _vp, _vp, _vp, _vp,     # k_out, v_out, out_offsets, out_strides
                                _i64, _i32, _vp, _u32, _vp]),
    "sc_pipeline_create": (_i32, [_i32, _i32, _i64, _i32, _i32, _i32, _i64, _i32, _u32, _vp]),
    "sc_pipeline_host_slabs": (_i32, [_vp, _vp, _vp, _vp, _vp]),
    "sc_pipeline_restore": (_i32, [_vp, _vp, _vp, _i32, _f64, _vp, _vp, _vp, _vp, _i64, _i32,
                                   _vp]),
    "sc_pipeline_offload": (_i32, [_vp, _i32, _vp, _i32, _vp, _vp, _vp, _vp, _i32, _vp]),
    "sc_pipeline_synchronize": (_i32, [_vp, _f64]),
    "sc_pipeline_join": (_i32, [_vp, _vp]),
    "sc_pipeline_status": (_i32, [_vp, _vp]),
    "sc_pipeline_restore_launches": (_i32, [_vp, _i32, _vp]),
    "sc_pipeline_plan": (_i32, [_vp, _i32, _vp, _i32, _vp, _vp]),
    "sc_pipeline_destroy": (_i32, [_vp]),
    "sc_ipc_export": (_i32, [_vp, _vp, _vp]),
    "sc_ipc_import": (_i32, [_vp, _i64, _vp, _vp]),
    "sc_ipc_close": (_i32, [_vp]),
}

_lock = threading.Lock()
_lib = None


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def load() -> ctypes.CDLL:
    """Load the library once (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{os.path.basename(LIB_PATH)} is not built: run "
                "`python -c 'import __graft_entry__ as g; g.build()'` (needs nvcc)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    if rc == SC_OK:
        return
    msg = load().sc_last_error().decode(errors="replace")
    text = f"{what}: {msg}" if msg else f"{what}: status {rc}"
    if rc == SC_ERR_INVALID_ARGUMENT:
        raise ValueError(text)
    if rc == SC_ERR_INVALID_DTYPE:
        raise TypeError(text)
    if rc == SC_ERR_TIMEOUT:
        raise TimeoutError(text)
    raise RuntimeError(text)


def strides(*values) -> ctypes.Array:
    arr = (ctypes.c_int64 * len(values))(*[int(v) for v in values])
    return arr


class StrideBuffer:
    """A reusable per-thread host buffer for the stride arrays of one call.

    The library copies the strides during the call, so one buffer per thread can serve
    every call; ``put`` writes values and returns their address.
    """

    SIZE = 64

    def __init__(self) -> None:
        self.buf = (ctypes.c_int64 * self.SIZE)()
        self.base = ctypes.addressof(self.buf)
        self.used = 0

    def reset(self) -> "StrideBuffer":
        self.used = 0
        return self

    def put(self, values) -> int:
        n = len(values)
        start = self.used
        self.buf[start:start + n] = values
        self.used = start + n
        return self.base + 8 * start


_tls = threading.local()


def stride_buffer() -> StrideBuffer:
    b = getattr(_tls, "strides", None)
    if b is None:
        b = _tls.strides = StrideBuffer()
    return b.reset()


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_handle(device: torch.device) -> int:
    """cudaStream_t of torch's current stream on ``device``."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if _raw_stream is not None:
        return _raw_stream(idx)
    return torch.cuda.current_stream(idx).cuda_stream


class on_device:
    """Make ``device`` current for the call only if it is not already (cheap no-op path)."""

    __slots__ = ("idx", "prev")

    def __init__(self, device: torch.device) -> None:
        self.idx = device.index
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if self.idx is not None and self.idx != cur:
            self.prev = cur
            torch.cuda.set_device(self.idx)
        return self

    def __exit__(self, *exc) -> None:
        if self.prev is not None:
            torch.cuda.set_device(self.prev)


_INV_FREQ: dict[tuple[int, float], np.ndarray] = {}


def inv_freq_table(head_dim: int, theta: float) -> np.ndarray:
    """Rotary inverse frequencies in float32, computed once per (head_dim, theta) with the
    reference's own expression (speccache/kernels/reference.py:151-153) so that the
    in-kernel cos/sin tables use the same bits."""
    key = (int(head_dim), float(theta))
    tab = _INV_FREQ.get(key)
    if tab is None:
        idx = torch.arange(0, head_dim // 2, dtype=torch.float32)
        tab = (1.0 / (float(theta) ** (2.0 * idx / head_dim))).numpy().astype(np.float32)
        tab = np.ascontiguousarray(tab)
        _INV_FREQ[key] = tab
    return tab


def inv_freq_ptr(head_dim: int, theta: float) -> int:
    return inv_freq_table(head_dim, theta).ctypes.data
