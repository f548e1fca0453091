"""INT8 absmax quantisation on the GPU — the offload twin of the restore kernels.

Drop-in for ``quantize_kv_int8`` / ``quantize_symmetric_int8``
(speccache/kernels/reference.py:179-209): int8 codes ``[T, H, D]`` and float16 scales
``[T, H, 1]``, bit-exact with the reference's CPU arithmetic (IEEE divisions,
round-half-even, clamp to +-127).  Runs on ``torch.cuda.current_stream()``.

Extensions: preallocated ``q_out`` / ``scale_out`` (any strides), float32 scales.
Inputs may be float16, bfloat16 or float32.  Non-finite inputs are outside the
contract (the reference's int8 cast of NaN is undefined as well).
"""

from __future__ import annotations

import torch

from .. import _lib
from .validation import require_cuda


def quantize_kv_int8(
    x: torch.Tensor,
    eps: float = 1e-5,
    *,
    q_out: torch.Tensor | None = None,
    scale_out: torch.Tensor | None = None,
    scale_dtype: torch.dtype = torch.float16,
) -> tuple[torch.Tensor, torch.Tensor]:
    if x.ndim != 3:
        raise ValueError(f"Input tensor must have shape [T, H, D], got {x.shape}")
    if x.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise TypeError(f"x must be float16, bfloat16 or float32, got {x.dtype}")
    require_cuda(x)
    t, h, d = x.shape
    if scale_out is not None:
        scale_dtype = scale_out.dtype
    if scale_dtype not in (torch.float16, torch.float32):
        raise TypeError(f"scale dtype must be float16 or float32, got {scale_dtype}")
    if q_out is None:
        q_out = torch.empty((t, h, d), dtype=torch.int8, device=x.device)
    elif q_out.shape != (t, h, d) or q_out.dtype != torch.int8 or q_out.device != x.device:
        raise ValueError(f"q_out must be int8 [{t}, {h}, {d}] on {x.device}")
    if scale_out is None:
        scale_out = torch.empty((t, h, 1), dtype=scale_dtype, device=x.device)
    elif scale_out.shape != (t, h, 1) or scale_out.device != x.device:
        raise ValueError(f"scale_out must be [{t}, {h}, 1] on {x.device}")
    lib = _lib.load()
    with torch.cuda.device(x.device):
        rc = lib.sc_quantize_int8(
            t, h, d, x.data_ptr(), _lib.DTYPE_CODE[x.dtype], _lib.strides(*x.stride()),
            float(eps), q_out.data_ptr(), _lib.strides(*q_out.stride()),
            scale_out.data_ptr(), _lib.DTYPE_CODE[scale_dtype],
            _lib.strides(scale_out.stride(0), scale_out.stride(1)), 0,
            _lib.stream_handle(x.device))
    _lib.check(rc, "quantize_kv_int8")
    return q_out, scale_out


quantize_symmetric_int8 = quantize_kv_int8
