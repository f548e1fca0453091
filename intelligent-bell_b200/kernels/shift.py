"""RoPE shift of already dequantised keys on the GPU.

The rotation of ``MultiLayerKVInjector.apply_rope_shift`` (speccache/serving/kv_injector.py:
246-283): float16/bfloat16 keys ``[T, H, D]`` or in the model layout ``[1, H, T, D]``,
rotated by the fp16 tables of ``delta_p`` with the reference's float32 arithmetic, result in
the same dtype and layout.  One launch of ``sc_rope_shift_keys``; the layout is handled by
strides (no permute copies), and the result may be written in place or into a cache view.
"""

from __future__ import annotations

import torch

from .. import _lib
from .restore import DEFAULT_THETA
from .validation import require_cuda

_KEY_DTYPES = (torch.float16, torch.bfloat16)


def token_major(x: torch.Tensor) -> torch.Tensor:
    """``[T, H, D]`` view of ``x`` (``[T, H, D]``, or ``[1, H, T, D]`` permuted without a copy)."""
    if x.ndim == 3:
        return x
    if x.ndim == 4:
        if x.shape[0] != 1:
            raise ValueError(f"model-layout keys must have batch 1, got {tuple(x.shape)}")
        return x[0].permute(1, 0, 2)
    raise ValueError(f"Unexpected tensor ndim={x.ndim}, expected 3 or 4.")


def rope_shift_keys(
    k: torch.Tensor,
    delta_p: int | float | torch.Tensor | None = None,
    *,
    cos_delta: torch.Tensor | None = None,
    sin_delta: torch.Tensor | None = None,
    theta: float = DEFAULT_THETA,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Rotate keys ``k`` by the relative shift ``delta_p`` (or by the given fp16 tables
    ``[1 | T, D/2]``).  Returns a new tensor of ``k``'s shape and dtype, or ``out`` (same
    shape, float16/bfloat16, any strides; it may be ``k`` itself)."""
    if k.dtype not in _KEY_DTYPES:
        raise TypeError(f"keys must be float16 or bfloat16, got {k.dtype}")
    require_cuda(k)
    kt = token_major(k)
    t, h, d = kt.shape
    if d % 2 != 0:
        raise ValueError(f"head_dim must be even, got {d}")
    if out is None:
        out = torch.empty(k.shape, dtype=k.dtype, device=k.device)
    elif out.shape != k.shape or out.device != k.device or out.dtype not in _KEY_DTYPES:
        raise ValueError(f"out must be a float16/bfloat16 tensor of shape {tuple(k.shape)} on "
                         f"{k.device}, got {tuple(out.shape)} {out.dtype} on {out.device}")
    ot = token_major(out)
    cos_ptr = sin_ptr = cs_strides = None
    dp = 0.0
    if cos_delta is not None or sin_delta is not None:
        if cos_delta is None or sin_delta is None:
            raise ValueError("cos_delta and sin_delta must be given together")
        for tab in (cos_delta, sin_delta):
            if tab.dtype != torch.float16 or tab.device != k.device or tab.ndim != 2:
                raise ValueError("cos/sin tables must be float16 [1 | T, D/2] on the keys' device")
            if tab.shape[1] != d // 2 or tab.shape[0] not in (1, t):
                raise ValueError(f"cos/sin tables must be [1, {d // 2}] or [{t}, {d // 2}], "
                                 f"got {tuple(tab.shape)}")
        if cos_delta.stride() != sin_delta.stride():
            raise ValueError("cos and sin tables must share strides")
        cos_ptr, sin_ptr = cos_delta.data_ptr(), sin_delta.data_ptr()
        cs_strides = _lib.strides(0 if cos_delta.shape[0] == 1 else cos_delta.stride(0),
                                  cos_delta.stride(1))
    elif delta_p is None:
        raise ValueError(
            "Either (cos_delta, sin_delta) tensors or delta_p displacement must be provided.")
    else:
        dp = float(delta_p.reshape(-1)[0]) if isinstance(delta_p, torch.Tensor) else float(delta_p)
    lib = _lib.load()
    with torch.cuda.device(k.device):
        rc = lib.sc_rope_shift_keys(
            t, h, d, kt.data_ptr(), _lib.DTYPE_CODE[k.dtype], _lib.strides(*kt.stride()),
            cos_ptr, sin_ptr, cs_strides, dp, float(theta), _lib.inv_freq_ptr(d, theta),
            ot.data_ptr(), _lib.DTYPE_CODE[out.dtype], _lib.strides(*ot.stride()),
            _lib.stream_handle(k.device))
    _lib.check(rc, "rope_shift_keys")
    return out
