"""Input contract of the restore operators (host-side, no device work).

Same checks, exception types and message text as the reference's
``validate_key_inputs`` / ``validate_value_inputs``
(speccache/kernels/reference.py:13-119), so callers that match on the messages keep
working.  One additive extension: ``out`` may be bfloat16 as well as float16.
"""

from __future__ import annotations

import torch

OUT_DTYPES = (torch.float16, torch.bfloat16)


def _check_out(out: torch.Tensor | None, t: int, h: int, d: int, device, key: bool) -> None:
    if out is None:
        return
    if out.shape != (t, h, d):
        if key:
            raise ValueError(f"Pre-allocated out tensor must have shape [{t}, {h}, {d}], got {out.shape}")
        raise ValueError(f"out tensor must have shape [{t}, {h}, {d}], got {out.shape}")
    if out.dtype not in OUT_DTYPES:
        raise TypeError(f"out tensor must be torch.float16 (or torch.bfloat16), got {out.dtype}")
    if out.device != device:
        raise ValueError(f"out tensor device ({out.device}) does not match input device ({device})")


def validate_key_core(k_quant: torch.Tensor, k_scale: torch.Tensor,
                      out: torch.Tensor | None = None) -> None:
    """The shift-independent part of the key contract (reference.py:24-42, 70-80)."""
    if k_quant.ndim != 3:
        raise ValueError(
            f"k_quant must be 3-dimensional [num_tokens, num_kv_heads, head_dim], "
            f"got ndim={k_quant.ndim} with shape {k_quant.shape}")
    t, h, d = k_quant.shape
    if d % 2 != 0:
        raise ValueError(f"head_dim must be even for RoPE half-pairing, got head_dim={d}")
    if k_quant.dtype != torch.int8:
        raise TypeError(f"k_quant must be torch.int8, got {k_quant.dtype}")
    if k_scale.ndim != 3 or k_scale.shape != (t, h, 1):
        raise ValueError(f"k_scale must have shape [{t}, {h}, 1], got {k_scale.shape}")
    if k_scale.dtype != torch.float16:
        raise TypeError(f"k_scale must be torch.float16, got {k_scale.dtype}")
    if k_scale.device != k_quant.device:
        raise ValueError(
            f"All tensors must reside on the same device ({k_quant.device}), but got devices: "
            f"k_scale={k_scale.device}")
    _check_out(out, t, h, d, k_quant.device, key=True)


def validate_key_inputs(k_quant: torch.Tensor, k_scale: torch.Tensor, cos_delta: torch.Tensor,
                        sin_delta: torch.Tensor, out: torch.Tensor | None = None) -> None:
    """Full key contract including the cos/sin tables (reference.py:13-80)."""
    validate_key_core(k_quant, k_scale, None)
    t, h, d = k_quant.shape
    d_half = d // 2
    if tuple(cos_delta.shape) not in {(1, d_half), (t, d_half)}:
        raise ValueError(
            f"cos_delta must have shape [1, {d_half}] or [{t}, {d_half}], got {cos_delta.shape}")
    if sin_delta.shape != cos_delta.shape:
        raise ValueError(
            f"sin_delta shape {sin_delta.shape} must match cos_delta shape {cos_delta.shape}")
    if cos_delta.dtype != torch.float16 or sin_delta.dtype != torch.float16:
        raise TypeError(
            f"cos_delta and sin_delta must be torch.float16, got "
            f"{cos_delta.dtype} and {sin_delta.dtype}")
    device = k_quant.device
    if k_scale.device != device or cos_delta.device != device or sin_delta.device != device:
        raise ValueError(
            f"All tensors must reside on the same device ({device}), but got devices: "
            f"k_scale={k_scale.device}, cos_delta={cos_delta.device}, sin_delta={sin_delta.device}")
    _check_out(out, t, h, d, device, key=True)


def validate_value_inputs(v_quant: torch.Tensor, v_scale: torch.Tensor,
                          out: torch.Tensor | None = None) -> None:
    """Value contract (reference.py:83-119)."""
    if v_quant.ndim != 3:
        raise ValueError(
            f"v_quant must be 3-dimensional [num_tokens, num_kv_heads, head_dim], "
            f"got ndim={v_quant.ndim} with shape {v_quant.shape}")
    t, h, d = v_quant.shape
    if v_quant.dtype != torch.int8:
        raise TypeError(f"v_quant must be torch.int8, got {v_quant.dtype}")
    if v_scale.ndim != 3 or v_scale.shape != (t, h, 1):
        raise ValueError(f"v_scale must have shape [{t}, {h}, 1], got {v_scale.shape}")
    if v_scale.dtype != torch.float16:
        raise TypeError(f"v_scale must be torch.float16, got {v_scale.dtype}")
    if v_scale.device != v_quant.device:
        raise ValueError(
            f"v_scale device ({v_scale.device}) does not match v_quant device ({v_quant.device})")
    _check_out(out, t, h, d, v_quant.device, key=False)


def require_cuda(t: torch.Tensor) -> None:
    """The operators run on the GPU only (no CPU fallback), like triton_rope_kv.py:287-290."""
    if not t.is_cuda:
        raise RuntimeError(
            f"SpecCache B200 kernels require an NVIDIA CUDA device, got device: {t.device}.")


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    """HF half-split rotation ``[x1, x2] -> [-x2, x1]`` (reference.py:168-176).

    A tensor utility kept for API compatibility; the restore kernels never call it.
    """
    d_half = x.shape[-1] // 2
    return torch.cat((-x[..., d_half:], x[..., :d_half]), dim=-1)
