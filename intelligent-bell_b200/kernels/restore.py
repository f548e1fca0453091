"""Restore operators: INT8 K dequant + relative RoPE shift, V dequant, cos/sin tables.

Drop-in replacements for the reference's kernel entry points
(speccache/kernels/triton_rope_kv.py:243-427 and the table helper in
speccache/kernels/reference.py:122-165), with the same names, arguments, ``out=``
semantics (written in place and returned) and exceptions.  They run the sm_100a kernels
of ``libspeccache_b200.so`` on ``torch.cuda.current_stream()``; nothing synchronises.

Two arithmetics, both within the reference's rtol = atol = 1e-2 of each other:
  * fp32 intermediate: ``x = q*s`` stays in fp32 before the rotation, the arithmetic of the
    reference's Triton kernel (triton_rope_kv.py:150-158).  It is the default of the names
    that replace the Triton wrappers (``triton_fused_k_dequant_rope_shift``,
    ``dequant_and_rope_key``, ``dequant_kv_cache``) and of ``pytorch_compiled_dequant_rope_shift``
    / ``dequant_and_rope_key_compiled`` (Inductor drops the fp16 round trip of the eager code).
  * fp16 intermediate: ``x`` is rounded to fp16 first, the reference's eager arithmetic
    (reference.py:257), used by ``pytorch_eager_dequant_rope_shift`` /
    ``dequant_and_rope_key_ref`` and by ``restore_layers`` (default).
Either way every product and sum is rounded as torch rounds its separate multiply and add,
so given the same cos/sin tables the outputs are bit-exact against the reference's torch
arithmetic of that kind.  ``fp32_intermediate=`` selects the other one on any of them.

Additive extensions (other defaults keep the reference's behaviour):
  * ``theta=`` for the ``delta_p`` path (the reference hard-wires 10000);
  * bfloat16 outputs (``out`` of dtype bf16, or ``out_dtype=torch.bfloat16``);
  * arbitrary input/output strides (no ``.contiguous()`` copies);
  * ``restore_layers`` restores many layers ``[L, T, H, D]`` in one launch.

Every name takes CUDA tensors only and raises ``RuntimeError`` for CPU tensors: there is
no CPU path.
"""

from __future__ import annotations

import torch

from .. import _lib
from .staging import host_array, to_device
from .validation import (
    OUT_DTYPES,
    require_cuda,
    validate_key_core,
    validate_key_inputs,
    validate_value_inputs,
)

DEFAULT_THETA = 10000.0


def compute_rope_cos_sin_delta(
    delta_positions,
    head_dim: int,
    theta_base: float = DEFAULT_THETA,
    device: torch.device | str | None = None,
    dtype: torch.dtype = torch.float16,
) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin tables ``[n, head_dim/2]`` for relative shifts (reference.py:122-165)."""
    if head_dim % 2 != 0:
        raise ValueError(f"head_dim must be even, got {head_dim}")
    if dtype not in _lib.DTYPE_CODE:
        raise TypeError(f"table dtype must be float16, bfloat16 or float32, got {dtype}")
    dp = torch.as_tensor(delta_positions)
    if device is not None:
        dev = torch.device(device)
    else:
        dev = dp.device
    if dev.type != "cuda":
        raise RuntimeError(
            f"SpecCache B200 kernels require an NVIDIA CUDA device, got device: {dev}.")
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    (dp,) = to_device([host_array(dp.reshape(-1), torch.float32)], dev)
    n = dp.numel()
    half = head_dim // 2
    cos = torch.empty((n, half), dtype=dtype, device=dev)
    sin = torch.empty((n, half), dtype=dtype, device=dev)
    lib = _lib.load()
    with torch.cuda.device(dev):
        rc = lib.sc_rope_cos_sin_delta(
            dp.data_ptr(), n, head_dim, float(theta_base), _lib.inv_freq_ptr(head_dim, theta_base),
            cos.data_ptr(), sin.data_ptr(), _lib.DTYPE_CODE[dtype], _lib.stream_handle(dev))
    _lib.check(rc, "compute_rope_cos_sin_delta")
    return cos, sin


def _strides4(t: torch.Tensor):
    """[layer, token, head, dim] strides of a 3-D ([T,H,X]) or 4-D ([L,T,H,X]) tensor."""
    if t.ndim == 3:
        return (0,) + tuple(t.stride())
    return tuple(t.stride())


def _launch(n_layers, n_tokens, n_heads, head_dim, kq, ks, vq, vs, cos, sin, dp, dp_dev, theta,
            ko, vo, fp32_intermediate, force_generic=False) -> None:
    lib = _lib.load()
    ref = kq if kq is not None else vq
    out = ko if ko is not None else vo
    if out.dtype not in OUT_DTYPES:
        raise TypeError(f"out tensor must be torch.float16 (or torch.bfloat16), got {out.dtype}")
    if ko is not None and vo is not None and ko.dtype != vo.dtype:
        raise TypeError(f"K and V outputs must share a dtype, got {ko.dtype} and {vo.dtype}")
    scale = ks if ks is not None else vs
    if scale.dtype not in (torch.float16, torch.float32):
        raise TypeError(f"scale must be torch.float16 (or torch.float32), got {scale.dtype}")
    flags = (_lib.SC_FLAG_FP32_INTERMEDIATE if fp32_intermediate else 0) | (
        _lib.SC_FLAG_FORCE_GENERIC if force_generic else 0)
    sb = _lib.stride_buffer()
    kq_s = sb.put(_strides4(kq)) if kq is not None else None
    ks_s = sb.put(_strides4(ks)[:3]) if ks is not None else None
    vq_s = sb.put(_strides4(vq)) if vq is not None else None
    vs_s = sb.put(_strides4(vs)[:3]) if vs is not None else None
    ko_s = sb.put(_strides4(ko)) if ko is not None else None
    vo_s = sb.put(_strides4(vo)) if vo is not None else None
    cs_s = None
    if cos is not None:
        cs_s = sb.put((0 if cos.shape[0] == 1 else cos.stride(0), cos.stride(1)))
    inv = _lib.inv_freq_ptr(head_dim, theta) if cos is None else None
    with _lib.on_device(ref.device):
        rc = lib.sc_dequant_rope_kv(
            n_layers, n_tokens, n_heads, head_dim,
            _lib.ptr(kq), kq_s, _lib.ptr(ks), ks_s,
            _lib.ptr(vq), vq_s, _lib.ptr(vs), vs_s,
            _lib.DTYPE_CODE[scale.dtype],
            _lib.ptr(cos), _lib.ptr(sin), cs_s,
            float(dp), _lib.ptr(dp_dev), float(theta), inv,
            _lib.ptr(ko), ko_s, _lib.ptr(vo), vo_s,
            _lib.DTYPE_CODE[out.dtype], flags, _lib.stream_handle(ref.device))
    _lib.check(rc, "sc_dequant_rope_kv")


def _resolve_shift(k_quant, cos_delta, sin_delta, delta_p, theta):
    """Return (cos, sin, dp_scalar, dp_device_tensor) for the key path."""
    if cos_delta is not None and sin_delta is not None:
        return cos_delta, sin_delta, 0.0, None
    if delta_p is None:
        raise ValueError(
            "Either (cos_delta, sin_delta) tensors or delta_p displacement must be provided.")
    if isinstance(delta_p, torch.Tensor):
        if delta_p.numel() == 1:
            if delta_p.is_cuda:
                dev_dp = delta_p.reshape(1).to(device=k_quant.device, dtype=torch.float32)
                return None, None, 0.0, dev_dp
            return None, None, float(delta_p.reshape(-1)[0].to(torch.float32)), None
        # one shift per token: build [T, D/2] tables with the table kernel
        c, s = compute_rope_cos_sin_delta(delta_p, k_quant.shape[-1], theta, device=k_quant.device)
        return c, s, 0.0, None
    return None, None, float(delta_p), None


def _new_out(like: torch.Tensor, out_dtype) -> torch.Tensor:
    dtype = torch.float16 if out_dtype is None else out_dtype
    if dtype not in OUT_DTYPES:
        raise TypeError(f"out_dtype must be torch.float16 or torch.bfloat16, got {dtype}")
    return torch.empty(like.shape, dtype=dtype, device=like.device)


def triton_fused_k_dequant_rope_shift(
    k_quant: torch.Tensor,
    k_scale: torch.Tensor,
    cos_delta: torch.Tensor | None = None,
    sin_delta: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    *,
    delta_p: int | torch.Tensor | None = None,
    theta: float = DEFAULT_THETA,
    out_dtype: torch.dtype | None = None,
    fp32_intermediate: bool = True,
) -> torch.Tensor:
    """Fused INT8 key dequant + relative RoPE shift (triton_rope_kv.py:243-345).

    ``k_quant`` int8 ``[T, H, D]``, ``k_scale`` fp16 ``[T, H, 1]``, cos/sin fp16
    ``[1 | T, D/2]`` or ``delta_p`` (int, or tensor of 1 or T shifts).  Default arithmetic:
    the Triton kernel's (``q*s`` kept in fp32).
    """
    validate_key_core(k_quant, k_scale, out)
    cos, sin, dp, dp_dev = _resolve_shift(k_quant, cos_delta, sin_delta, delta_p, theta)
    if cos is not None:
        validate_key_inputs(k_quant, k_scale, cos, sin, out)
    require_cuda(k_quant)
    if out is None:
        out = _new_out(k_quant, out_dtype)
    t, h, d = k_quant.shape
    _launch(1, t, h, d, k_quant, k_scale, None, None, cos, sin, dp, dp_dev, theta, out, None,
            fp32_intermediate)
    return out


dequant_and_rope_key = triton_fused_k_dequant_rope_shift


def pytorch_eager_dequant_rope_shift(
    k_quant: torch.Tensor,
    k_scale: torch.Tensor,
    cos_delta: torch.Tensor | None = None,
    sin_delta: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    *,
    delta_p: int | torch.Tensor | None = None,
) -> torch.Tensor:
    """The reference's eager dequant + shift (reference.py:212-280) on the CUDA kernel.

    Same arguments and result as the reference function: the dequantised key is rounded to
    fp16 before the rotation (reference.py:257); a ``delta_p`` without tables uses theta
    10000 like the reference.  CUDA tensors only.
    """
    return triton_fused_k_dequant_rope_shift(k_quant, k_scale, cos_delta, sin_delta, out,
                                             delta_p=delta_p, fp32_intermediate=False)


dequant_and_rope_key_ref = pytorch_eager_dequant_rope_shift


def pytorch_compiled_dequant_rope_shift(
    k_quant: torch.Tensor,
    k_scale: torch.Tensor,
    cos_delta: torch.Tensor | None = None,
    sin_delta: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    *,
    delta_p: int | torch.Tensor | None = None,
) -> torch.Tensor:
    """Replaces the reference's ``torch.compile`` of the eager function (reference.py:310-322).

    Inductor does not keep the eager code's fp16 round trip of ``q*s``
    (``torch._inductor.config.emulate_precision_casts`` is off by default), so this runs the
    kernel with the dequantised key kept in fp32.  CUDA tensors only.
    """
    return triton_fused_k_dequant_rope_shift(k_quant, k_scale, cos_delta, sin_delta, out,
                                             delta_p=delta_p, fp32_intermediate=True)


dequant_and_rope_key_compiled = pytorch_compiled_dequant_rope_shift


def dequant_value(
    v_quant: torch.Tensor,
    v_scale: torch.Tensor,
    out: torch.Tensor | None = None,
    *,
    out_dtype: torch.dtype | None = None,
) -> torch.Tensor:
    """INT8 value dequant ``cvt(q * s)`` (triton_rope_kv.py:352-411)."""
    validate_value_inputs(v_quant, v_scale, out)
    require_cuda(v_quant)
    if out is None:
        out = _new_out(v_quant, out_dtype)
    t, h, d = v_quant.shape
    _launch(1, t, h, d, None, None, v_quant, v_scale, None, None, 0.0, None, DEFAULT_THETA, None,
            out, False)
    return out


def dequant_value_ref(
    v_quant: torch.Tensor,
    v_scale: torch.Tensor,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """The reference's eager value dequant (reference.py:283-307) on the CUDA kernel.

    ``fp16(q*s)`` has one rounding of an exact product, so the eager, compiled and Triton
    versions all give the same bits.  CUDA tensors only.
    """
    return dequant_value(v_quant, v_scale, out)


# torch.compile of the eager value dequant (reference.py:318-327): the same bits.
dequant_value_compiled = dequant_value_ref


def dequant_kv_cache(
    k_quant: torch.Tensor,
    k_scale: torch.Tensor,
    v_quant: torch.Tensor,
    v_scale: torch.Tensor,
    cos_delta: torch.Tensor | None = None,
    sin_delta: torch.Tensor | None = None,
    k_out: torch.Tensor | None = None,
    v_out: torch.Tensor | None = None,
    *,
    delta_p: int | torch.Tensor | None = None,
    theta: float = DEFAULT_THETA,
    out_dtype: torch.dtype | None = None,
    fp32_intermediate: bool = True,
) -> tuple[torch.Tensor, torch.Tensor]:
    """K (shifted) and V (plain) in one launch (triton_rope_kv.py:414-427).  Default
    arithmetic: the Triton kernel's (``q*s`` kept in fp32)."""
    validate_key_core(k_quant, k_scale, k_out)
    validate_value_inputs(v_quant, v_scale, v_out)
    cos, sin, dp, dp_dev = _resolve_shift(k_quant, cos_delta, sin_delta, delta_p, theta)
    if cos is not None:
        validate_key_inputs(k_quant, k_scale, cos, sin, k_out)
    require_cuda(k_quant)
    require_cuda(v_quant)
    if k_out is None:
        k_out = _new_out(k_quant, out_dtype if v_out is None else v_out.dtype)
    if v_out is None:
        v_out = _new_out(v_quant, k_out.dtype)
    if k_quant.shape == v_quant.shape and k_out.dtype == v_out.dtype and k_quant.device == v_quant.device:
        t, h, d = k_quant.shape
        _launch(1, t, h, d, k_quant, k_scale, v_quant, v_scale, cos, sin, dp, dp_dev, theta,
                k_out, v_out, fp32_intermediate)
    else:
        t, h, d = k_quant.shape
        _launch(1, t, h, d, k_quant, k_scale, None, None, cos, sin, dp, dp_dev, theta, k_out,
                None, fp32_intermediate)
        t, h, d = v_quant.shape
        _launch(1, t, h, d, None, None, v_quant, v_scale, None, None, 0.0, None, theta, None,
                v_out, False)
    return k_out, v_out


def restore_layers(
    k_quant: torch.Tensor | None,
    k_scale: torch.Tensor | None,
    v_quant: torch.Tensor | None,
    v_scale: torch.Tensor | None,
    *,
    delta_p: float | torch.Tensor = 0,
    theta: float = DEFAULT_THETA,
    k_out: torch.Tensor | None = None,
    v_out: torch.Tensor | None = None,
    out_dtype: torch.dtype = torch.bfloat16,
    fp32_intermediate: bool = False,
    force_generic: bool = False,
) -> tuple[torch.Tensor | None, torch.Tensor | None]:
    """Restore many layers at once: ``[L, T, H, D]`` int8 codes with ``[L, T, H, 1]``
    scales -> ``[L, T, H, D]`` outputs (any strides, e.g. views of ``[L, 1, H, Tmax, D]``
    model-layout caches), every layer shifted by the same ``delta_p``.  One launch.
    """
    ref = k_quant if k_quant is not None else v_quant
    if ref is None:
        raise ValueError("neither K nor V given")
    if ref.ndim != 4:
        raise ValueError(f"expected [L, T, H, D] codes, got shape {tuple(ref.shape)}")
    for q, s in ((k_quant, k_scale), (v_quant, v_scale)):
        if q is None:
            continue
        if q.dtype != torch.int8:
            raise TypeError(f"codes must be torch.int8, got {q.dtype}")
        if q.shape != ref.shape or s is None or s.shape != ref.shape[:3] + (1,):
            raise ValueError("K/V codes and scales must be [L, T, H, D] and [L, T, H, 1]")
        require_cuda(q)
    n_l, t, h, d = ref.shape
    if d % 2 != 0:
        raise ValueError(f"head_dim must be even for RoPE half-pairing, got head_dim={d}")
    dp_dev = None
    dp = 0.0
    if isinstance(delta_p, torch.Tensor):
        if delta_p.numel() != 1:
            raise ValueError("restore_layers takes one shift for all layers")
        if delta_p.is_cuda:
            dp_dev = delta_p.reshape(1).to(device=ref.device, dtype=torch.float32)
        else:
            dp = float(delta_p.reshape(-1)[0].to(torch.float32))
    else:
        dp = float(delta_p)
    if k_quant is not None and k_out is None:
        k_out = torch.empty(ref.shape, dtype=out_dtype, device=ref.device)
    if v_quant is not None and v_out is None:
        v_out = torch.empty(ref.shape, dtype=out_dtype, device=ref.device)
    for o in (k_out, v_out):
        if o is not None and (o.shape != ref.shape or o.device != ref.device):
            raise ValueError(f"outputs must be [L, T, H, D] = {tuple(ref.shape)} on {ref.device}")
    _launch(n_l, t, h, d, k_quant, k_scale, v_quant, v_scale, None, None, dp, dp_dev, theta,
            k_out if k_quant is not None else None, v_out if v_quant is not None else None,
            fp32_intermediate, force_generic)
    return k_out, v_out
