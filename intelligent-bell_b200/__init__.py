"""speccache-b200: SpecCache Path-1 KV restore on B200 (sm_100a).

The reference's kernel API (``speccache.kernels``) on hand-written CUDA kernels behind
the C ABI of ``libspeccache_b200.so`` (declared in ``include/speccache_b200.h``):

* ``triton_fused_k_dequant_rope_shift`` / ``dequant_value`` / ``dequant_kv_cache`` —
  INT8 K dequant + relative RoPE shift and V dequant (and the reference's eager ``*_ref`` and
  compiled ``*_compiled`` names on the same kernels);
* ``quantize_kv_int8`` — the bit-exact offload twin;
* ``compute_rope_cos_sin_delta`` — shift tables;
* ``restore_paged`` — ragged, paged gather + restore in one launch;
* ``restore_layers`` — many layers in one launch;
* ``cache.KVRestorePipeline`` — pinned-host -> GPU multi-layer restore.

The directory name is not a Python identifier; import it with
``importlib.import_module("intelligent-bell_b200")`` (it also registers the alias
``speccache_b200`` in ``sys.modules``).
"""

import sys as _sys

from . import _lib
from ._build import LIB_PATH, build_library
from .kernels import (
    compute_rope_cos_sin_delta,
    dequant_and_rope_key,
    dequant_and_rope_key_compiled,
    dequant_and_rope_key_ref,
    dequant_kv_cache,
    dequant_value,
    dequant_value_compiled,
    dequant_value_ref,
    fused_k_dequant_rope_shift_kernel,
    paged_status,
    pytorch_compiled_dequant_rope_shift,
    pytorch_eager_dequant_rope_shift,
    quantize_kv_int8,
    quantize_symmetric_int8,
    restore_layers,
    restore_paged,
    rope_shift_keys,
    rotate_half,
    triton_fused_k_dequant_rope_shift,
    validate_key_inputs,
    validate_value_inputs,
)

__version__ = "0.1.0"


def preload(device=None) -> None:
    """Load every kernel of the library on ``device`` (default: the current device) now.

    CUDA loads a kernel's module at its first launch, and that load waits for the device to
    go idle: a first call enqueued behind running work would block until the work ends.  Call
    this once per GPU at start-up (``KVRestorePipeline`` does it for its own kernels).
    """
    import torch

    lib = _lib.load()
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        _lib.check(lib.sc_preload_kernels(), "sc_preload_kernels")

_sys.modules.setdefault("speccache_b200", _sys.modules[__name__])

__all__ = [
    "LIB_PATH",
    "build_library",
    "preload",
    "compute_rope_cos_sin_delta",
    "dequant_and_rope_key",
    "dequant_and_rope_key_compiled",
    "dequant_and_rope_key_ref",
    "dequant_kv_cache",
    "dequant_value",
    "dequant_value_compiled",
    "dequant_value_ref",
    "fused_k_dequant_rope_shift_kernel",
    "paged_status",
    "pytorch_compiled_dequant_rope_shift",
    "pytorch_eager_dequant_rope_shift",
    "quantize_kv_int8",
    "quantize_symmetric_int8",
    "restore_layers",
    "restore_paged",
    "rope_shift_keys",
    "rotate_half",
    "triton_fused_k_dequant_rope_shift",
    "validate_key_inputs",
    "validate_value_inputs",
]
