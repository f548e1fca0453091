"""sm_100a kernels of the KV-restore path, under the reference's public names
(speccache/kernels/__init__.py:3-39).

The reference's eager/compiled oracles (``pytorch_eager_dequant_rope_shift``,
``dequant_value_ref``, the ``torch.compile`` variants) are not part of this package:
every name here runs the CUDA library, and there is no CPU path.
"""

from .paged import paged_status, restore_paged
from .quantize import quantize_kv_int8, quantize_symmetric_int8
from .restore import (
    compute_rope_cos_sin_delta,
    dequant_and_rope_key,
    dequant_kv_cache,
    dequant_value,
    restore_layers,
    triton_fused_k_dequant_rope_shift,
)
from .shift import rope_shift_keys
from .validation import rotate_half, validate_key_inputs, validate_value_inputs

# The reference exports its Triton kernel object under this name; here it names the
# fused entry point of the CUDA library that replaces it.
fused_k_dequant_rope_shift_kernel = "sc_dequant_rope_kv"

__all__ = [
    "compute_rope_cos_sin_delta",
    "dequant_and_rope_key",
    "dequant_kv_cache",
    "dequant_value",
    "fused_k_dequant_rope_shift_kernel",
    "paged_status",
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
