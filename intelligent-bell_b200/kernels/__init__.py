"""sm_100a kernels of the KV-restore path, under the reference's public names
(speccache/kernels/__init__.py:3-39: all fifteen of them, plus additive extensions).

Every name here runs the CUDA library and there is no CPU path: the reference's eager
(``*_ref``) and ``torch.compile`` (``*_compiled``) entry points run the same kernels with
the arithmetic of the function they replace (fp16 or fp32 intermediate of ``q*s``).
"""

from .paged import paged_status, restore_paged
from .quantize import quantize_kv_int8, quantize_symmetric_int8
from .restore import (
    compute_rope_cos_sin_delta,
    dequant_and_rope_key,
    dequant_and_rope_key_compiled,
    dequant_and_rope_key_ref,
    dequant_kv_cache,
    dequant_value,
    dequant_value_compiled,
    dequant_value_ref,
    pytorch_compiled_dequant_rope_shift,
    pytorch_eager_dequant_rope_shift,
    restore_layers,
    triton_fused_k_dequant_rope_shift,
)
from .shift import rope_shift_keys
from .validation import rotate_half, validate_key_inputs, validate_value_inputs


class _FusedKernelHandle:
    """Stands where the reference exports its Triton kernel object
    (``fused_k_dequant_rope_shift_kernel``, triton_rope_kv.py:42-170).

    The kernel behind it is the library's CUDA entry point ``sc_dequant_rope_kv``, which is
    not launched Triton-style: indexing it with a grid or calling it raises ``TypeError``
    with that explanation instead of an unrelated error.  Call
    ``triton_fused_k_dequant_rope_shift`` (or ``sc_dequant_rope_kv`` through the C ABI).
    """

    __slots__ = ()
    entry_point = "sc_dequant_rope_kv"
    library = "libspeccache_b200.so"

    def _refuse(self):
        raise TypeError(
            "fused_k_dequant_rope_shift_kernel is the CUDA kernel behind sc_dequant_rope_kv "
            "(libspeccache_b200.so), not a Triton kernel: it cannot be launched with "
            "kernel[grid](...); call triton_fused_k_dequant_rope_shift(...) instead")

    def __getitem__(self, grid):
        self._refuse()

    def __call__(self, *args, **kwargs):
        self._refuse()

    def __repr__(self) -> str:
        return f"<CUDA kernel {self.entry_point} in {self.library}>"


fused_k_dequant_rope_shift_kernel = _FusedKernelHandle()

__all__ = [
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
