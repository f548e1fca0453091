"""KV cache sink and multi-layer injector with the reference's interfaces.

``SpecDynamicCache`` keeps the interface of speccache/serving/kv_injector.py:38-133
(``update``, ``truncate``, ``get_seq_length``, ``to_legacy_cache``, ...) but stores each
layer in a preallocated ``[B, H, capacity, D]`` buffer: ``update`` copies the new tokens
in place instead of re-concatenating the whole layer (kv_injector.py:97-100), ``truncate``
only moves the length (kv_injector.py:104-115), and the restore kernels write straight
into ``append_views`` (the ``[T, H, D] -> [1, H, T, D]`` permute of kv_injector.py:222-232
becomes store addressing).

``MultiLayerKVInjector`` keeps the interface of kv_injector.py:136-498 over a
``KVRestorePipeline``: unified pinned slabs ``[L, blocks, chunk, H, D]`` with one
``PinnedKVPool`` view per layer, and ``reconstruct_and_inject_multi_layer`` restoring every
layer through the C++ pipeline into the cache.
"""

from __future__ import annotations

from collections.abc import Sequence
from typing import Any

import torch

from ..cache.pinned_pool import PinnedKVPool
from ..cache.pipeline import KVRestorePipeline
from ..kernels.restore import dequant_kv_cache
from ..kernels.shift import rope_shift_keys, token_major


class SpecDynamicCache:
    """HF-style per-layer KV cache in ``[batch, heads, seq, head_dim]`` layout."""

    def __init__(self, capacity: int = 0) -> None:
        self._k: list[torch.Tensor | None] = []
        self._v: list[torch.Tensor | None] = []
        self._len: list[int] = []
        self._default_capacity = int(capacity)

    # -- reference interface ----------------------------------------------------------------
    @property
    def key_cache(self) -> list[torch.Tensor | None]:
        return [None if k is None else k[:, :, :n] for k, n in zip(self._k, self._len)]

    @property
    def value_cache(self) -> list[torch.Tensor | None]:
        return [None if v is None else v[:, :, :n] for v, n in zip(self._v, self._len)]

    def __len__(self) -> int:
        return len(self._k)

    def __getitem__(self, layer_idx: int) -> tuple[torch.Tensor, torch.Tensor]:
        n = self._len[layer_idx]
        return self._k[layer_idx][:, :, :n], self._v[layer_idx][:, :, :n]

    def get_seq_length(self, layer_idx: int = 0) -> int:
        if len(self._k) <= layer_idx or self._k[layer_idx] is None:
            return 0
        return self._len[layer_idx]

    def get_max_length(self) -> int:
        return max(self._len) if self._len else 0

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int,
               cache_kwargs: Any | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        """Append ``[B, H, T, D]`` states to the layer; returns the cumulative views."""
        t = key_states.shape[-2]
        k_dst, v_dst = self._append(layer_idx, key_states, t)
        k_dst.copy_(key_states)
        v_dst.copy_(value_states)
        self._len[layer_idx] += t
        return self[layer_idx]

    def truncate(self, max_seq_len: int) -> None:
        for i in range(len(self._len)):
            if self._k[i] is not None and self._len[i] > max_seq_len:
                self._len[i] = max(0, int(max_seq_len))

    def to_legacy_cache(self) -> tuple[tuple[torch.Tensor, torch.Tensor], ...]:
        return tuple(self[i] for i in range(len(self._k)) if self._k[i] is not None)

    @classmethod
    def from_legacy_cache(cls, past_key_values: Sequence[tuple[torch.Tensor, torch.Tensor]]) -> "SpecDynamicCache":
        cache = cls()
        for layer_idx, (k, v) in enumerate(past_key_values):
            cache.update(k, v, layer_idx=layer_idx)
        return cache

    # -- zero-copy appends for the restore kernels -------------------------------------------
    def reserve(self, layer_idx: int, extra_tokens: int, *, batch: int, heads: int, head_dim: int,
                dtype: torch.dtype, device: torch.device) -> None:
        """Make room for ``extra_tokens`` more tokens in the layer (growing geometrically)."""
        while len(self._k) <= layer_idx:
            self._k.append(None)
            self._v.append(None)
            self._len.append(0)
        buf = self._k[layer_idx]
        need = self._len[layer_idx] + int(extra_tokens)
        if buf is not None:
            if buf.shape[0] != batch or buf.shape[1] != heads or buf.shape[3] != head_dim:
                raise ValueError(f"layer {layer_idx} holds [{buf.shape[0]}, {buf.shape[1]}, *, "
                                 f"{buf.shape[3]}], got [{batch}, {heads}, *, {head_dim}]")
            if buf.dtype != dtype or buf.device != device:
                raise ValueError(f"layer {layer_idx} holds {buf.dtype} on {buf.device}")
            if buf.shape[2] >= need:
                return
        cap = max(need, self._default_capacity, 2 * (buf.shape[2] if buf is not None else 0))
        cap = (cap + 15) // 16 * 16
        k_new = torch.empty((batch, heads, cap, head_dim), dtype=dtype, device=device)
        v_new = torch.empty_like(k_new)
        n = self._len[layer_idx]
        if buf is not None and n:
            k_new[:, :, :n].copy_(buf[:, :, :n])
            v_new[:, :, :n].copy_(self._v[layer_idx][:, :, :n])
        self._k[layer_idx], self._v[layer_idx] = k_new, v_new

    def append_views(self, layer_idx: int, n_tokens: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Token-major ``[n_tokens, H, D]`` views of the next tokens of batch row 0, for a
        kernel to write into; call :meth:`commit` once written."""
        start = self._len[layer_idx]
        k = self._k[layer_idx][0, :, start:start + n_tokens].permute(1, 0, 2)
        v = self._v[layer_idx][0, :, start:start + n_tokens].permute(1, 0, 2)
        return k, v

    def commit(self, layer_idx: int, n_tokens: int) -> None:
        self._len[layer_idx] += int(n_tokens)

    def _append(self, layer_idx: int, like: torch.Tensor, t: int):
        b, h, _, d = like.shape
        self.reserve(layer_idx, t, batch=b, heads=h, head_dim=d, dtype=like.dtype, device=like.device)
        start = self._len[layer_idx]
        return (self._k[layer_idx][:, :, start:start + t], self._v[layer_idx][:, :, start:start + t])


class MultiLayerKVInjector:
    """Layer-wise pinned pools over one restore pipeline (kv_injector.py:136-215)."""

    def __init__(self, num_layers: int, num_kv_heads: int, head_dim: int,
                 device: torch.device | None = None, max_blocks: int = 128, chunk_size: int = 64,
                 *, theta: float = 10000.0, out_dtype: torch.dtype = torch.float16,
                 n_slots: int = 2) -> None:
        self.num_layers, self.num_kv_heads, self.head_dim = num_layers, num_kv_heads, head_dim
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if self.device.type != "cuda":
            raise RuntimeError(f"MultiLayerKVInjector needs a CUDA device, got {self.device}")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.chunk_size, self.max_blocks = chunk_size, max_blocks
        self.theta, self.out_dtype = theta, out_dtype
        self.pipeline = KVRestorePipeline(num_layers, max_blocks, chunk_size, num_kv_heads, head_dim,
                                          device=self.device, n_slots=n_slots)
        self.unified_k_quant, self.unified_k_scale = self.pipeline.k_quant, self.pipeline.k_scale
        self.unified_v_quant, self.unified_v_scale = self.pipeline.v_quant, self.pipeline.v_scale
        self.layer_pools = [PinnedKVPool(max_blocks, chunk_size, num_kv_heads, head_dim,
                                         pipeline=self.pipeline, layer=layer)
                            for layer in range(num_layers)]

    @staticmethod
    def format_to_model_layout(x: torch.Tensor) -> torch.Tensor:
        """``[T, H, D] -> [1, H, T, D]`` (kv_injector.py:222-232)."""
        if x.ndim == 3:
            return x.permute(1, 0, 2).unsqueeze(0).contiguous()
        if x.ndim == 4:
            return x
        raise ValueError(f"Unexpected tensor ndim={x.ndim}, expected 3 or 4.")

    @staticmethod
    def format_to_engine_layout(x: torch.Tensor) -> torch.Tensor:
        """``[1, H, T, D] -> [T, H, D]`` (kv_injector.py:234-244)."""
        if x.ndim == 4:
            return x.squeeze(0).permute(1, 0, 2).contiguous()
        if x.ndim == 3:
            return x
        raise ValueError(f"Unexpected tensor ndim={x.ndim}, expected 3 or 4.")

    def apply_rope_shift(self, k_fp16: torch.Tensor, delta_p: int) -> torch.Tensor:
        """Rotate dequantised keys (``[T, H, D]`` or ``[1, H, T, D]``, float16/bfloat16) by
        ``delta_p``; same layout and dtype, a zero shift returns ``k_fp16`` itself
        (kv_injector.py:246-283).  One kernel launch, no layout copies."""
        if delta_p == 0:
            return k_fp16
        return rope_shift_keys(k_fp16, delta_p, theta=self.theta)

    def inject_layer_kv(self, cache: SpecDynamicCache, layer_idx: int, k_tensor: torch.Tensor,
                        v_tensor: torch.Tensor, delta_p: int = 0) -> None:
        """Append ``[T, H, D]`` or ``[1, H, T, D]`` keys/values to a cache layer, keys shifted
        by ``delta_p`` (kv_injector.py:285-301).  The shift kernel writes straight into the
        cache's next slots; without a shift the tokens are copied there."""
        if k_tensor.ndim == 4 and k_tensor.shape[0] != 1 and delta_p == 0:
            cache.update(k_tensor, v_tensor, layer_idx=layer_idx)  # batched model layout
            return
        kt, vt = token_major(k_tensor), token_major(v_tensor)
        if kt.shape != vt.shape or kt.dtype != vt.dtype or kt.device != vt.device:
            raise ValueError(f"keys {tuple(kt.shape)} {kt.dtype} and values {tuple(vt.shape)} "
                             f"{vt.dtype} differ")
        t, h, d = kt.shape
        cache.reserve(layer_idx, t, batch=1, heads=h, head_dim=d, dtype=kt.dtype, device=kt.device)
        k_dst, v_dst = cache.append_views(layer_idx, t)
        if delta_p != 0:
            rope_shift_keys(kt, delta_p, theta=self.theta, out=k_dst)
        else:
            k_dst.copy_(kt)
        v_dst.copy_(vt)
        cache.commit(layer_idx, t)

    def inject_multi_layer(self, cache: SpecDynamicCache, layer_k_list: Sequence[torch.Tensor],
                           layer_v_list: Sequence[torch.Tensor], delta_p: int = 0) -> None:
        """:meth:`inject_layer_kv` for every layer (kv_injector.py:303-322)."""
        if len(layer_k_list) != len(layer_v_list):
            raise ValueError(f"Mismatch in layer counts: {len(layer_k_list)} keys vs "
                             f"{len(layer_v_list)} values")
        for layer_idx, (k, v) in enumerate(zip(layer_k_list, layer_v_list, strict=True)):
            self.inject_layer_kv(cache, layer_idx, k, v, delta_p=delta_p)

    def reconstruct_layer_chunk(self, layer_idx: int, block_id: int, delta_p: int,
                                cos_delta: torch.Tensor | None = None,
                                sin_delta: torch.Tensor | None = None,
                                transfer_stream: torch.cuda.Stream | None = None):
        """One block of one layer: H2D of its codes and the fused restore (kv_injector.py:324-390)."""
        kq_h, ks_h, vq_h, vs_h = self.layer_pools[layer_idx].get_block_views(block_id)
        stream = transfer_stream or torch.cuda.current_stream(self.device)
        with torch.cuda.stream(stream):
            dev = [x.to(self.device, non_blocking=True) for x in (kq_h, ks_h, vq_h, vs_h)]
        if stream != torch.cuda.current_stream(self.device):
            torch.cuda.current_stream(self.device).wait_stream(stream)
            for x in dev:
                x.record_stream(torch.cuda.current_stream(self.device))
        # The eager arithmetic (fp16 intermediate), like every restore path of the injector.
        return dequant_kv_cache(*dev, cos_delta, sin_delta, delta_p=delta_p if cos_delta is None else None,
                                theta=self.theta, out_dtype=self.out_dtype, fp32_intermediate=False)

    def reconstruct_and_inject_multi_layer(self, cache: SpecDynamicCache, block_ids: list[int],
                                           delta_ps: list[int]):
        """Restore ``block_ids`` (block i shifted by ``delta_ps[i]``) for every layer straight
        into ``cache`` (kv_injector.py:392-498); returns ``cache.to_legacy_cache()``."""
        if not block_ids:
            return cache.to_legacy_cache()
        n_tok = len(block_ids) * self.chunk_size
        k_views, v_views = [], []
        for layer in range(self.num_layers):
            cache.reserve(layer, n_tok, batch=1, heads=self.num_kv_heads, head_dim=self.head_dim,
                          dtype=self.out_dtype, device=self.device)
            k, v = cache.append_views(layer, n_tok)
            k_views.append(k)
            v_views.append(v)
        for pool in self.layer_pools:
            for b in block_ids:
                pool.touch(b)
        self.pipeline.restore(block_ids, delta_ps, k_views, v_views, theta=self.theta)
        for layer in range(self.num_layers):
            cache.commit(layer, n_tok)
        return cache.to_legacy_cache()

    def offload_multi_layer(self, block_ids: list[int], layer_k: Sequence[torch.Tensor],
                            layer_v: Sequence[torch.Tensor]) -> None:
        """Quantize each layer's ``[n*chunk, H, D]`` K/V on the GPU into the pinned slabs (the
        runner's cold-miss offload, speccache/serving/pipeline.py:506-524, for every layer)."""
        for layer, (k, v) in enumerate(zip(layer_k, layer_v, strict=True)):
            self.pipeline.offload(layer, block_ids, k, v)

    def close(self) -> None:
        self.pipeline.close()


KVInjector = MultiLayerKVInjector
