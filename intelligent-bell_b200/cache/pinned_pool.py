"""Pinned host slab pool with the reference's ``PinnedKVPool`` interface.

Mirrors speccache/cache/pinned_pool.py:42-527: the same constructor arguments, slab
attributes (``k_quant``, ``k_scale``, ``v_quant``, ``v_scale``, ``original_start_pos``),
slot allocation with LRU eviction and eviction callback, ``write_block`` checks and error
messages, zero-copy block views and coalesced views.  Differences:

* Without caller-given slabs the pool is one layer of a ``KVRestorePipeline``: its slabs
  are page-locked by the library (``cudaHostAlloc``, allocated from a thread bound to the
  GPU's NUMA node), and ``execute_async_dma_and_rope`` restores blocks to the GPU through
  the pipeline (one copy per run of consecutive block ids, restore kernel per layer) in
  place of the per-chunk Python loop of speccache/cache/engine.py:441-601.
* The slot bookkeeping (which block is free, LRU order) is host policy, kept small.
"""

from __future__ import annotations

import time
from collections import OrderedDict
from collections.abc import Callable
from dataclasses import dataclass, field

import torch


@dataclass
class OriginalPositionMetadata:
    """Metadata of one cached block (pinned_pool.py:27-35)."""

    block_id: int
    start_pos: int
    token_ids: tuple[int, ...] = field(default_factory=tuple)
    created_at: float = field(default_factory=time.time)
    last_accessed: float = field(default_factory=time.time)


BlockMetadata = OriginalPositionMetadata


class PinnedKVPool:
    """Page-locked host slabs ``[max_blocks, chunk, H, D]`` int8 + ``[..., 1]`` fp16."""

    def __init__(
        self,
        max_blocks: int,
        chunk_size: int,
        num_heads: int,
        head_dim: int,
        on_evict_callback: Callable[[int], None] | None = None,
        k_quant_slab: torch.Tensor | None = None,
        k_scale_slab: torch.Tensor | None = None,
        v_quant_slab: torch.Tensor | None = None,
        v_scale_slab: torch.Tensor | None = None,
        *,
        device: torch.device | str | int | None = None,
        pipeline=None,
        layer: int = 0,
    ) -> None:
        if max_blocks <= 0:
            raise ValueError(f"max_blocks must be positive, got {max_blocks}")
        if chunk_size <= 0:
            raise ValueError(f"chunk_size must be positive, got {chunk_size}")
        self.max_blocks, self.chunk_size = int(max_blocks), int(chunk_size)
        self.num_heads, self.head_dim = int(num_heads), int(head_dim)
        self.on_evict_callback = on_evict_callback
        self.pipeline, self.layer = pipeline, int(layer)
        self._owns_pipeline = False
        codes = (self.max_blocks, self.chunk_size, self.num_heads, self.head_dim)
        scales = codes[:3] + (1,)
        if k_quant_slab is None and pipeline is None:
            from .pipeline import KVRestorePipeline

            self.pipeline = KVRestorePipeline(1, self.max_blocks, self.chunk_size,
                                              self.num_heads, self.head_dim, device=device)
            self._owns_pipeline = True
        if k_quant_slab is None:
            p = self.pipeline
            self.k_quant, self.k_scale = p.k_quant[self.layer], p.k_scale[self.layer]
            self.v_quant, self.v_scale = p.v_quant[self.layer], p.v_scale[self.layer]
            self._is_pinned = True
        else:
            self.k_quant = k_quant_slab
            self.k_scale = k_scale_slab if k_scale_slab is not None else torch.empty(scales, dtype=torch.float16)
            self.v_quant = v_quant_slab if v_quant_slab is not None else torch.empty(codes, dtype=torch.int8)
            self.v_scale = v_scale_slab if v_scale_slab is not None else torch.empty(scales, dtype=torch.float16)
            self._is_pinned = self.pipeline is not None or bool(getattr(self.k_quant, "is_pinned", lambda: False)())
        self.original_start_pos = torch.full((self.max_blocks,), -1, dtype=torch.long)
        self._free_block_ids: list[int] = list(range(self.max_blocks))
        self._active_lru: OrderedDict[int, OriginalPositionMetadata] = OrderedDict()

    # -- bookkeeping (pinned_pool.py:205-273, 504-527) -------------------------------------
    @property
    def is_pinned(self) -> bool:
        return self._is_pinned

    @property
    def allocated_count(self) -> int:
        return len(self._active_lru)

    @property
    def free_count(self) -> int:
        return len(self._free_block_ids)

    @property
    def allocated_blocks(self) -> list[int]:
        return list(self._active_lru.keys())

    def allocate(self, block_id: int | None = None, start_pos: int = -1) -> int:
        if block_id is not None:
            if block_id in self._free_block_ids:
                self._free_block_ids.remove(block_id)
        elif self._free_block_ids:
            block_id = self._free_block_ids.pop()
        else:
            block_id, _ = self._active_lru.popitem(last=False)
            if self.on_evict_callback is not None:
                self.on_evict_callback(block_id)
        self._active_lru[block_id] = OriginalPositionMetadata(block_id=block_id, start_pos=start_pos)
        return block_id

    def touch(self, block_id: int) -> None:
        meta = self._active_lru.get(block_id)
        if meta is not None:
            meta.last_accessed = time.time()
            self._active_lru.move_to_end(block_id)

    def get_start_pos(self, block_id: int) -> int:
        if block_id not in self._active_lru:
            raise KeyError(f"Block ID {block_id} is not an allocated active block.")
        return int(self.original_start_pos[block_id].item())

    def free(self, block_id: int) -> None:
        if block_id in self._active_lru:
            del self._active_lru[block_id]
            self.original_start_pos[block_id] = -1
            self._free_block_ids.append(block_id)
            if self.on_evict_callback is not None:
                self.on_evict_callback(block_id)

    def clear(self) -> None:
        for bid in list(self._active_lru.keys()):
            if self.on_evict_callback is not None:
                self.on_evict_callback(bid)
        self._active_lru.clear()
        self.original_start_pos.fill_(-1)
        self._free_block_ids = list(range(self.max_blocks))

    # -- slab access (pinned_pool.py:275-464) -----------------------------------------------
    def write_block(self, block_id: int, k_q=None, k_s=None, v_q=None, v_s=None,
                    start_pos: int = -1, token_ids: tuple[int, ...] | None = None, *,
                    k_quant=None, k_scale=None, v_quant=None, v_scale=None) -> None:
        if block_id not in self._active_lru:
            raise KeyError(f"Block ID {block_id} is not an allocated active block.")
        kq = k_q if k_q is not None else k_quant
        ks = k_s if k_s is not None else k_scale
        vq = v_q if v_q is not None else v_quant
        vs = v_s if v_s is not None else v_scale
        if kq is None or ks is None or vq is None or vs is None:
            raise ValueError("Quantized key/value and scale factor tensors must be provided.")
        kv_shape = (self.chunk_size, self.num_heads, self.head_dim)
        s_shape = (self.chunk_size, self.num_heads, 1)
        for name, t, shape, dtype in (("k_q", kq, kv_shape, torch.int8), ("k_s", ks, s_shape, torch.float16),
                                      ("v_q", vq, kv_shape, torch.int8), ("v_s", vs, s_shape, torch.float16)):
            if tuple(t.shape) != shape or t.dtype != dtype:
                raise ValueError(f"{name} shape {t.shape} dtype {t.dtype} invalid.")
        self.k_quant[block_id].copy_(kq)
        self.k_scale[block_id].copy_(ks)
        self.v_quant[block_id].copy_(vq)
        self.v_scale[block_id].copy_(vs)
        self.original_start_pos[block_id] = start_pos
        meta = self._active_lru[block_id]
        meta.start_pos = start_pos
        if token_ids is not None:
            meta.token_ids = token_ids
        self.touch(block_id)

    def get_block_views(self, block_id: int):
        if block_id not in self._active_lru:
            raise KeyError(f"Block ID {block_id} is not an allocated active block.")
        self.touch(block_id)
        return self.k_quant[block_id], self.k_scale[block_id], self.v_quant[block_id], self.v_scale[block_id]

    def get_coalesced_views(self, block_ids: list[int]):
        """Host views ``[n*chunk, H, D]``: zero-copy for consecutive ids, else a gathered
        copy (the GPU restore never needs it: the pipeline copies runs directly)."""
        if not block_ids:
            e_kv = torch.empty((0, self.num_heads, self.head_dim), dtype=torch.int8)
            e_s = torch.empty((0, self.num_heads, 1), dtype=torch.float16)
            return e_kv, e_s, e_kv, e_s
        for b in block_ids:
            self.touch(b)
        n_tok = len(block_ids) * self.chunk_size
        if all(block_ids[i] == block_ids[0] + i for i in range(len(block_ids))):
            sl = slice(block_ids[0], block_ids[-1] + 1)
            return tuple(x[sl].reshape(n_tok, self.num_heads, -1)
                         for x in (self.k_quant, self.k_scale, self.v_quant, self.v_scale))
        idx = torch.as_tensor(block_ids, dtype=torch.long)
        return tuple(x.index_select(0, idx).reshape(n_tok, self.num_heads, -1)
                     for x in (self.k_quant, self.k_scale, self.v_quant, self.v_scale))

    # -- GPU restore (engine.py:441-601) ----------------------------------------------------
    def execute_async_dma_and_rope(self, block_ids: list[int], delta_ps: list[int],
                                   dest_k_out: torch.Tensor | None = None,
                                   dest_v_out: torch.Tensor | None = None, *, sync: bool = True,
                                   theta: float = 10000.0,
                                   out_dtype: torch.dtype = torch.float16):
        """Restore ``block_ids`` (block i shifted by ``delta_ps[i]``) into ``[n*chunk, H, D]``
        GPU tensors through the pipeline; returns ``(K, V)``."""
        if self.pipeline is None or self.pipeline.num_layers != 1:
            raise RuntimeError("execute_async_dma_and_rope needs a single-layer pool backed by "
                               "a KVRestorePipeline (construct the pool without slabs)")
        for b in block_ids:
            self.touch(b)
        n_tok = len(block_ids) * self.chunk_size
        dev = self.pipeline.device
        shape = (n_tok, self.num_heads, self.head_dim)
        if dest_k_out is None:
            dest_k_out = torch.empty(shape, dtype=out_dtype, device=dev)
        if dest_v_out is None:
            dest_v_out = torch.empty(shape, dtype=dest_k_out.dtype, device=dev)
        if n_tok:
            self.pipeline.restore(block_ids, delta_ps, [dest_k_out], [dest_v_out], theta=theta)
            if sync:
                self.pipeline.synchronize()
        return dest_k_out, dest_v_out

    def close(self) -> None:
        if self._owns_pipeline and self.pipeline is not None:
            self.pipeline.close()
            self.pipeline = None


PinnedHostPool = PinnedKVPool
