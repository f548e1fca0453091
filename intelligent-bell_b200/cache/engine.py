"""Routing-decision front end of the restore pipeline.

The reference engine routes each prompt chunk (radix tree, then semantic index) and hands
the reusable chunks, as ``ChunkRoutingDecision`` records, to ``execute_async_dma_and_rope``
(speccache/cache/engine.py:441-601).  That loop stages one chunk at a time into two device
slots and launches a key kernel and a value kernel per chunk.  The routing indexes are
control plane and stay outside this package; this module keeps the decision records
(engine.py:45-68) as the input format and replaces the loop: the reusable decisions become
one pipeline restore, in which runs of consecutive block ids travel as one copy each and
one kernel per layer restores every block with its own ``delta_p``.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from enum import Enum

import torch

from .pinned_pool import PinnedKVPool


class ChunkRoutingStatus(str, Enum):
    """Routing state of a prompt chunk (engine.py:45-51)."""

    EXACT_REUSE = "EXACT_REUSE"
    SEMANTIC_REUSE = "SEMANTIC_REUSE"
    SPECULATIVE_DRAFT = "SPECULATIVE_DRAFT"
    CACHE_MISS = "CACHE_MISS"


@dataclass
class ChunkRoutingDecision:
    """Routing decision and transfer metadata of one prompt chunk (engine.py:54-67)."""

    chunk_index: int
    target_start_pos: int
    target_end_pos: int
    token_ids: tuple[int, ...]
    status: ChunkRoutingStatus
    similarity: float = 0.0
    block_id: int | None = None
    cached_position: int | None = None
    delta_p: int = 0
    continuation_tokens: list[int] = field(default_factory=list)


_REUSE = (ChunkRoutingStatus.EXACT_REUSE, ChunkRoutingStatus.SEMANTIC_REUSE)


def reusable(decisions) -> list[ChunkRoutingDecision]:
    """Decisions whose block is restored: exact or semantic reuse with a block id
    (engine.py:449-454), in their given order."""
    return [d for d in decisions if d.status in _REUSE and d.block_id is not None]


class RestoreEngine:
    """The engine's pool and DMA + RoPE step, fed by routing decisions.

    Args mirror ``SpecCacheEngine`` (engine.py:71-85) for the parts on this path:
    ``chunk_size``, ``num_kv_heads``, ``head_dim``, ``max_blocks``, ``device``.  ``pool`` may
    be an existing pipeline-backed ``PinnedKVPool``; ``theta`` is the RoPE base of the shifts
    (the reference fixes 10000).
    """

    def __init__(self, chunk_size: int = 128, num_kv_heads: int = 8, head_dim: int = 128,
                 max_blocks: int = 1024, device: torch.device | str | int | None = None, *,
                 pool: PinnedKVPool | None = None, theta: float = 10000.0) -> None:
        if pool is None:
            pool = PinnedKVPool(max_blocks=max_blocks, chunk_size=chunk_size,
                                num_heads=num_kv_heads, head_dim=head_dim, device=device)
            self._owns_pool = True
        else:
            self._owns_pool = False
        self.pool = pool
        self.chunk_size, self.num_kv_heads, self.head_dim = pool.chunk_size, pool.num_heads, pool.head_dim
        self.max_blocks = pool.max_blocks
        self.theta = float(theta)

    @property
    def device(self) -> torch.device:
        """The GPU the restores write to (the pool's pipeline device)."""
        if self.pool.pipeline is not None:
            return self.pool.pipeline.device
        return torch.device("cuda", torch.cuda.current_device())

    def register_chunk(self, token_ids, cached_position: int, k_quant: torch.Tensor,
                       k_scale: torch.Tensor, v_quant: torch.Tensor, v_scale: torch.Tensor,
                       embedding=None, continuation_tokens=None) -> int:
        """Store a quantized chunk in the pool (engine.py:186-228); returns its block id.

        ``embedding`` and ``continuation_tokens`` feed the reference's routing indexes, which
        are not part of this package; they are accepted and ignored.
        """
        tokens = tuple(token_ids)
        if len(tokens) != self.chunk_size:
            raise ValueError(
                f"token_ids length ({len(tokens)}) must equal chunk_size ({self.chunk_size}).")
        block_id = self.pool.allocate()
        self.pool.write_block(block_id=block_id, k_q=k_quant, k_s=k_scale, v_q=v_quant,
                              v_s=v_scale, start_pos=cached_position, token_ids=tokens)
        return block_id

    def execute_async_dma_and_rope(self, reused_decisions, dest_k_out: torch.Tensor | None = None,
                                   dest_v_out: torch.Tensor | None = None, sync: bool = True):
        """Restore the reusable decisions' blocks into ``[n*chunk, H, D]`` GPU caches, block i
        shifted by its ``delta_p``; returns ``(K, V)`` (engine.py:441-601).

        With no reusable decision the result is two empty float16 ``[0, H, D]`` tensors
        (engine.py:456-460).  ``dest_k_out``/``dest_v_out`` are written in place (float16, as
        the reference, or bfloat16).  With ``sync=False`` nothing blocks: the results are
        ordered on the current CUDA stream, and ``pool.pipeline.synchronize()`` waits for them.
        """
        valid = reusable(reused_decisions)
        if not valid:
            empty = torch.empty((0, self.num_kv_heads, self.head_dim), dtype=torch.float16,
                                device=self.device)
            return empty, empty
        out_dtype = dest_k_out.dtype if dest_k_out is not None else torch.float16
        return self.pool.execute_async_dma_and_rope(
            [int(d.block_id) for d in valid], [int(d.delta_p) for d in valid], dest_k_out,
            dest_v_out, sync=sync, theta=self.theta, out_dtype=out_dtype)

    def close(self) -> None:
        if self._owns_pool:
            self.pool.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc) -> None:
        self.close()
