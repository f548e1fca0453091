"""Host-side restore machinery: pinned slabs, the pool interface and the H2D pipeline."""

from .engine import ChunkRoutingDecision, ChunkRoutingStatus, RestoreEngine, reusable
from .peer import HeadShardGather, SharedBuffer
from .pinned_pool import BlockMetadata, OriginalPositionMetadata, PinnedHostPool, PinnedKVPool
from .pipeline import KVRestorePipeline
from .sharding import head_shard, shard_view

__all__ = ["BlockMetadata", "ChunkRoutingDecision", "ChunkRoutingStatus", "HeadShardGather",
           "KVRestorePipeline", "OriginalPositionMetadata", "PinnedHostPool", "PinnedKVPool",
           "RestoreEngine", "SharedBuffer", "head_shard", "reusable", "shard_view"]
