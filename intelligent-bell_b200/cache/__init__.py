"""Host-side restore machinery: pinned slabs, the pool interface and the H2D pipeline."""

from .peer import HeadShardGather, SharedBuffer
from .pinned_pool import BlockMetadata, OriginalPositionMetadata, PinnedHostPool, PinnedKVPool
from .pipeline import KVRestorePipeline
from .sharding import head_shard, shard_view

__all__ = ["BlockMetadata", "HeadShardGather", "KVRestorePipeline", "OriginalPositionMetadata",
           "PinnedHostPool", "PinnedKVPool", "SharedBuffer", "head_shard", "shard_view"]
