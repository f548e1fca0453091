"""Host-side restore machinery: pinned slabs, the pool interface and the H2D pipeline."""

from .pinned_pool import BlockMetadata, OriginalPositionMetadata, PinnedHostPool, PinnedKVPool
from .pipeline import KVRestorePipeline

__all__ = ["BlockMetadata", "KVRestorePipeline", "OriginalPositionMetadata", "PinnedHostPool",
           "PinnedKVPool"]
