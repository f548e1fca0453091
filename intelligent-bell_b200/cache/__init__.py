"""Host-side restore machinery: pinned slabs and the multi-layer H2D pipeline."""

from .pipeline import KVRestorePipeline

__all__ = ["KVRestorePipeline"]
