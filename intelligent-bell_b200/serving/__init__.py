"""Cache sink and multi-layer injector over the restore pipeline."""

from .kv_injector import KVInjector, MultiLayerKVInjector, SpecDynamicCache

__all__ = ["KVInjector", "MultiLayerKVInjector", "SpecDynamicCache"]
