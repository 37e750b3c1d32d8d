"""B200-native (sm_100a) hot path of kv_cache_adapter.

``KVCacheAdapter`` / ``InMemoryBlockStoreBackend`` keep the reference's
public API (its package __init__.py:1-19); the clock sweep, slot metadata
updates and KV block/token moves run in the CUDA kernels of
``libkvca_b200.so`` (C ABI: include/kvca.h), reached through
``kv_cache_adapter_b200.kv_cache_adapter_cuda``.
"""
from .adapter import (
    BlockStoreBackend,
    HostTierBackend,
    InMemoryBlockStoreBackend,
    KVCacheAdapter,
)
from .errors import BlockNotFoundError, InsufficientCapacityError, KVCacheAdapterError

__all__ = [
    "BlockNotFoundError",
    "BlockStoreBackend",
    "HostTierBackend",
    "InMemoryBlockStoreBackend",
    "InsufficientCapacityError",
    "KVCacheAdapter",
    "KVCacheAdapterError",
]
