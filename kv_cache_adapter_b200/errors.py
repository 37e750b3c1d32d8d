"""Exception types of the adapter API (same hierarchy as adapter.py:50-59 of
the reference, so callers' ``except`` clauses keep working)."""
from __future__ import annotations


class KVCacheAdapterError(RuntimeError):
    pass


class BlockNotFoundError(KVCacheAdapterError):
    pass


class InsufficientCapacityError(KVCacheAdapterError):
    pass
