"""An op set with the product module's API, computed by the CPU oracle.

Injected into ``KVCacheAdapter(native_ext=...)`` and
``InMemoryBlockStoreBackend(ops=...)`` by the CPU tests, so the adapter's
orchestration (which ops it calls, in which order, with which arguments) is
checked against fixtures recorded from the reference, without a GPU.
"""
from __future__ import annotations

import torch

import oracle
from oracle import moves
from kv_cache_adapter_b200.errors import InsufficientCapacityError


def _translate(fn, *args, **kwargs):
    try:
        return fn(*args, **kwargs)
    except oracle.OracleInsufficientCapacity as exc:
        raise InsufficientCapacityError(str(exc)) from None
    except oracle.OracleBadIndex as exc:
        raise IndexError(str(exc)) from None


class OracleOps:
    calls: list[str]

    def __init__(self) -> None:
        self.calls = []

    def inspect_load_requests(self, l2p, slot_meta, ids, check=None):
        self.calls.append("inspect_load_requests")
        return list(_translate(oracle.inspect_load_requests, l2p, slot_meta, ids))

    def inspect_save_requests(self, l2p, slot_meta, ids, check=None):
        self.calls.append("inspect_save_requests")
        return list(_translate(oracle.inspect_save_requests, l2p, slot_meta, ids))

    def pop_reusable_slots(self, slot_meta, search_start, blocked, count, order=None, check=True):
        self.calls.append("pop_reusable_slots")
        return _translate(oracle.pop_reusable_slots, slot_meta, search_start, blocked, count,
                          order=order or "grouped")

    def commit_load_metadata(self, *args, check=None):
        self.calls.append("commit_load_metadata")
        _translate(oracle.commit_load_metadata, *args)

    def commit_save_metadata(self, *args, check=None):
        self.calls.append("commit_save_metadata")
        _translate(oracle.commit_save_metadata, *args)

    def release_metadata(self, l2p, slot_meta, ids, check=None):
        self.calls.append("release_metadata")
        _translate(oracle.release_metadata, l2p, slot_meta, ids)

    def gather_blocks(self, actual_blocks, slot_ids, out=None, check=None):
        self.calls.append("gather_blocks")
        return moves.gather_blocks(actual_blocks, slot_ids)

    def scatter_blocks(self, actual_blocks, slot_ids, block_data, skip_negative=False, check=None):
        self.calls.append("scatter_blocks")
        if skip_negative:
            keep = slot_ids >= 0
            slot_ids, block_data = slot_ids[keep], block_data[keep]
        moves.scatter_blocks(actual_blocks, slot_ids, block_data)

    def copy_blocks(self, src, src_ids, dst, dst_ids, check=None):
        self.calls.append("copy_blocks")
        moves.copy_blocks(src, src_ids, dst, dst_ids)

    def gather_layers(self, caches, slot_ids, out=None, blocks_per_chunk=None, check=None):
        self.calls.append("gather_layers")
        got = moves.gather_layers(list(caches), slot_ids, blocks_per_chunk=blocks_per_chunk)
        if out is None:
            return got
        out.copy_(got)
        return out

    def scatter_layers(self, caches, slot_ids, chunks, blocks_per_chunk=None, check=None):
        self.calls.append("scatter_layers")
        moves.scatter_layers(list(caches), slot_ids, chunks, blocks_per_chunk=blocks_per_chunk)

    def gather_tokens(self, caches, slot_mapping, out=None, tokens_per_chunk=None, check=None):
        self.calls.append("gather_tokens")
        got = moves.gather_tokens(list(caches), slot_mapping, tokens_per_chunk=tokens_per_chunk)
        if out is None:
            return got
        out.copy_(got)
        return out

    def scatter_tokens(self, caches, slot_mapping, chunks, tokens_per_chunk=None, check=None):
        self.calls.append("scatter_tokens")
        moves.scatter_tokens(list(caches), slot_mapping, chunks, tokens_per_chunk=tokens_per_chunk)
