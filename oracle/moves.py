"""Block and token moves restated with the reference's own torch CPU ops.

TEST INFRASTRUCTURE ONLY (checker and timed CPU baseline).  Each function is
the composition of ``index_select`` / ``index_copy_`` calls the reference
makes for that move, applied plane by plane (one plane = one layer's K or V
cache), and arranged into the chunk layout the CUDA row mover writes:

* block chunks: ``(num_chunks, num_planes, blocks_per_chunk, *block)``;
* token chunks: ``(num_chunks, num_planes, tokens_per_chunk, *row)``.
"""
from __future__ import annotations

from typing import Sequence

import torch


def gather_blocks(actual_blocks: torch.Tensor, slot_ids: torch.Tensor) -> torch.Tensor:
    """adapter.py:543: eviction payloads = actual_blocks.index_select(0, slots)."""
    return actual_blocks.index_select(0, slot_ids)


def scatter_blocks(actual_blocks: torch.Tensor, slot_ids: torch.Tensor, data: torch.Tensor) -> None:
    """adapter.py:653-656: actual_blocks.index_copy_(0, slots, block_data)."""
    actual_blocks.index_copy_(0, slot_ids, data)


def copy_blocks(src: torch.Tensor, src_ids: torch.Tensor, dst: torch.Tensor, dst_ids: torch.Tensor) -> None:
    """adapter.py:779-787: storage.index_select(ids) then actual_blocks.index_copy_(slots, ...)."""
    dst.index_copy_(0, dst_ids, src.index_select(0, src_ids))


def gather_layers(caches: Sequence[torch.Tensor], slot_ids: torch.Tensor,
                  blocks_per_chunk: int | None = None) -> torch.Tensor:
    """Per plane ``index_select`` (adapter.py:543), stacked into block chunks."""
    k = int(slot_ids.numel())
    cb = k if blocks_per_chunk is None else int(blocks_per_chunk)
    per_plane = torch.stack([c.index_select(0, slot_ids) for c in caches], dim=0)  # (P, k, *block)
    block = tuple(per_plane.shape[2:])
    return per_plane.reshape(len(caches), k // cb, cb, *block).transpose(0, 1).contiguous()


def scatter_layers(caches: Sequence[torch.Tensor], slot_ids: torch.Tensor, chunks: torch.Tensor,
                   blocks_per_chunk: int | None = None) -> None:
    """Per plane ``index_copy_`` (adapter.py:653-656) from block chunks."""
    k = int(slot_ids.numel())
    cb = k if blocks_per_chunk is None else int(blocks_per_chunk)
    block = tuple(chunks.shape[3:])
    per_plane = chunks.reshape(k // cb, len(caches), cb, *block).transpose(0, 1).reshape(len(caches), k, *block)
    for p, c in enumerate(caches):
        c.index_copy_(0, slot_ids, per_plane[p])


def physical_slot_mapping(slot_ids: torch.Tensor, block_size: int) -> torch.Tensor:
    """adapter.py:1275-1285: slot_mapping[i*bs + t] = slot_ids[i]*bs + t."""
    offsets = torch.arange(block_size, dtype=torch.int64, device=slot_ids.device)
    return (slot_ids.reshape(-1, 1) * block_size + offsets.reshape(1, -1)).reshape(-1)


def gather_tokens(caches: Sequence[torch.Tensor], slot_mapping: torch.Tensor,
                  tokens_per_chunk: int | None = None, fill: float = 0) -> torch.Tensor:
    """Token rows selected by ``slot_mapping`` from each plane: token slot s sits
    at block s // block_size, offset s % block_size (the inverse of the
    mapping arithmetic at adapter.py:1275-1285).  Rows whose mapping is negative
    stay ``fill``."""
    t = int(slot_mapping.numel())
    tpc = t if tokens_per_chunk is None else int(tokens_per_chunk)
    block_size = int(caches[0].shape[1])
    row = tuple(caches[0].shape[2:])
    valid = slot_mapping >= 0
    positions = torch.nonzero(valid).flatten()
    slots = slot_mapping[valid]
    blocks, offs = slots // block_size, slots % block_size
    out = torch.full((len(caches), t, *row), fill, dtype=caches[0].dtype)
    for p, c in enumerate(caches):
        out[p].index_copy_(0, positions, c[blocks, offs])
    return out.reshape(len(caches), t // tpc, tpc, *row).transpose(0, 1).contiguous()


def scatter_tokens(caches: Sequence[torch.Tensor], slot_mapping: torch.Tensor, chunks: torch.Tensor,
                   tokens_per_chunk: int | None = None) -> None:
    """reshape-and-cache: plane[block, offset of slot_mapping[t]] = row t;
    negative mappings are skipped.  Works on strided plane views."""
    t = int(slot_mapping.numel())
    tpc = t if tokens_per_chunk is None else int(tokens_per_chunk)
    block_size = int(caches[0].shape[1])
    row = tuple(chunks.shape[3:])
    per_plane = chunks.reshape(t // tpc, len(caches), tpc, *row).transpose(0, 1).reshape(len(caches), t, *row)
    valid = slot_mapping >= 0
    positions = torch.nonzero(valid).flatten()
    slots = slot_mapping[valid]
    blocks, offs = slots // block_size, slots % block_size
    for p, c in enumerate(caches):
        c[blocks, offs] = per_plane[p].index_select(0, positions)
