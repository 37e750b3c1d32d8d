"""``kv_cache_adapter_cuda``: the torch-facing op set over the sm_100a C ABI.

The metadata ops keep the names, argument order and in-place behaviour of the
packed-slot-meta extension API that adapter.py calls on its native branch
(csrc/ascend/adapter_meta_kernels.h:6-47 of the reference; call sites
adapter.py:316-330, :397-415, :437-454, :477-491, :557-593, :615-645).  The
row movers replace the torch indexing the reference uses to move KV bytes
(adapter.py:543, :653-656, :779-787) and its slot_mapping transfer
(adapter.py:1200-1243, :1275-1285).

Every op launches on the current CUDA stream of its tensors' device.  Errors
found on the device land in a per-device status word.  ``pop_reusable_slots``
always reads it (its capacity error must surface before the caller moves
data, as in the reference, whose pop synchronises at ``torch::nonzero``);
the other ops read it when ``check`` is true (the default comes from
KVCA_SYNC_CHECKS, on unless set to 0) and otherwise leave errors for the
next check or ``check_status()``.
"""
from __future__ import annotations

import contextlib
import ctypes
import math
import os
from typing import Sequence

import torch

from . import _lib
from .errors import BlockNotFoundError, InsufficientCapacityError

__all__ = [
    "pop_reusable_slots",
    "choose_pop_launch_warps",
    "inspect_load_requests",
    "inspect_save_requests",
    "commit_load_metadata",
    "commit_save_metadata",
    "release_metadata",
    "clock_stream",
    "gather_blocks",
    "scatter_blocks",
    "copy_blocks",
    "gather_layers",
    "scatter_layers",
    "gather_tokens",
    "scatter_tokens",
    "plan_load",
    "plan_save",
    "append_step",
    "append_steps",
    "copy_tokens",
    "scatter_tokens_gather_layers",
    "move_cycle",
    "exchange_blocks",
    "batched_fused_single_layer_kv_transfer",
    "load_device_store",
    "save_device_store",
    "DeviceStoreSession",
    "check_status",
    "status_word",
    "raise_status",
    "library_path",
    "PlaneTable",
]

_lib_handle = _lib.load()

SYNC_CHECKS = os.getenv("KVCA_SYNC_CHECKS", "1") != "0"
POP_ORDERS = {"grouped": _lib.KVCA_POP_ORDER_GROUPED, "prefix": _lib.KVCA_POP_ORDER_PREFIX}
_DEFAULT_POP_ORDER = os.getenv("KVCA_POP_ORDER", "grouped")

_status_words: dict[int, torch.Tensor] = {}
_pop_bitmaps: dict[tuple[int, int, int], torch.Tensor] = {}


def library_path() -> str:
    return str(_lib.lib_path())


# ---------------------------------------------------------------------------
# plumbing
# ---------------------------------------------------------------------------


def _ptr(t: torch.Tensor | None) -> ctypes.c_void_p:
    if t is None or t.numel() == 0:
        return ctypes.c_void_p(0)
    return ctypes.c_void_p(t.data_ptr())


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _index(device: torch.device) -> int:
    return device.index if device.index is not None else torch.cuda.current_device()


def _stream(device: torch.device) -> ctypes.c_void_p:
    if _raw_stream is not None:
        return ctypes.c_void_p(_raw_stream(_index(device)))
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _on(device: torch.device):
    """The device's context for a launch (no switch when it is current)."""
    if _index(device) == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(device)


def _status(device: torch.device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    st = _status_words.get(idx)
    if st is None:
        st = torch.zeros(2, dtype=torch.int64, device=torch.device("cuda", idx))
        _status_words[idx] = st
    return st


def _raise_for(code: int, value: int, what: str) -> None:
    if code == _lib.KVCA_ERR_INSUFFICIENT_CAPACITY:
        raise InsufficientCapacityError(
            "No reusable actual block is available; all resident blocks are pinned"
        )
    if code == _lib.KVCA_ERR_BAD_INDEX:
        raise IndexError(f"{what}: index {value} is out of range")
    if code == _lib.KVCA_ERR_BAD_ARGUMENT:
        raise ValueError(f"{what}: invalid arguments")
    if code == _lib.KVCA_ERR_BLOCK_NOT_FOUND:
        raise BlockNotFoundError("some logical blocks are not in backend")
    if code == _lib.KVCA_ERR_DEVICE_TIMEOUT:
        raise RuntimeError(f"{what}: a bounded device-side wait gave up (CTA {value})")
    raise RuntimeError(f"{what}: CUDA launch failed (code {code})")


def _host_rc(rc: int, what: str) -> None:
    if rc != _lib.KVCA_OK:
        _raise_for(rc, 0, what)


def check_status(device: torch.device | int | None = None, what: str = "kv_cache_adapter_cuda") -> None:
    """Synchronise with the device's status word; raise (and clear) a latched error."""
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    elif isinstance(device, int):
        device = torch.device("cuda", device)
    st = _status(device)
    code, value = st.tolist()
    if code != 0:
        st.zero_()
        _raise_for(int(code), int(value), what)


def status_word(device: torch.device | int | None = None) -> torch.Tensor:
    """The device's status word (code, value), int64, that every launch of
    this module reports into (first error wins).  A pipelined caller copies it
    to pinned host memory after each step and reads it a step later, instead
    of synchronising every step with check_status."""
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    elif isinstance(device, int):
        device = torch.device("cuda", device)
    return _status(device)


def raise_status(code: int, value: int, what: str = "kv_cache_adapter_cuda") -> None:
    """Raise the error a (code, value) pair read from status_word stands for;
    the caller clears the word (status_word(dev).zero_()) before going on."""
    if code != 0:
        _raise_for(int(code), int(value), what)


def _maybe_check(device: torch.device, check: bool | None, what: str) -> None:
    if SYNC_CHECKS if check is None else check:
        check_status(device, what)


def _require(t: torch.Tensor, dtype: torch.dtype | tuple[torch.dtype, ...], name: str) -> None:
    """1-D, contiguous, CUDA, exact dtype (kv_adapter_cuda.cu:43-51 of the reference)."""
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    dtypes = dtype if isinstance(dtype, tuple) else (dtype,)
    if t.dtype not in dtypes:
        raise TypeError(f"{name} has incorrect dtype {t.dtype}")
    if t.dim() != 1:
        raise ValueError(f"{name} must be 1D")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _meta_bits(slot_meta: torch.Tensor) -> int:
    if slot_meta.dtype == torch.uint8:
        return 8
    if slot_meta.dtype == torch.uint16:
        return 16
    raise TypeError(f"slot_meta must be uint8 or uint16, got {slot_meta.dtype}")


_META_DTYPES = (torch.uint8, torch.uint16)

# ---------------------------------------------------------------------------
# slot metadata (packed slot_meta ABI)
# ---------------------------------------------------------------------------


def inspect_load_requests(logical_to_physical: torch.Tensor, slot_meta: torch.Tensor,
                          logical_block_ids: torch.Tensor, *, check: bool | None = None):
    """-> [current_physical:int64, resident:bool, updated_pins:int64, updated_usage:meta]."""
    _require(logical_to_physical, torch.int64, "logical_to_physical")
    _require(slot_meta, _META_DTYPES, "slot_meta")
    _require(logical_block_ids, torch.int64, "logical_block_ids")
    dev = logical_block_ids.device
    k = logical_block_ids.numel()
    cur = torch.empty(k, dtype=torch.int64, device=dev)
    resident = torch.empty(k, dtype=torch.bool, device=dev)
    pins = torch.empty(k, dtype=torch.int64, device=dev)
    usage = torch.empty(k, dtype=slot_meta.dtype, device=dev)
    with _on(dev):
        rc = _lib_handle.kvca_inspect_load_requests(
            _meta_bits(slot_meta), _ptr(logical_to_physical), logical_to_physical.numel(),
            _ptr(slot_meta), slot_meta.numel(), _ptr(logical_block_ids), k, _ptr(cur),
            _ptr(resident), _ptr(pins), _ptr(usage), _ptr(_status(dev)), _stream(dev))
    _host_rc(rc, "inspect_load_requests")
    _maybe_check(dev, check, "inspect_load_requests")
    return [cur, resident, pins, usage]


def inspect_save_requests(logical_to_physical: torch.Tensor, slot_meta: torch.Tensor,
                          logical_block_ids: torch.Tensor, *, check: bool | None = None):
    """-> [current_physical:int64, existing:bool, final_usage:meta]."""
    _require(logical_to_physical, torch.int64, "logical_to_physical")
    _require(slot_meta, _META_DTYPES, "slot_meta")
    _require(logical_block_ids, torch.int64, "logical_block_ids")
    dev = logical_block_ids.device
    k = logical_block_ids.numel()
    cur = torch.empty(k, dtype=torch.int64, device=dev)
    existing = torch.empty(k, dtype=torch.bool, device=dev)
    usage = torch.empty(k, dtype=slot_meta.dtype, device=dev)
    with _on(dev):
        rc = _lib_handle.kvca_inspect_save_requests(
            _meta_bits(slot_meta), _ptr(logical_to_physical), logical_to_physical.numel(),
            _ptr(slot_meta), slot_meta.numel(), _ptr(logical_block_ids), k, _ptr(cur),
            _ptr(existing), _ptr(usage), _ptr(_status(dev)), _stream(dev))
    _host_rc(rc, "inspect_save_requests")
    _maybe_check(dev, check, "inspect_save_requests")
    return [cur, existing, usage]


def _bitmap(dev: torch.device, num_slots: int) -> torch.Tensor:
    """The pop scratch of this (device, stream, table size), kept for reuse:
    kvca_pop_scratch_bytes(num_slots) bytes, returned as a view of its first
    part, the blocked-slot bitmap (zero between calls); the rest is the
    whole-GPU pop's working area of large tables."""
    words = (num_slots + 31) // 32
    key = (_index(dev), _stream(dev).value or 0, words)
    bm = _pop_bitmaps.get(key)
    if bm is None:
        total = max(words, int(_lib_handle.kvca_pop_scratch_bytes(num_slots)) // 4)
        bm = torch.zeros(total, dtype=torch.int32, device=dev)[:words]
        _pop_bitmaps[key] = bm
    return bm


def pop_reusable_slots(slot_meta: torch.Tensor, search_start: torch.Tensor,
                       blocked_slot_ids: torch.Tensor, count: int, *,
                       order: str | None = None, check: bool = True) -> torch.Tensor:
    """Clock sweep; ages ``slot_meta`` and advances ``search_start`` in place.

    ``order="grouped"`` (default) follows the reference's strict path
    (adapter.py:472-525); ``order="prefix"`` the reference CUDA kernel's
    selection (kv_adapter_cuda.cu:101-231).  Raises InsufficientCapacityError
    when fewer than ``count`` slots are reusable, before changing anything.
    ``check=False`` skips the synchronising status read (a caller that knows
    the pool has room, or checks later with ``check_status``).
    """
    _require(slot_meta, _META_DTYPES, "slot_meta")
    _require(search_start, torch.int64, "search_start")
    _require(blocked_slot_ids, torch.int64, "blocked_slot_ids")
    if search_start.numel() != 1:
        raise ValueError("search_start must have shape (1,)")
    count = int(count)
    if count < 0:
        raise ValueError("count must be non-negative")
    dev = slot_meta.device
    out = torch.empty(count, dtype=torch.int64, device=dev)
    if count == 0:
        return out
    n = slot_meta.numel()
    if n == 0:
        raise InsufficientCapacityError(
            "No reusable actual block is available; all resident blocks are pinned")
    order_code = POP_ORDERS[order or _DEFAULT_POP_ORDER]
    with _on(dev):
        rc = _lib_handle.kvca_pop_reusable_slots(
            _meta_bits(slot_meta), order_code, _ptr(slot_meta), n, _ptr(search_start),
            _ptr(blocked_slot_ids), blocked_slot_ids.numel(), count, _ptr(out),
            _ptr(_bitmap(dev, n)), _ptr(_status(dev)), _stream(dev))
    _host_rc(rc, "pop_reusable_slots")
    if check:
        check_status(dev, "pop_reusable_slots")
    return out


def choose_pop_launch_warps(num_slots: int) -> int:
    """Warps per CTA the pop kernel uses for ``num_slots`` slots (binding.cpp:74-78)."""
    if int(num_slots) <= 0:
        raise ValueError("num_slots must be positive")
    return int(_lib_handle.kvca_choose_pop_launch_warps(int(num_slots)))


def commit_load_metadata(logical_to_physical, physical_to_logical, slot_meta,
                         evicted_logical_block_ids, miss_logical_block_ids, miss_physical_slot_ids,
                         hit_slot_ids, hit_pin_counts, hit_usage_counts, miss_usage_counts, *,
                         check: bool | None = None) -> None:
    _require(logical_to_physical, torch.int64, "logical_to_physical")
    _require(physical_to_logical, torch.int64, "physical_to_logical")
    _require(slot_meta, _META_DTYPES, "slot_meta")
    for t, name in ((evicted_logical_block_ids, "evicted_logical_block_ids"),
                    (miss_logical_block_ids, "miss_logical_block_ids"),
                    (miss_physical_slot_ids, "miss_physical_slot_ids"),
                    (hit_slot_ids, "hit_slot_ids")):
        _require(t, torch.int64, name)
    dev = slot_meta.device
    hit_pin_counts = hit_pin_counts.to(device=dev, dtype=torch.int64).contiguous()
    hit_usage_counts = hit_usage_counts.to(device=dev, dtype=slot_meta.dtype).contiguous()
    miss_usage_counts = miss_usage_counts.to(device=dev, dtype=slot_meta.dtype).contiguous()
    if miss_logical_block_ids.numel() != miss_physical_slot_ids.numel() or \
            miss_usage_counts.numel() != miss_physical_slot_ids.numel():
        raise ValueError("miss ids, slots and usage counts must have the same length")
    if hit_pin_counts.numel() != hit_slot_ids.numel() or hit_usage_counts.numel() != hit_slot_ids.numel():
        raise ValueError("hit slots, pins and usage counts must have the same length")
    with _on(dev):
        rc = _lib_handle.kvca_commit_load_metadata(
            _meta_bits(slot_meta), _ptr(logical_to_physical), logical_to_physical.numel(),
            _ptr(physical_to_logical), _ptr(slot_meta), slot_meta.numel(),
            _ptr(evicted_logical_block_ids), evicted_logical_block_ids.numel(),
            _ptr(miss_logical_block_ids), _ptr(miss_physical_slot_ids),
            miss_logical_block_ids.numel(), _ptr(hit_slot_ids), _ptr(hit_pin_counts),
            _ptr(hit_usage_counts), hit_slot_ids.numel(), _ptr(miss_usage_counts),
            _ptr(_status(dev)), _stream(dev))
    _host_rc(rc, "commit_load_metadata")
    _maybe_check(dev, check, "commit_load_metadata")


def commit_save_metadata(logical_to_physical, physical_to_logical, slot_meta,
                         evicted_logical_block_ids, logical_block_ids, physical_slot_ids,
                         final_pin_counts, final_usage_counts, *, check: bool | None = None) -> None:
    _require(logical_to_physical, torch.int64, "logical_to_physical")
    _require(physical_to_logical, torch.int64, "physical_to_logical")
    _require(slot_meta, _META_DTYPES, "slot_meta")
    for t, name in ((evicted_logical_block_ids, "evicted_logical_block_ids"),
                    (logical_block_ids, "logical_block_ids"),
                    (physical_slot_ids, "physical_slot_ids")):
        _require(t, torch.int64, name)
    dev = slot_meta.device
    final_pin_counts = final_pin_counts.to(device=dev, dtype=slot_meta.dtype).contiguous()
    final_usage_counts = final_usage_counts.to(device=dev, dtype=slot_meta.dtype).contiguous()
    k = logical_block_ids.numel()
    if physical_slot_ids.numel() != k or final_pin_counts.numel() != k or final_usage_counts.numel() != k:
        raise ValueError("ids, slots, pins and usage counts must have the same length")
    with _on(dev):
        rc = _lib_handle.kvca_commit_save_metadata(
            _meta_bits(slot_meta), _ptr(logical_to_physical), logical_to_physical.numel(),
            _ptr(physical_to_logical), _ptr(slot_meta), slot_meta.numel(),
            _ptr(evicted_logical_block_ids), evicted_logical_block_ids.numel(),
            _ptr(logical_block_ids), _ptr(physical_slot_ids), _ptr(final_pin_counts),
            _ptr(final_usage_counts), k, _ptr(_status(dev)), _stream(dev))
    _host_rc(rc, "commit_save_metadata")
    _maybe_check(dev, check, "commit_save_metadata")


def release_metadata(logical_to_physical, slot_meta, logical_block_ids, *,
                     check: bool | None = None) -> None:
    _require(logical_to_physical, torch.int64, "logical_to_physical")
    _require(slot_meta, _META_DTYPES, "slot_meta")
    _require(logical_block_ids, torch.int64, "logical_block_ids")
    dev = slot_meta.device
    with _on(dev):
        rc = _lib_handle.kvca_release_metadata(
            _meta_bits(slot_meta), _ptr(logical_to_physical), logical_to_physical.numel(),
            _ptr(slot_meta), slot_meta.numel(), _ptr(logical_block_ids), logical_block_ids.numel(),
            _ptr(_status(dev)), _stream(dev))
    _host_rc(rc, "release_metadata")
    _maybe_check(dev, check, "release_metadata")


_stream_scratch: dict[tuple[int, int, int], torch.Tensor] = {}


def _clock_scratch(dev: torch.device, num_slots: int) -> torch.Tensor:
    words = int(_lib_handle.kvca_clock_stream_scratch_bytes(num_slots)) // 4
    key = (_index(dev), _stream(dev).value or 0, words)
    buf = _stream_scratch.get(key)
    if buf is None:
        buf = torch.zeros(words, dtype=torch.int32, device=dev)
        _stream_scratch[key] = buf
    return buf


def clock_stream(slot_meta: torch.Tensor, search_start: torch.Tensor, num_steps: int,
                 alloc_per_step: int, reaccess: torch.Tensor, reaccess_per_step: int, *,
                 victims: torch.Tensor | None = None, order: str | None = None,
                 method: str = "batched", ctas: int = 0, check: bool | None = None):
    """Run ``num_steps`` of (pop ``alloc_per_step`` victims, refill them with
    usage 1, bump the step's ``reaccess_per_step`` re-accessed slots) in one
    launch.  Returns (victims, steps_done tensor).

    ``method="batched"`` resolves runs of steps that need no aging at once
    (same results) on a cooperative grid of ``ctas`` CTAs (0: one per SM, 1:
    one CTA); ``method="steps"`` runs the steps one after another."""
    _require(slot_meta, _META_DTYPES, "slot_meta")
    _require(search_start, torch.int64, "search_start")
    _require(reaccess, torch.int64, "reaccess")
    dev = slot_meta.device
    num_steps, alloc_per_step, reaccess_per_step = int(num_steps), int(alloc_per_step), int(reaccess_per_step)
    if reaccess.numel() < num_steps * reaccess_per_step:
        raise ValueError("reaccess holds fewer than num_steps * reaccess_per_step ids")
    if victims is None:
        victims = torch.empty(num_steps * alloc_per_step, dtype=torch.int64, device=dev)
    else:
        _require(victims, torch.int64, "victims")
        if victims.numel() < num_steps * alloc_per_step:
            raise ValueError("victims is too small")
    steps_done = torch.zeros(1, dtype=torch.int64, device=dev)
    order_code = POP_ORDERS[order or _DEFAULT_POP_ORDER]
    with _on(dev):
        if method == "batched":
            rc = _lib_handle.kvca_clock_stream_batched(
                _meta_bits(slot_meta), order_code, _ptr(slot_meta), slot_meta.numel(), _ptr(search_start),
                num_steps, alloc_per_step, _ptr(reaccess), reaccess_per_step, _ptr(victims), _ptr(steps_done),
                _ptr(_clock_scratch(dev, slot_meta.numel())), int(ctas), _ptr(_status(dev)), _stream(dev))
        elif method == "steps":
            rc = _lib_handle.kvca_clock_stream(
                _meta_bits(slot_meta), order_code, _ptr(slot_meta), slot_meta.numel(), _ptr(search_start),
                num_steps, alloc_per_step, _ptr(reaccess), reaccess_per_step, _ptr(victims), _ptr(steps_done),
                _ptr(_status(dev)), _stream(dev))
        else:
            raise ValueError(f"unknown clock stream method {method!r}")
    _host_rc(rc, "clock_stream")
    _maybe_check(dev, check, "clock_stream")
    return victims, steps_done


def append_step(slot_meta: torch.Tensor, search_start: torch.Tensor, logical_to_physical: torch.Tensor,
                physical_to_logical: torch.Tensor, need: torch.Tensor, cur_block: torch.Tensor,
                cur_logical: torch.Tensor, pos: torch.Tensor, block_size: int, next_logical: torch.Tensor,
                victims: torch.Tensor, slot_mapping: torch.Tensor, *, order: str | None = None,
                check: bool | None = None) -> None:
    """One decode step of block bookkeeping in one launch (see
    kvca_append_step): new blocks for the sequences ``need`` (pop ->
    commit as fresh pinned saves -> release the full blocks), then this
    step's ``slot_mapping`` and the positions advanced.  ``victims`` takes
    ``need.numel()`` slots.  Nothing is read back: capturable in a graph."""
    for t, name in ((search_start, "search_start"), (logical_to_physical, "logical_to_physical"),
                    (physical_to_logical, "physical_to_logical"), (need, "need"), (cur_block, "cur_block"),
                    (cur_logical, "cur_logical"), (pos, "pos"), (next_logical, "next_logical"),
                    (victims, "victims"), (slot_mapping, "slot_mapping")):
        _require(t, torch.int64, name)
    _require(slot_meta, _META_DTYPES, "slot_meta")
    seqs = cur_block.numel()
    if cur_logical.numel() != seqs or pos.numel() != seqs or slot_mapping.numel() != seqs:
        raise ValueError("cur_block, cur_logical, pos and slot_mapping need one entry per sequence")
    c = need.numel()
    if victims.numel() < c:
        raise ValueError("victims must hold one slot per sequence in need")
    dev = slot_meta.device
    n = slot_meta.numel()
    with _on(dev):
        rc = _lib_handle.kvca_append_step(
            _meta_bits(slot_meta), POP_ORDERS[order or _DEFAULT_POP_ORDER], _ptr(slot_meta), n, _ptr(search_start),
            _ptr(logical_to_physical), logical_to_physical.numel(), _ptr(physical_to_logical), _ptr(need), c,
            _ptr(cur_block), _ptr(cur_logical), _ptr(pos), seqs, int(block_size), _ptr(next_logical),
            _ptr(victims), _ptr(slot_mapping), _ptr(_bitmap(dev, n)), _ptr(_status(dev)), _stream(dev))
    _host_rc(rc, "append_step")
    _maybe_check(dev, check, "append_step")


def append_steps(slot_meta: torch.Tensor, search_start: torch.Tensor, logical_to_physical: torch.Tensor,
                 physical_to_logical: torch.Tensor, need: torch.Tensor, need_offsets: torch.Tensor,
                 cur_block: torch.Tensor, cur_logical: torch.Tensor, pos: torch.Tensor, block_size: int,
                 next_logical: torch.Tensor, victims: torch.Tensor, slot_mapping: torch.Tensor, *,
                 order: str | None = None, check: bool | None = None) -> None:
    """``need_offsets.numel() - 1`` decode steps of ``append_step`` in one
    launch (see kvca_append_steps): step s serves the sequences
    ``need[need_offsets[s]:need_offsets[s + 1]]``, its victims go to the same
    positions of ``victims`` and its slot_mapping to ``slot_mapping[s]``
    (shape ``(steps, seqs)``).  Equal to that many ``append_step`` calls; an
    error at step s leaves the earlier steps done.  Nothing is read back:
    capturable in a graph."""
    for t, name in ((search_start, "search_start"), (logical_to_physical, "logical_to_physical"),
                    (physical_to_logical, "physical_to_logical"), (need, "need"), (need_offsets, "need_offsets"),
                    (cur_block, "cur_block"), (cur_logical, "cur_logical"), (pos, "pos"),
                    (next_logical, "next_logical"), (victims, "victims"), (slot_mapping.reshape(-1), "slot_mapping")):
        _require(t, torch.int64, name)
    _require(slot_meta, _META_DTYPES, "slot_meta")
    if not slot_mapping.is_contiguous():
        raise ValueError("slot_mapping must be contiguous")
    seqs = cur_block.numel()
    steps = need_offsets.numel() - 1
    if steps < 0:
        raise ValueError("need_offsets needs one entry more than there are steps")
    if cur_logical.numel() != seqs or pos.numel() != seqs or slot_mapping.numel() != steps * seqs:
        raise ValueError("cur_block, cur_logical and pos need one entry per sequence, slot_mapping one per "
                         "sequence and step")
    if victims.numel() < need.numel():
        raise ValueError("victims must hold one slot per entry of need")
    dev = slot_meta.device
    with _on(dev):
        rc = _lib_handle.kvca_append_steps(
            _meta_bits(slot_meta), POP_ORDERS[order or _DEFAULT_POP_ORDER], _ptr(slot_meta), slot_meta.numel(),
            _ptr(search_start), _ptr(logical_to_physical), logical_to_physical.numel(), _ptr(physical_to_logical),
            _ptr(need), _ptr(need_offsets), need.numel(), steps, _ptr(cur_block), _ptr(cur_logical), _ptr(pos),
            seqs, int(block_size), _ptr(next_logical), _ptr(victims), _ptr(slot_mapping), _ptr(_status(dev)),
            _stream(dev))
    _host_rc(rc, "append_steps")
    _maybe_check(dev, check, "append_steps")


class LoadPlan:
    """Result of ``plan_load``: views sized by the plan's counts."""

    __slots__ = ("result", "hit_slots", "hit_pins", "hit_usage", "miss_ids", "victims", "evict_ids",
                 "evict_slots")

    def __init__(self, **kw):
        for k, v in kw.items():
            setattr(self, k, v)


class SavePlan:
    """Result of ``plan_save``: views sized by the plan's counts."""

    __slots__ = ("selected", "move_slots", "final_pins", "final_usage", "allocated", "evict_ids", "evict_slots")

    def __init__(self, **kw):
        for k, v in kw.items():
            setattr(self, k, v)


def _plan_counts(counts: torch.Tensor, what: str) -> list[int]:
    """The call's only synchronisation: the plan's counts, its error, and an
    error latched earlier by an unchecked launch (raised first)."""
    vals = counts.tolist()
    if vals[5] != 0 or vals[3] != 0:
        _status(counts.device).zero_()
        if vals[5] != 0:
            _raise_for(int(vals[5]), int(vals[6]), "an earlier unchecked launch")
        try:
            _raise_for(int(vals[3]), int(vals[4]), what)
        except BlockNotFoundError as exc:
            exc.counts = vals  # the plan's counts: the spill has run
            raise
    return vals


def plan_load(logical_to_physical: torch.Tensor, physical_to_logical: torch.Tensor, slot_meta: torch.Tensor,
              search_start: torch.Tensor, logical_block_ids: torch.Tensor, *,
              order: str | None = None) -> LoadPlan:
    """inspect + hit/miss split + pop + eviction plan of KVCacheAdapter.load
    (adapter.py:264-305) in one launch and one synchronisation.  Mutates
    slot_meta (aging) and search_start like pop_reusable_slots."""
    for t, name in ((logical_to_physical, "logical_to_physical"), (physical_to_logical, "physical_to_logical"),
                    (search_start, "search_start"), (logical_block_ids, "logical_block_ids")):
        _require(t, torch.int64, name)
    _require(slot_meta, _META_DTYPES, "slot_meta")
    dev = slot_meta.device
    k = logical_block_ids.numel()
    buf = torch.empty((7, k), dtype=torch.int64, device=dev)
    hit_usage = torch.empty(k, dtype=slot_meta.dtype, device=dev)
    counts = torch.empty(7, dtype=torch.int64, device=dev)
    n = slot_meta.numel()
    with _on(dev):
        rc = _lib_handle.kvca_plan_load(
            _meta_bits(slot_meta), POP_ORDERS[order or _DEFAULT_POP_ORDER], _ptr(logical_to_physical),
            logical_to_physical.numel(), _ptr(physical_to_logical), _ptr(slot_meta), n, _ptr(search_start),
            _ptr(logical_block_ids), k, _ptr(_bitmap(dev, n)), _ptr(buf[0]), _ptr(buf[1]), _ptr(buf[2]),
            _ptr(hit_usage), _ptr(buf[3]), _ptr(buf[4]), _ptr(buf[5]), _ptr(buf[6]), _ptr(counts),
            _ptr(_status(dev)), _stream(dev))
    _host_rc(rc, "plan_load")
    nh, nm, ne = _plan_counts(counts, "plan_load")[:3]
    return LoadPlan(result=buf[0], hit_slots=buf[1, :nh], hit_pins=buf[2, :nh], hit_usage=hit_usage[:nh],
                    miss_ids=buf[3, :nm], victims=buf[4, :nm], evict_ids=buf[5, :ne], evict_slots=buf[6, :ne])


def plan_save(logical_to_physical: torch.Tensor, physical_to_logical: torch.Tensor, slot_meta: torch.Tensor,
              search_start: torch.Tensor, logical_block_ids: torch.Tensor, *,
              order: str | None = None) -> SavePlan:
    """inspect + existing/missing split + pop + final pins/usage + eviction
    plan of KVCacheAdapter.save (adapter.py:221-243) in one launch and one
    synchronisation."""
    for t, name in ((logical_to_physical, "logical_to_physical"), (physical_to_logical, "physical_to_logical"),
                    (search_start, "search_start"), (logical_block_ids, "logical_block_ids")):
        _require(t, torch.int64, name)
    _require(slot_meta, _META_DTYPES, "slot_meta")
    dev = slot_meta.device
    k = logical_block_ids.numel()
    buf = torch.empty((5, k), dtype=torch.int64, device=dev)
    small = torch.empty((2, k), dtype=slot_meta.dtype, device=dev)
    counts = torch.empty(7, dtype=torch.int64, device=dev)
    n = slot_meta.numel()
    with _on(dev):
        rc = _lib_handle.kvca_plan_save(
            _meta_bits(slot_meta), POP_ORDERS[order or _DEFAULT_POP_ORDER], _ptr(logical_to_physical),
            logical_to_physical.numel(), _ptr(physical_to_logical), _ptr(slot_meta), n, _ptr(search_start),
            _ptr(logical_block_ids), k, _ptr(_bitmap(dev, n)), _ptr(buf[0]), _ptr(buf[4]), _ptr(small[0]),
            _ptr(small[1]), _ptr(buf[1]), _ptr(buf[2]), _ptr(buf[3]), _ptr(counts), _ptr(_status(dev)),
            _stream(dev))
    _host_rc(rc, "plan_save")
    nx, nm, ne = _plan_counts(counts, "plan_save")[:3]
    return SavePlan(selected=buf[0], move_slots=buf[4], final_pins=small[0], final_usage=small[1],
                    allocated=buf[1, :nm], evict_ids=buf[2, :ne], evict_slots=buf[3, :ne])


def _rows_of(t: torch.Tensor, name: str) -> tuple[int, int]:
    """(row stride, row bytes) of a tensor whose dim 0 indexes dense rows."""
    if not _dense_suffix(t, 1):
        raise ValueError(f"{name}: each row must be contiguous")
    esz = t.element_size()
    return int(t.stride(0)) * esz, int(math.prod(t.shape[1:])) * esz


def _store_desc(storage: torch.Tensor, present: torch.Tensor, scratch: torch.Tensor,
                actual_blocks: torch.Tensor) -> tuple[_lib.DeviceStore, int, int]:
    """Descriptor of a store driven from actual_blocks' GPU: storage on that GPU,
    or in pinned host memory (a host tier; present and scratch stay on the GPU)."""
    on_host = storage.device.type == "cpu"
    if (storage.device != actual_blocks.device and not on_host) or storage.dtype != actual_blocks.dtype \
            or storage.shape[1:] != actual_blocks.shape[1:]:
        raise ValueError("storage and actual_blocks must share device (or storage be pinned host memory), "
                         "dtype and block shape")
    if on_host and not host_memory_usable(storage):
        raise ValueError("host storage must be pinned (torch pin_memory)")
    if present.device != actual_blocks.device or scratch.device != actual_blocks.device:
        raise ValueError("present and scratch must be on actual_blocks' device")
    _require(present, torch.bool, "present")
    _require(scratch, torch.int32, "scratch")
    n_logical = storage.shape[0]
    if present.numel() != n_logical or scratch.numel() != n_logical:
        raise ValueError("present and scratch need one entry per stored block")
    s_stride, row_bytes = _rows_of(storage, "storage")
    a_stride, _ = _rows_of(actual_blocks, "actual_blocks")
    flags = _lib.KVCA_FLAG_HOST_MEMORY if on_host else 0
    return (_lib.DeviceStore(storage.data_ptr(), s_stride, present.data_ptr(), scratch.data_ptr(), flags),
            a_stride, row_bytes)


_store_descs: dict[tuple, tuple] = {}


def _store_desc_cached(storage: torch.Tensor, present: torch.Tensor, scratch: torch.Tensor,
                       actual_blocks: torch.Tensor) -> tuple[_lib.DeviceStore, int, int]:
    """_store_desc, remembered for the same tensors: the descriptor is a pure
    function of the key (addresses, shapes, strides, dtypes, devices and,
    for host storage, pinning), which the adapter passes unchanged on every
    call."""
    key = tuple((t.data_ptr(), tuple(t.shape), t.stride(), t.dtype, t.device)
                for t in (storage, present, scratch, actual_blocks)) + \
        ((storage.is_pinned(),) if storage.device.type == "cpu" else ())
    got = _store_descs.get(key)
    if got is None:
        got = _store_desc(storage, present, scratch, actual_blocks)
        if len(_store_descs) >= 64:
            _store_descs.clear()
        _store_descs[key] = got
    return got


class _StoreCallBuffers:
    """Work space of the device-store calls on one (device, stream): device
    work arrays grown to the largest request so far, the count vector, and a
    pinned host copy of it.  Each call ends by reading its counts (a stream
    synchronisation), so the next call on the stream may reuse them."""

    def __init__(self, dev: torch.device):
        self.dev = dev
        self.cap = 0
        self.work = self.work_meta = None
        self.counts = torch.empty(8, dtype=torch.int64, device=dev)
        self.counts_host = torch.empty(8, dtype=torch.int64, pin_memory=True)

    def get(self, k: int, meta_dtype: torch.dtype) -> tuple[torch.Tensor, torch.Tensor]:
        if self.work is None or k > self.cap or self.work_meta.dtype != meta_dtype:
            self.cap = max(k, 2 * self.cap, 64)
            self.work = torch.empty(9 * self.cap, dtype=torch.int64, device=self.dev)
            self.work_meta = torch.empty(2 * self.cap, dtype=meta_dtype, device=self.dev)
        return self.work, self.work_meta

    def read_counts(self, n: int) -> list[int]:
        self.counts_host.copy_(self.counts, non_blocking=True)
        torch.cuda.current_stream(self.dev).synchronize()
        return self.counts_host.tolist()[:n]


_store_buffers: dict[tuple[int, int], _StoreCallBuffers] = {}


def _store_call_buffers(dev: torch.device) -> _StoreCallBuffers:
    idx = _index(dev)
    key = (idx, _stream(dev).value or 0)
    got = _store_buffers.get(key)
    if got is None:
        if len(_store_buffers) >= 64:  # many short-lived streams: start over
            _store_buffers.clear()
        got = _StoreCallBuffers(torch.device("cuda", idx))
        _store_buffers[key] = got
    return got


def _store_counts(vals: list[int], what: str, dev: torch.device) -> list[int]:
    """_plan_counts on counts already read to the host."""
    if vals[5] != 0 or vals[3] != 0:
        _status(dev).zero_()
        if vals[5] != 0:
            _raise_for(int(vals[5]), int(vals[6]), "an earlier unchecked launch")
        try:
            _raise_for(int(vals[3]), int(vals[4]), what)
        except BlockNotFoundError as exc:
            exc.counts = vals  # the plan's counts: the spill has run
            raise
    return vals


def load_device_store(logical_to_physical: torch.Tensor, physical_to_logical: torch.Tensor, slot_meta: torch.Tensor,
                      search_start: torch.Tensor, logical_block_ids: torch.Tensor, actual_blocks: torch.Tensor,
                      storage: torch.Tensor, present: torch.Tensor, scratch: torch.Tensor, *,
                      order: str | None = None) -> tuple[torch.Tensor, list[int]]:
    """KVCacheAdapter.load against a block store on the same GPU (storage row
    l = logical block l): plan, spill, presence check, fill and commit as one
    enqueued sequence, then one read of the counts.  Returns (slots, counts);
    raises InsufficientCapacityError / BlockNotFoundError / IndexError with
    the reference's state effects."""
    for t, name in ((logical_to_physical, "logical_to_physical"), (physical_to_logical, "physical_to_logical"),
                    (search_start, "search_start"), (logical_block_ids, "logical_block_ids")):
        _require(t, torch.int64, name)
    _require(slot_meta, _META_DTYPES, "slot_meta")
    desc, a_stride, row_bytes = _store_desc_cached(storage, present, scratch, actual_blocks)
    dev = slot_meta.device
    k = logical_block_ids.numel()
    n = slot_meta.numel()
    bufs = _store_call_buffers(dev)
    work, work_meta = bufs.get(k, slot_meta.dtype)
    result = torch.empty(k, dtype=torch.int64, device=dev)
    with _on(dev):
        rc = _lib_handle.kvca_load_device_store(
            _meta_bits(slot_meta), POP_ORDERS[order or _DEFAULT_POP_ORDER], _ptr(logical_to_physical),
            logical_to_physical.numel(), _ptr(physical_to_logical), _ptr(slot_meta), n, _ptr(search_start),
            _ptr(logical_block_ids), k, _ptr(_bitmap(dev, n)), ctypes.byref(desc), actual_blocks.data_ptr(),
            a_stride, row_bytes, _ptr(work), _ptr(work_meta), _ptr(result), _ptr(bufs.counts), _ptr(_status(dev)),
            _stream(dev))
        _host_rc(rc, "load_device_store")
        vals = bufs.read_counts(8)
    return result, _store_counts(vals, "load_device_store", dev)


def save_device_store(logical_to_physical: torch.Tensor, physical_to_logical: torch.Tensor, slot_meta: torch.Tensor,
                      search_start: torch.Tensor, logical_block_ids: torch.Tensor, block_data: torch.Tensor,
                      actual_blocks: torch.Tensor, storage: torch.Tensor, present: torch.Tensor,
                      scratch: torch.Tensor, *, order: str | None = None) -> list[int]:
    """KVCacheAdapter.save against a block store on the same GPU: plan, spill,
    commit and data scatter as one enqueued sequence, then one read of the
    counts (returned)."""
    for t, name in ((logical_to_physical, "logical_to_physical"), (physical_to_logical, "physical_to_logical"),
                    (search_start, "search_start"), (logical_block_ids, "logical_block_ids")):
        _require(t, torch.int64, name)
    _require(slot_meta, _META_DTYPES, "slot_meta")
    desc, a_stride, row_bytes = _store_desc_cached(storage, present, scratch, actual_blocks)
    dev = slot_meta.device
    k = logical_block_ids.numel()
    _chunk_tensor(block_data, (k, *actual_blocks.shape[1:]), actual_blocks.dtype, dev, "block_data")
    n = slot_meta.numel()
    bufs = _store_call_buffers(dev)
    work, work_meta = bufs.get(k, slot_meta.dtype)
    with _on(dev):
        rc = _lib_handle.kvca_save_device_store(
            _meta_bits(slot_meta), POP_ORDERS[order or _DEFAULT_POP_ORDER], _ptr(logical_to_physical),
            logical_to_physical.numel(), _ptr(physical_to_logical), _ptr(slot_meta), n, _ptr(search_start),
            _ptr(logical_block_ids), k, _ptr(_bitmap(dev, n)), ctypes.byref(desc), actual_blocks.data_ptr(),
            a_stride, row_bytes, block_data.data_ptr(), _ptr(work), _ptr(work_meta), _ptr(bufs.counts),
            _ptr(_status(dev)), _stream(dev))
        _host_rc(rc, "save_device_store")
        vals = bufs.read_counts(7)
    return _store_counts(vals, "save_device_store", dev)


class DeviceStoreSession:
    """load_device_store / save_device_store for one adapter and store, with
    the arguments that do not change between calls described once
    (kvca_adapter_session): a call is one C call that enqueues the whole load
    or save, copies the counts to pinned host memory and waits for the
    stream.  The tensors must keep their storage for the session's life (the
    adapter's tables and cache and the store's rows, present mask and
    scratch); the work arrays grow with the largest request; the session
    follows the current stream of the device."""

    def __init__(self, logical_to_physical: torch.Tensor, physical_to_logical: torch.Tensor,
                 slot_meta: torch.Tensor, search_start: torch.Tensor, actual_blocks: torch.Tensor,
                 storage: torch.Tensor, present: torch.Tensor, scratch: torch.Tensor, *, order: str | None = None):
        for t, name in ((logical_to_physical, "logical_to_physical"), (physical_to_logical, "physical_to_logical"),
                        (search_start, "search_start")):
            _require(t, torch.int64, name)
        _require(slot_meta, _META_DTYPES, "slot_meta")
        desc, a_stride, row_bytes = _store_desc(storage, present, scratch, actual_blocks)
        self.device = slot_meta.device
        self.index = _index(self.device)
        self.row_shape = tuple(actual_blocks.shape[1:])
        self.dtype = actual_blocks.dtype
        self.tensors = (logical_to_physical, physical_to_logical, slot_meta, search_start, actual_blocks, storage,
                        present, scratch)
        self.meta_dtype = slot_meta.dtype
        self.counts = torch.zeros(8, dtype=torch.int64, device=self.device)
        self.counts_host = torch.zeros(16, dtype=torch.int64, pin_memory=True)  # counts, then the sequence
        self.counts_view = (ctypes.c_int64 * 8).from_address(self.counts_host.data_ptr())
        n = slot_meta.numel()
        self.s = _lib.AdapterSession(
            _meta_bits(slot_meta), POP_ORDERS[order or _DEFAULT_POP_ORDER], logical_to_physical.data_ptr(),
            logical_to_physical.numel(), physical_to_logical.data_ptr(), slot_meta.data_ptr(), n,
            search_start.data_ptr(), _bitmap(self.device, n).data_ptr(), desc, actual_blocks.data_ptr(), a_stride,
            row_bytes, None, None, 0, self.counts.data_ptr(), self.counts_host.data_ptr(),
            _status(self.device).data_ptr(), _stream(self.device).value, 0)
        self.ref = ctypes.byref(self.s)
        self.work = self.work_meta = None
        self._grow(64)

    def _grow(self, k: int) -> None:
        cap = max(k, 2 * int(self.s.work_ids), 64)
        self.work = torch.empty(9 * cap, dtype=torch.int64, device=self.device)
        self.work_meta = torch.empty(2 * cap, dtype=self.meta_dtype, device=self.device)
        self.s.work = self.work.data_ptr()
        self.s.work_meta = self.work_meta.data_ptr()
        self.s.work_ids = cap

    def _prepare(self, k: int) -> None:
        if k > self.s.work_ids:
            self._grow(k)
        stream = _raw_stream(self.index) if _raw_stream is not None else _stream(self.device).value
        if stream != self.s.stream:
            self.s.stream = stream

    def load(self, logical_block_ids: torch.Tensor) -> tuple[torch.Tensor, list[int]]:
        """As load_device_store: (slots, counts)."""
        k = logical_block_ids.numel()
        self._prepare(k)
        result = torch.empty(k, dtype=torch.int64, device=self.device)
        _host_rc(_lib_handle.kvca_session_load(self.ref, logical_block_ids.data_ptr(), k, result.data_ptr()),
                 "load_device_store")
        return result, _store_counts(self.counts_view[:], "load_device_store", self.device)

    def save(self, logical_block_ids: torch.Tensor, block_data: torch.Tensor) -> list[int]:
        """As save_device_store: counts."""
        k = logical_block_ids.numel()
        if block_data.dtype != self.dtype or tuple(block_data.shape) != (k, *self.row_shape) \
                or not block_data.is_contiguous() or block_data.device != self.device:
            _chunk_tensor(block_data, (k, *self.row_shape), self.dtype, self.device, "block_data")
        self._prepare(k)
        _host_rc(_lib_handle.kvca_session_save(self.ref, logical_block_ids.data_ptr(), k, block_data.data_ptr()),
                 "save_device_store")
        return _store_counts(self.counts_view[:7], "save_device_store", self.device)


# ---------------------------------------------------------------------------
# row movers
# ---------------------------------------------------------------------------


def _dense_suffix(t: torch.Tensor, start: int) -> bool:
    """True when dims ``start:`` of ``t`` are laid out contiguously."""
    expected = 1
    for size, stride in zip(reversed(t.shape[start:]), reversed(t.stride()[start:])):
        if size != 1 and stride != expected:
            return False
        expected *= size
    return True


class PlaneTable:
    """Plane table of a paged cache side: one device address per plane (layer x
    K/V), all planes sharing shape, dtype, strides and device.

    Build it once with ``PlaneTable(planes, row_dim)`` and pass it wherever a
    list of planes is accepted, to skip re-validating the planes on every call.
    ``row_dim`` is 1 for block-granular moves (rows are whole blocks) and 2
    for token-granular moves (planes are ``(num_blocks, block_size, *row)``).
    """

    def __init__(self, planes: Sequence[torch.Tensor], row_dim: int = 1, name: str = "caches"):
        if isinstance(planes, torch.Tensor):
            planes = [planes]
        planes = list(planes)
        if not planes:
            raise ValueError(f"{name} must hold at least one plane")
        if len(planes) > _lib.KVCA_MAX_PLANES:
            raise ValueError(f"{name}: at most {_lib.KVCA_MAX_PLANES} planes per call")
        first = planes[0]
        self.host = not first.is_cuda
        if self.host and not all(host_memory_usable(p) for p in planes):
            raise ValueError(f"{name} must be CUDA tensors or pinned host memory")
        if first.dim() < row_dim:
            raise ValueError(f"{name} planes must have at least {row_dim} dims")
        for p in planes[1:]:
            if (p.shape != first.shape or p.dtype != first.dtype or p.stride() != first.stride()
                    or p.device != first.device):
                raise ValueError(f"{name} planes must share shape, dtype, strides and device")
        if not _dense_suffix(first, row_dim):
            raise ValueError(f"{name}: the row dims of each plane must be contiguous")
        esz = first.element_size()
        self.planes = planes
        self.device = first.device
        self.dtype = first.dtype
        self.num_blocks = int(first.shape[0])
        self.block_size = int(first.shape[1]) if row_dim == 2 else 1
        self.row_shape = tuple(first.shape[row_dim:])
        self.row_bytes = int(math.prod(self.row_shape)) * esz
        self.block_stride = int(first.stride(0)) * esz
        self.row_stride = int(first.stride(1)) * esz if row_dim == 2 else self.row_bytes
        self.row_dim = row_dim
        self._table = (ctypes.c_uint64 * len(planes))(*[p.data_ptr() for p in planes])

    def desc(self, index: torch.Tensor | None) -> _lib.PagedDesc:
        return _lib.PagedDesc(
            ctypes.cast(self._table, ctypes.POINTER(ctypes.c_uint64)), self.num_blocks,
            self.block_size, self.block_stride, self.row_stride,
            ctypes.c_void_p(index.data_ptr()) if index is not None and index.numel() else None)


_single_plane_tables: dict[tuple, PlaneTable] = {}


def host_memory_usable(t: torch.Tensor) -> bool:
    """True when every byte of ``t`` is pinned host memory that kernels reach
    at the same address (torch ``pin_memory`` allocations)."""
    if t.is_cuda or t.numel() == 0:
        return False
    span = (sum((n - 1) * st for n, st in zip(t.shape, t.stride())) + 1) * t.element_size()
    return bool(_lib_handle.kvca_host_memory_usable(ctypes.c_void_p(t.data_ptr()), span))


def _move_device(*sides) -> torch.device:
    """The GPU a move runs on: the one CUDA side (the other may be host memory)."""
    devs = {s.device for s in sides if s is not None and s.device.type == "cuda"}
    if len(devs) != 1:
        raise ValueError("a move needs its CUDA tensors on one device (the other side may be pinned host memory)")
    return devs.pop()


def _host_flag(*sides) -> int:
    return _lib.KVCA_FLAG_HOST_MEMORY if any(s is not None and s.device.type != "cuda" for s in sides) else 0


def _planes(caches, row_dim: int, name: str, *, allow_host: bool = False) -> PlaneTable:
    table = _plane_table(caches, row_dim, name)
    if table.host and not allow_host:
        raise ValueError(f"{name} must be CUDA tensors")
    return table


def _plane_table(caches, row_dim: int, name: str) -> PlaneTable:
    if isinstance(caches, PlaneTable):
        if caches.row_dim != row_dim:
            raise ValueError(f"{name}: plane table built for row_dim {caches.row_dim}, need {row_dim}")
        return caches
    if isinstance(caches, (list, tuple)) and len(caches) == 1 and isinstance(caches[0], torch.Tensor):
        # One-plane tables (actual_blocks, backend storage) are rebuilt on every
        # call otherwise; the table depends only on address, layout and dtype.
        t = caches[0]
        key = (t.data_ptr(), tuple(t.shape), t.stride(), t.dtype, t.device, row_dim)
        table = _single_plane_tables.get(key)
        if table is None:
            table = PlaneTable(caches, row_dim, name)
            table.planes = [None]  # no reference kept: the cache must not hold memory alive
            if len(_single_plane_tables) >= 64:
                _single_plane_tables.clear()
            _single_plane_tables[key] = table
        return table
    return PlaneTable(caches, row_dim, name)


def _chunk_desc(t: torch.Tensor, rows_per_chunk: int, num_planes: int, row_bytes: int) -> _lib.ChunkDesc:
    plane_stride = rows_per_chunk * row_bytes
    return _lib.ChunkDesc(t.data_ptr(), rows_per_chunk, num_planes * plane_stride, row_bytes,
                          plane_stride)


def _require_index(idx: torch.Tensor, device: torch.device, name: str) -> None:
    _require(idx, torch.int64, name)
    if idx.device != device:
        raise ValueError(f"{name} must be on {device}")


def _launch_move(fn_name: str, src, dst, num_planes: int, num_rows: int, row_bytes: int,
                 flags: int, device: torch.device, check: bool | None) -> None:
    if num_rows == 0:
        return
    with _on(device):
        rc = getattr(_lib_handle, fn_name)(
            ctypes.byref(src), ctypes.byref(dst), num_planes, num_rows, row_bytes, flags,
            _ptr(_status(device)), _stream(device))
    _host_rc(rc, fn_name)
    _maybe_check(device, check, fn_name)


def _chunk_tensor(out: torch.Tensor | None, shape: tuple[int, ...], dtype, device, name: str) -> torch.Tensor:
    """The contiguous chunk side: ``out`` if it fits (on ``device``, or in
    pinned host memory when ``device`` is a GPU), else a new tensor on ``device``."""
    if out is None:
        return torch.empty(shape, dtype=dtype, device=device)
    on_host = out.device.type == "cpu" and device.type == "cuda"
    if tuple(out.shape) != tuple(shape) or out.dtype != dtype or (out.device != device and not on_host):
        raise ValueError(f"{name} must be {tuple(shape)} {dtype} on {device} or in pinned host memory")
    if not out.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if on_host and not host_memory_usable(out):
        raise ValueError(f"{name}: host tensors must be pinned (torch pin_memory)")
    return out


def gather_blocks(actual_blocks: torch.Tensor, slot_ids: torch.Tensor,
                  out: torch.Tensor | None = None, *, check: bool | None = None) -> torch.Tensor:
    """``actual_blocks.index_select(0, slot_ids)`` (adapter.py:543)."""
    pl = _planes([actual_blocks], 1, "actual_blocks", allow_host=True)
    dev = _move_device(pl, slot_ids)
    _require_index(slot_ids, dev, "slot_ids")
    k = slot_ids.numel()
    out = _chunk_tensor(out, (k, *pl.row_shape), pl.dtype, dev, "out")
    _launch_move("kvca_gather", pl.desc(slot_ids), _chunk_desc(out, max(k, 1), 1, pl.row_bytes),
                 1, k, pl.row_bytes, _host_flag(pl, out), dev, check)
    return out


def scatter_blocks(actual_blocks: torch.Tensor, slot_ids: torch.Tensor, block_data: torch.Tensor,
                   *, skip_negative: bool = False, check: bool | None = None) -> None:
    """``actual_blocks.index_copy_(0, slot_ids, block_data)`` (adapter.py:653-656).
    Slots must be distinct (a repeated slot receives one of its rows); with
    ``skip_negative`` rows whose slot is negative are not written."""
    pl = _planes([actual_blocks], 1, "actual_blocks", allow_host=True)
    dev = _move_device(pl, slot_ids)
    _require_index(slot_ids, dev, "slot_ids")
    k = slot_ids.numel()
    _chunk_tensor(block_data, (k, *pl.row_shape), pl.dtype, dev, "block_data")
    flags = (_lib.KVCA_FLAG_SKIP_NEGATIVE if skip_negative else 0) | _host_flag(pl, block_data)
    _launch_move("kvca_scatter", _chunk_desc(block_data, max(k, 1), 1, pl.row_bytes),
                 pl.desc(slot_ids), 1, k, pl.row_bytes, flags, dev, check)


def copy_blocks(src_blocks: torch.Tensor, src_ids: torch.Tensor, dst_blocks: torch.Tensor,
                dst_ids: torch.Tensor, *, check: bool | None = None) -> None:
    """``dst.index_copy_(0, dst_ids, src.index_select(0, src_ids))`` in one pass
    (adapter.py:779-787).  ``src_blocks`` and ``dst_blocks`` must not overlap."""
    s = _planes([src_blocks], 1, "src_blocks", allow_host=True)
    d = _planes([dst_blocks], 1, "dst_blocks", allow_host=True)
    if s.row_bytes != d.row_bytes or s.dtype != d.dtype:
        raise ValueError("src_blocks and dst_blocks must share block shape and dtype")
    if s.host and d.host:
        raise ValueError("at most one of src_blocks / dst_blocks may be host memory")
    dev = _move_device(s, d, src_ids)
    _require_index(src_ids, dev, "src_ids")
    _require_index(dst_ids, dev, "dst_ids")
    if src_ids.numel() != dst_ids.numel():
        raise ValueError("src_ids and dst_ids must have the same length")
    _launch_move("kvca_copy_paged", s.desc(src_ids), d.desc(dst_ids), 1, src_ids.numel(),
                 s.row_bytes, _host_flag(s, d), dev, check)


def exchange_blocks(actual_blocks: torch.Tensor, slot_ids: torch.Tensor, store: torch.Tensor,
                    spill_ids: torch.Tensor, fill_ids: torch.Tensor, *, check: bool | None = None) -> None:
    """For each j: ``store[spill_ids[j]] = actual_blocks[slot_ids[j]]`` (old
    bytes), then ``actual_blocks[slot_ids[j]] = store[fill_ids[j]]``, in one
    launch; negative spill / fill ids skip that part.  The eviction spill and
    the miss fill of a load (adapter.py:735-756, :779-787) in one pass: with
    ``store`` in pinned host memory both directions of the host link are
    busy at once.  Spilled and filled store rows must be disjoint."""
    a = _planes([actual_blocks], 1, "actual_blocks")
    st = _planes([store], 1, "store", allow_host=True)
    if a.row_bytes != st.row_bytes or a.dtype != st.dtype:
        raise ValueError("actual_blocks and store must share block shape and dtype")
    dev = _move_device(a, st, slot_ids)
    for t, name in ((slot_ids, "slot_ids"), (spill_ids, "spill_ids"), (fill_ids, "fill_ids")):
        _require_index(t, dev, name)
    k = slot_ids.numel()
    if spill_ids.numel() != k or fill_ids.numel() != k:
        raise ValueError("slot_ids, spill_ids and fill_ids must have the same length")
    if k == 0:
        return
    slots_desc, store_desc = a.desc(slot_ids), st.desc(spill_ids)
    with _on(dev):
        rc = _lib_handle.kvca_exchange(ctypes.byref(slots_desc), ctypes.byref(store_desc),
                                       _ptr(fill_ids), k, a.row_bytes,
                                       _lib.KVCA_FLAG_SKIP_NEGATIVE | _host_flag(st), _ptr(_status(dev)), _stream(dev))
    _host_rc(rc, "exchange_blocks")
    _maybe_check(dev, check, "exchange_blocks")


def _chunks_of(k: int, per_chunk: int | None, what: str) -> tuple[int, int]:
    per = k if per_chunk is None else int(per_chunk)
    if per < 1 or (k and k % per):
        raise ValueError(f"{what} ({k}) must be a positive multiple of the chunk length ({per})")
    return (k // per if per else 0), per


def gather_layers(caches: Sequence[torch.Tensor], slot_ids: torch.Tensor,
                  out: torch.Tensor | None = None, *, blocks_per_chunk: int | None = None,
                  check: bool | None = None) -> torch.Tensor:
    """Gather blocks ``slot_ids`` of every plane (layer x K/V) in one launch into
    chunks ``(num_chunks, num_planes, blocks_per_chunk, *block)``: per plane,
    ``cache.index_select(0, slot_ids)`` (adapter.py:543)."""
    pl = _planes(caches, 1, "caches")
    _require_index(slot_ids, pl.device, "slot_ids")
    k = slot_ids.numel()
    nc, cb = _chunks_of(k, blocks_per_chunk, "len(slot_ids)") if k else (0, max(1, blocks_per_chunk or 1))
    P = len(pl.planes)
    out = _chunk_tensor(out, (nc, P, cb, *pl.row_shape), pl.dtype, pl.device, "out")
    _launch_move("kvca_gather", pl.desc(slot_ids), _chunk_desc(out, cb, P, pl.row_bytes), P, k,
                 pl.row_bytes, _host_flag(out), pl.device, check)
    return out


def scatter_layers(caches: Sequence[torch.Tensor], slot_ids: torch.Tensor, chunks: torch.Tensor,
                   *, blocks_per_chunk: int | None = None, check: bool | None = None) -> None:
    """Inverse of gather_layers: per plane ``cache.index_copy_(0, slot_ids, ...)``."""
    pl = _planes(caches, 1, "caches")
    _require_index(slot_ids, pl.device, "slot_ids")
    k = slot_ids.numel()
    nc, cb = _chunks_of(k, blocks_per_chunk, "len(slot_ids)") if k else (0, max(1, blocks_per_chunk or 1))
    P = len(pl.planes)
    _chunk_tensor(chunks, (nc, P, cb, *pl.row_shape), pl.dtype, pl.device, "chunks")
    _launch_move("kvca_scatter", _chunk_desc(chunks, cb, P, pl.row_bytes), pl.desc(slot_ids), P,
                 k, pl.row_bytes, _host_flag(chunks), pl.device, check)


def gather_tokens(caches: Sequence[torch.Tensor], slot_mapping: torch.Tensor,
                  out: torch.Tensor | None = None, *, tokens_per_chunk: int | None = None,
                  check: bool | None = None) -> torch.Tensor:
    """Token rows ``slot_mapping[t]`` (= block * block_size + offset,
    adapter.py:1275-1285) of every plane ``(num_blocks, block_size, *row)`` into
    chunks ``(num_chunks, num_planes, tokens_per_chunk, *row)``.  Negative
    mappings are padding: their rows are left untouched in ``out``."""
    pl = _planes(caches, 2, "caches")
    _require_index(slot_mapping, pl.device, "slot_mapping")
    t = slot_mapping.numel()
    nc, tpc = _chunks_of(t, tokens_per_chunk, "len(slot_mapping)") if t else (0, max(1, tokens_per_chunk or 1))
    P = len(pl.planes)
    out = _chunk_tensor(out, (nc, P, tpc, *pl.row_shape), pl.dtype, pl.device, "out")
    _launch_move("kvca_gather", pl.desc(slot_mapping), _chunk_desc(out, tpc, P, pl.row_bytes), P,
                 t, pl.row_bytes, _lib.KVCA_FLAG_SKIP_NEGATIVE | _host_flag(out), pl.device, check)
    return out


def scatter_tokens(caches: Sequence[torch.Tensor], slot_mapping: torch.Tensor, chunks: torch.Tensor,
                   *, tokens_per_chunk: int | None = None, check: bool | None = None) -> None:
    """reshape-and-cache: token row t of every plane goes to ``slot_mapping[t]``;
    negative mappings are skipped."""
    pl = _planes(caches, 2, "caches")
    _require_index(slot_mapping, pl.device, "slot_mapping")
    t = slot_mapping.numel()
    nc, tpc = _chunks_of(t, tokens_per_chunk, "len(slot_mapping)") if t else (0, max(1, tokens_per_chunk or 1))
    P = len(pl.planes)
    _chunk_tensor(chunks, (nc, P, tpc, *pl.row_shape), pl.dtype, pl.device, "chunks")
    _launch_move("kvca_scatter", _chunk_desc(chunks, tpc, P, pl.row_bytes), pl.desc(slot_mapping),
                 P, t, pl.row_bytes, _lib.KVCA_FLAG_SKIP_NEGATIVE | _host_flag(chunks), pl.device, check)


def scatter_tokens_gather_layers(token_caches, slot_mapping: torch.Tensor, chunks: torch.Tensor, block_caches,
                                 slot_ids: torch.Tensor, out: torch.Tensor, *, tokens_per_chunk: int | None = None,
                                 blocks_per_chunk: int | None = None, inputs_ready: bool = False,
                                 check: bool | None = None) -> None:
    """``scatter_tokens(token_caches, slot_mapping, chunks)`` and
    ``gather_layers(block_caches, slot_ids, out)`` in one launch
    (kvca_scatter_gather).  The two moves must touch disjoint bytes: nothing
    orders one before the other.  A decode step's token scatter and the spill
    gather of the blocks the next step evicts (which this step does not
    write) are such a pair.  ``inputs_ready`` (KVCA_FLAG_INPUTS_READY): no
    kernel that may still run when this launch starts writes ``chunks``,
    ``slot_mapping`` or ``slot_ids`` (true in a chain of these calls whose
    inputs were made before it), so the launch reads them while the
    launches before it drain."""
    tp = _planes(token_caches, 2, "token_caches")
    bp = _planes(block_caches, 1, "block_caches")
    dev = tp.device
    if bp.device != dev:
        raise ValueError("token_caches and block_caches must be on one device")
    _require_index(slot_mapping, dev, "slot_mapping")
    _require_index(slot_ids, dev, "slot_ids")
    t = slot_mapping.numel()
    nc, tpc = _chunks_of(t, tokens_per_chunk, "len(slot_mapping)") if t else (0, max(1, tokens_per_chunk or 1))
    P = len(tp.planes)
    _chunk_tensor(chunks, (nc, P, tpc, *tp.row_shape), tp.dtype, dev, "chunks")
    k = slot_ids.numel()
    gc, cb = _chunks_of(k, blocks_per_chunk, "len(slot_ids)") if k else (0, max(1, blocks_per_chunk or 1))
    Q = len(bp.planes)
    _chunk_tensor(out, (gc, Q, cb, *bp.row_shape), bp.dtype, dev, "out")
    if t == 0 and k == 0:
        return
    ready = _lib.KVCA_FLAG_INPUTS_READY if inputs_ready else 0
    s_src, s_dst = _chunk_desc(chunks, tpc, P, tp.row_bytes), tp.desc(slot_mapping)
    g_src, g_dst = bp.desc(slot_ids), _chunk_desc(out, cb, Q, bp.row_bytes)
    with _on(dev):
        rc = _lib_handle.kvca_scatter_gather(
            ctypes.byref(s_src), ctypes.byref(s_dst), P, t, tp.row_bytes, ctypes.byref(g_src), ctypes.byref(g_dst),
            Q, k, bp.row_bytes, _lib.KVCA_FLAG_SKIP_NEGATIVE | ready, ready, _ptr(_status(dev)), _stream(dev))
    _host_rc(rc, "scatter_tokens_gather_layers")
    _maybe_check(dev, check, "scatter_tokens_gather_layers")


_cycle_scratches: dict[tuple, torch.Tensor] = {}


def _cycle_scratch(dev: torch.device, num_blocks: int) -> torch.Tensor:
    """kvca_move_cycle's scratch for this (device, stream, cache size): zeroed
    once, kept for reuse (the launches keep it consistent)."""
    words = int(_lib_handle.kvca_move_cycle_scratch_bytes(num_blocks)) // 8
    key = (_index(dev), _stream(dev).value or 0, words)
    buf = _cycle_scratches.get(key)
    if buf is None:
        buf = torch.zeros(words, dtype=torch.int64, device=dev)
        _cycle_scratches[key] = buf
    return buf


def move_cycle(token_caches, slot_mapping: torch.Tensor, token_rows: torch.Tensor, block_caches,
               victims: torch.Tensor, offsets: torch.Tensor, spill: torch.Tensor, *, blocks_per_chunk: int = 1,
               check: bool | None = None) -> None:
    """The moves of a booked decode cycle in one launch (kvca_move_cycle).
    For each step q of ``slot_mapping`` (``(num_steps, num_seqs)``, as
    ``append_steps`` writes it), in order: the spill gather of
    ``victims[offsets[q]:offsets[q + 1]]`` into rows ``offsets[q]`` .. of
    ``spill`` (``gather_layers``' chunk layout, ``blocks_per_chunk`` rows per
    chunk), then the scatter of step q's token rows (``token_rows`` in
    ``scatter_tokens``' chunk layout with ``num_seqs`` tokens per chunk:
    ``(num_steps, P, num_seqs, *row)``, or ``(1, P, num_seqs, *row)`` to
    scatter the same rows every step) through ``slot_mapping[q]``.
    ``offsets``: int64 on the device, ``num_steps + 1`` entries from 0.  Rows
    wait for earlier steps only where they depend on them; slots must be
    distinct across the call, negative slots and victims are skipped."""
    tp = _planes(token_caches, 2, "token_caches")
    bp = _planes(block_caches, 1, "block_caches")
    dev = tp.device
    if bp.device != dev:
        raise ValueError("token_caches and block_caches must be on one device")
    if slot_mapping.dim() != 2:
        raise ValueError("slot_mapping must be a (num_steps, num_seqs) tensor")
    steps, seqs = slot_mapping.shape
    _require_index(slot_mapping.view(-1) if slot_mapping.is_contiguous() else slot_mapping, dev, "slot_mapping")
    _require_index(victims, dev, "victims")
    _require_index(offsets, dev, "offsets")
    if offsets.numel() != steps + 1:
        raise ValueError("offsets must have num_steps + 1 entries")
    P = len(tp.planes)
    if len(bp.planes) != P:
        raise ValueError("token_caches and block_caches must have the same planes")
    if token_rows.dim() < 1 or token_rows.shape[0] not in (1, steps):
        raise ValueError("token_rows must be (num_steps or 1, P, num_seqs, *row)")
    _chunk_tensor(token_rows, (token_rows.shape[0], P, seqs, *tp.row_shape), tp.dtype, dev, "token_rows")
    cb = int(blocks_per_chunk)
    if cb < 1 or spill.dim() < 3 or spill.shape[2] != cb:
        raise ValueError("spill must be (chunks, P, blocks_per_chunk, *block_row)")
    _chunk_tensor(spill, (spill.shape[0], P, cb, *bp.row_shape), bp.dtype, dev, "spill")
    if token_rows.device != dev or spill.device != dev:
        raise ValueError("token_rows and spill must be on the cache's device")
    if steps == 0 or seqs == 0:
        return
    rb = tp.row_bytes
    tokens = _lib.ChunkDesc(token_rows.data_ptr(), seqs, 0 if token_rows.shape[0] == 1 else P * seqs * rb, rb,
                            seqs * rb)
    with _on(dev):
        rc = _lib_handle.kvca_move_cycle(
            ctypes.byref(tokens), ctypes.byref(tp.desc(slot_mapping)), rb, ctypes.byref(bp.desc(victims)),
            victims.numel(), ctypes.byref(_chunk_desc(spill, cb, P, bp.row_bytes)), bp.row_bytes, P, _ptr(offsets),
            steps, seqs,
            spill.shape[0] * cb, _lib.KVCA_FLAG_SKIP_NEGATIVE, _ptr(_cycle_scratch(dev, tp.num_blocks)),
            _ptr(_status(dev)), _stream(dev))
    _host_rc(rc, "move_cycle")
    _maybe_check(dev, check, "move_cycle")


def copy_tokens(src_caches, src_mapping: torch.Tensor, dst_caches, dst_mapping: torch.Tensor, *,
                check: bool | None = None) -> None:
    """Token row ``src_mapping[t]`` of every source plane to token row
    ``dst_mapping[t]`` of the matching destination plane, in one launch; both
    sides are ``(num_blocks, block_size, *row)`` planes (block sizes may
    differ), one side may be pinned host memory, negative mappings on either
    side skip the token."""
    s = _planes(src_caches, 2, "src_caches", allow_host=True)
    d = _planes(dst_caches, 2, "dst_caches", allow_host=True)
    if len(s.planes) != len(d.planes) or s.row_bytes != d.row_bytes or s.dtype != d.dtype:
        raise ValueError("src and dst planes must match in count, row shape and dtype")
    if s.host and d.host:
        raise ValueError("at most one side may be host memory")
    dev = _move_device(s, d, src_mapping)
    _require_index(src_mapping, dev, "src_mapping")
    _require_index(dst_mapping, dev, "dst_mapping")
    if src_mapping.numel() != dst_mapping.numel():
        raise ValueError("src_mapping and dst_mapping must have the same length")
    _launch_move("kvca_copy_paged", s.desc(src_mapping), d.desc(dst_mapping), len(s.planes), src_mapping.numel(),
                 s.row_bytes, _lib.KVCA_FLAG_SKIP_NEGATIVE | _host_flag(s, d), dev, check)


def _pool_rows(memory_objs: Sequence[torch.Tensor], shape: torch.Size, dtype) -> tuple[torch.Tensor, torch.Tensor]:
    """The buffer the memory objects are rows of, as ``(n_rows, *shape)``, and
    each object's row index.  Every object must be a contiguous ``shape``
    view at a whole-row offset of one buffer (a pinned pool, a host tier's
    arena, or a device tensor)."""
    first = memory_objs[0]
    storage = first.untyped_storage()
    base = storage.data_ptr()
    row_bytes = math.prod(shape) * first.element_size()
    rows = []
    for m in memory_objs:
        if (m.untyped_storage().data_ptr() != base or m.dtype != dtype or tuple(m.shape) != tuple(shape)
                or not m.is_contiguous() or (m.data_ptr() - base) % row_bytes):
            raise ValueError("memory objects must be contiguous rows of one buffer, all of the transfer shape")
        rows.append((m.data_ptr() - base) // row_bytes)
    n_rows = storage.nbytes() // row_bytes
    pool = torch.empty(0, dtype=dtype, device=first.device).set_(storage, 0, (n_rows, *shape))
    return pool, torch.tensor(rows, dtype=torch.int64)


def batched_fused_single_layer_kv_transfer(memory_objs: Sequence[torch.Tensor], staging_cache, kv_blocks: torch.Tensor,
                                           slot_mapping: torch.Tensor, chunk_offsets: Sequence[int],
                                           chunk_sizes: Sequence[int], to_memory_objs: bool, num_layers: int = 1,
                                           token_major: bool = True, reserved: bool = False, *,
                                           check: bool | None = None) -> None:
    """Token-granular K/V transfer of one layer between merged paged blocks and
    per-chunk memory objects, the op the reference calls on its accelerator
    host path (``lmcache_ascend.c_ops``, adapter.py:1208-1219 to the memory
    objects, :1231-1242 back), as one copy kernel over both K and V.

    ``kv_blocks`` ``(m, *block)`` with a merged block ``(bs, 2, H, D)``
    (``token_major``) or ``(2, bs, H, D)``; token slot s is token ``s % bs`` of
    block ``s // bs``.  Memory object i, of transfer shape ``(T, 2, H*D)`` or
    ``(2, T, H*D)`` with T = ``chunk_sizes[i]``, holds the tokens
    ``slot_mapping[chunk_offsets[i] : chunk_offsets[i] + T]`` in order.  The
    objects must be rows of one buffer (pinned host or device), as a pinned
    pool hands them out.  ``staging_cache`` is not needed (rows move
    directly) and ignored; ``num_layers`` must be 1; ``reserved`` is ignored.
    Negative slots are skipped."""
    from .adapter import _MergedKVBlockLayout

    if num_layers != 1:
        raise ValueError("single-layer transfer: num_layers must be 1")
    layout = _MergedKVBlockLayout.detect(kv_blocks.shape[1:])
    if layout is None or layout.token_major != bool(token_major):
        raise ValueError("kv_blocks must be merged K/V blocks of the stated token order")
    n = len(memory_objs)
    if n == 0:
        return
    if len(chunk_offsets) != n or len(chunk_sizes) != n or len(set(int(c) for c in chunk_sizes)) != 1:
        raise ValueError("one offset and one (common) size per memory object")
    T = int(chunk_sizes[0])
    tshape = torch.Size((T, 2, layout.hidden_dim) if layout.token_major else (2, T, layout.hidden_dim))
    pool, rows = _pool_rows(memory_objs, tshape, kv_blocks.dtype)
    dev = kv_blocks.device
    _require_index(slot_mapping, dev, "slot_mapping")
    offs = torch.tensor([int(o) for o in chunk_offsets], dtype=torch.int64)
    if int(offs.min()) < 0 or int(offs.max()) + T > slot_mapping.numel():
        raise ValueError("chunks must lie inside slot_mapping")
    t = torch.arange(T, dtype=torch.int64)
    kv_map = slot_mapping.index_select(0, (offs.view(-1, 1) + t.view(1, -1)).view(-1).to(dev))
    pool_map = (rows.view(-1, 1) * T + t.view(1, -1)).view(-1).to(dev)
    kv_planes = layout.token_planes(kv_blocks)
    if layout.token_major:
        pool_planes = [pool[:, :, 0], pool[:, :, 1]]
    else:
        pool_planes = [pool[:, 0], pool[:, 1]]
    if to_memory_objs:
        copy_tokens(kv_planes, kv_map, pool_planes, pool_map, check=check)
    else:
        copy_tokens(pool_planes, pool_map, kv_planes, kv_map, check=check)
