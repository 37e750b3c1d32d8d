"""KVCacheAdapter on B200: the reference's operator API with every metadata
update, clock sweep and KV byte move running in the sm_100a kernels.

Public surface and behaviour follow the reference's adapter.py:
``KVCacheAdapter`` (adapter.py:126-677), ``InMemoryBlockStoreBackend``
(adapter.py:679-833), ``_MergedKVBlockLayout`` (adapter.py:81-123), the
packed slot-meta codec (adapter.py:17-36, :1414-1432) and the error types
(adapter.py:50-59).

Differences, all on purpose:
  * CUDA ``actual_blocks`` go through the packed-slot-meta op set, so pin
    and usage updates persist (the reference's CUDA branch hands its kernels
    derived temporaries and loses them; its NPU branch does what is done
    here).
  * Gathers and scatters of KV blocks run in the row-mover kernels instead of
    ``index_select`` / ``index_copy_``.
  * There is no pure-torch path: a CUDA adapter without the native library
    raises, and CPU tensors need an explicitly supplied op set (``native_ext``),
    which the test suite uses to check this orchestration against the
    reference on CPU.
"""
from __future__ import annotations

import functools
import importlib
import math
import os
import time
from dataclasses import dataclass
from typing import Any, Protocol

import torch

from .errors import BlockNotFoundError, InsufficientCapacityError, KVCacheAdapterError

ID_DTYPE = torch.int64
_SLOT_META_BITS = int(os.getenv("KVCA_SLOT_META_BITS", "8"))
if _SLOT_META_BITS == 8:
    SLOT_META_DTYPE = torch.uint8
    PIN_COUNT_BITS = 4
    USAGE_COUNT_BITS = 4
elif _SLOT_META_BITS == 16:
    SLOT_META_DTYPE = torch.uint16
    PIN_COUNT_BITS = 8
    USAGE_COUNT_BITS = 8
else:
    raise ValueError("KVCA_SLOT_META_BITS must be 8 or 16")

USAGE_DTYPE = SLOT_META_DTYPE
PIN_COUNT_DTYPE = SLOT_META_DTYPE
PIN_COUNT_MAX = (1 << PIN_COUNT_BITS) - 1
USAGE_COUNT_MAX = (1 << USAGE_COUNT_BITS) - 1
_PIN_COUNT_MASK = PIN_COUNT_MAX
_USAGE_COUNT_MASK = USAGE_COUNT_MAX
_USAGE_COUNT_SHIFT = PIN_COUNT_BITS

STATE_FREE = 0
STATE_RESERVED = 1
STATE_LOADING = 2
STATE_RESIDENT = 3
STATE_NAMES = {
    STATE_FREE: "free",
    STATE_RESERVED: "reserved",
    STATE_LOADING: "loading",
    STATE_RESIDENT: "resident",
}

__all__ = [
    "KVCacheAdapter",
    "InMemoryBlockStoreBackend",
    "BlockStoreBackend",
    "KVCacheAdapterError",
    "BlockNotFoundError",
    "HostTierBackend",
    "InsufficientCapacityError",
]


class BlockStoreBackend(Protocol):
    def save_blocks(self, logical_block_ids: torch.Tensor, block_data: torch.Tensor) -> None:
        ...

    def load_blocks(
        self,
        logical_block_ids: torch.Tensor,
        actual_blocks: torch.Tensor,
        physical_slot_ids: torch.Tensor,
    ) -> None:
        ...


@dataclass(frozen=True)
class _EvictionPlan:
    logical_block_ids: torch.Tensor
    payloads: torch.Tensor


@dataclass(frozen=True)
class _MergedKVBlockLayout:
    """Merged K/V block shape ``(bs, 2, *hidden)`` (token-major) or
    ``(2, bs, *hidden)`` (adapter.py:81-123)."""

    block_shape: torch.Size
    block_size: int
    hidden_dim: int
    token_major: bool

    @classmethod
    def detect(cls, block_shape) -> "_MergedKVBlockLayout | None":
        shape = torch.Size(block_shape)
        if len(shape) != 4:
            return None
        if shape[1] == 2:
            block_size, token_major = int(shape[0]), True
        elif shape[0] == 2:
            block_size, token_major = int(shape[1]), False
        else:
            return None
        hidden = int(shape[2]) * int(shape[3])
        return cls(block_shape=shape, block_size=block_size, hidden_dim=hidden, token_major=token_major)

    @property
    def transfer_shape(self) -> torch.Size:
        if self.token_major:
            return torch.Size((self.block_size, 2, self.hidden_dim))
        return torch.Size((2, self.block_size, self.hidden_dim))

    def flatten_block_batch(self, block_batch: torch.Tensor) -> torch.Tensor:
        return block_batch.contiguous().view((block_batch.shape[0],) + tuple(self.transfer_shape))

    def restore_block_tensor(self, stored_tensor: torch.Tensor) -> torch.Tensor:
        return stored_tensor.view(self.block_shape)

    def token_planes(self, actual_blocks: torch.Tensor) -> list[torch.Tensor]:
        """The K and V planes of a merged cache ``(m, *block_shape)`` as
        ``(m, block_size, hidden_dim)`` views for token-granular moves."""
        m = actual_blocks.shape[0]
        flat = actual_blocks.view(m, *self.transfer_shape)
        if self.token_major:
            return [flat[:, :, 0], flat[:, :, 1]]
        return [flat[:, 0], flat[:, 1]]

    def physical_slot_mapping(self, physical_slot_ids: torch.Tensor) -> torch.Tensor:
        """slot_mapping[i * bs + t] = slot[i] * bs + t (adapter.py:1275-1285)."""
        offsets = torch.arange(self.block_size, dtype=ID_DTYPE, device=physical_slot_ids.device)
        return (physical_slot_ids.reshape(-1, 1) * self.block_size + offsets.reshape(1, -1)).reshape(-1)

    def dense_slot_mapping(self, num_blocks: int, *, device: torch.device) -> torch.Tensor:
        """adapter.py:1266-1273."""
        return torch.arange(num_blocks * self.block_size, dtype=ID_DTYPE, device=device)

    def chunk_offsets(self, num_blocks: int) -> list[int]:
        """adapter.py:1287-1290."""
        return [i * self.block_size for i in range(num_blocks)]

    def chunk_sizes(self, num_blocks: int) -> list[int]:
        """adapter.py:1292-1295."""
        return [self.block_size] * num_blocks


class KVCacheAdapter:
    """Maps n logical ids onto m resident physical slots in ``actual_blocks``.

    Contract (adapter.py:127-134):
    - ``actual_blocks`` is the real ``(m, ...)`` resident tensor
    - ``logical_block_ids`` must be ``torch.int64`` on the same device as ``actual_blocks``
    - ``block_data`` must be on the same device/dtype/shape layout as ``actual_blocks``
    - callers serialize access; this adapter is not thread-safe
    """

    def __init__(
        self,
        num_actual_blocks: int,
        num_logical_blocks: int,
        actual_blocks: torch.Tensor,
        backend: BlockStoreBackend,
        *,
        prefer_native_extension: bool = True,
        prefer_cuda_extension: bool | None = None,
        native_ext: Any | None = None,
        pop_order: str | None = None,
    ) -> None:
        if prefer_cuda_extension is not None:
            prefer_native_extension = prefer_cuda_extension
        if not isinstance(actual_blocks, torch.Tensor):
            raise TypeError("actual_blocks must be torch.Tensor")
        if actual_blocks.ndim < 1:
            raise ValueError("actual_blocks must have a leading block dimension")
        if num_actual_blocks <= 0:
            raise ValueError("num_actual_blocks must be positive")
        if num_logical_blocks <= 0:
            raise ValueError("num_logical_blocks must be positive")
        if num_actual_blocks > num_logical_blocks:
            raise ValueError("num_actual_blocks must be <= num_logical_blocks")
        if actual_blocks.shape[0] != num_actual_blocks:
            raise ValueError("actual_blocks leading dimension must equal num_actual_blocks")

        self.num_actual_blocks = int(num_actual_blocks)
        self.num_logical_blocks = int(num_logical_blocks)
        self.actual_blocks = actual_blocks
        self.backend = backend
        self.pop_order = pop_order or os.getenv("KVCA_POP_ORDER", "grouped")

        device = actual_blocks.device
        self._platform = device.type
        self._logical_to_physical = torch.full((num_logical_blocks,), -1, dtype=ID_DTYPE, device=device)
        self._physical_to_logical = torch.full((num_actual_blocks,), -1, dtype=ID_DTYPE, device=device)
        self._slot_meta = torch.zeros((num_actual_blocks,), dtype=SLOT_META_DTYPE, device=device)
        self._search_start = torch.zeros((1,), dtype=ID_DTYPE, device=device)
        self._native_ext, self.runtime_path = self._detect_native_extension(
            prefer_native_extension=prefer_native_extension, native_ext=native_ext)
        # An op set with plan_load / plan_save runs the inspect -> split -> pop ->
        # eviction-plan part of load / save as one launch with one host sync.
        self._planned = all(callable(getattr(self._native_ext, n, None)) for n in ("plan_load", "plan_save"))
        self._session = None  # DeviceStoreSession over the backend's device store (see _store_session)
        self._session_key = None

    # -- views of the packed words (the reference's properties, adapter.py:185-203);
    # each read builds a new tensor, so writing to one changes nothing
    _pin_count = property(lambda self: _slot_meta_pin_counts(self._slot_meta))
    _usage_count = property(lambda self: _slot_meta_usage_counts(self._slot_meta))
    _reusable_mask = property(lambda self: _slot_meta_pin_counts(self._slot_meta).eq(0))

    @property
    def _slot_state(self) -> torch.Tensor:
        """STATE_RESIDENT for slots that hold a logical block, else STATE_FREE."""
        state = torch.full_like(self._physical_to_logical, STATE_FREE)
        return state.masked_fill_(self._physical_to_logical.ge(0), STATE_RESIDENT)

    # -- public API ---------------------------------------------------------

    def save(self, logical_block_ids: torch.Tensor, block_data: torch.Tensor) -> None:
        """adapter.py:205-255."""
        _require_id_tensor(logical_block_ids, name="logical_block_ids")
        _require_same_device(logical_block_ids, expected_device=self.actual_blocks.device, name="logical_block_ids")
        self._validate_logical_block_ids(logical_block_ids)
        _require_block_data_tensor(block_data, expected_blocks=logical_block_ids.shape[0], name="block_data")
        _require_same_device(block_data, expected_device=self.actual_blocks.device, name="block_data")
        _require_same_dtype(block_data, reference=self.actual_blocks, name="block_data")
        _require_trailing_shape(block_data, self.actual_blocks, name="block_data")
        if logical_block_ids.numel() == 0:
            return
        logical_block_ids = logical_block_ids.contiguous()
        if self._planned:
            store = self._device_store()
            if store is not None:
                self._save_device_store(logical_block_ids, block_data, store)
            else:
                self._save_planned(logical_block_ids, block_data)
            return

        current_physical, existing_mask, inspected_usage = self._inspect_save_requests(logical_block_ids)
        existing_positions = _positions(existing_mask)
        missing_positions = _positions(existing_mask, False)
        existing_physical = current_physical.index_select(0, existing_positions)
        missing_ids = logical_block_ids.index_select(0, missing_positions)
        allocated_physical = self._pop_reusable_slots(missing_ids.shape[0], blocked_slot_ids=existing_physical)

        selected_physical = current_physical.clone()
        if missing_ids.numel() > 0:
            selected_physical.index_copy_(0, missing_positions, allocated_physical)

        # pins and usage are read after the sweep, which may have aged usage
        final_pin_counts = _slot_meta_pin_counts(_take(self._slot_meta, selected_physical))
        final_usage_counts = inspected_usage
        if missing_ids.numel() > 0 and existing_physical.numel() > 0:
            final_usage_counts = torch.ones_like(logical_block_ids, dtype=torch.int32)
            final_usage_counts.index_copy_(
                0,
                existing_positions,
                _saturating_increment_usage(_slot_meta_usage_counts(_take(self._slot_meta, existing_physical)))
                .to(dtype=torch.int32),
            )
            final_usage_counts = final_usage_counts.to(dtype=USAGE_DTYPE)
        eviction_plan = self._build_eviction_plan(logical_block_ids, selected_physical)
        if eviction_plan.logical_block_ids.numel() > 0:
            self.backend.save_blocks(eviction_plan.logical_block_ids, eviction_plan.payloads)

        self._copy_into_actual_blocks(selected_physical, block_data)
        self._commit_save_metadata(
            evicted_logical_block_ids=eviction_plan.logical_block_ids,
            logical_block_ids=logical_block_ids,
            physical_slot_ids=selected_physical,
            final_pin_counts=final_pin_counts,
            final_usage_counts=final_usage_counts,
        )

    def load(self, logical_block_ids: torch.Tensor) -> torch.Tensor:
        """adapter.py:257-307."""
        _require_id_tensor(logical_block_ids, name="logical_block_ids")
        _require_same_device(logical_block_ids, expected_device=self.actual_blocks.device, name="logical_block_ids")
        self._validate_logical_block_ids(logical_block_ids)
        if logical_block_ids.numel() == 0:
            return torch.empty_like(logical_block_ids)
        logical_block_ids = logical_block_ids.contiguous()
        if self._planned:
            store = self._device_store()
            if store is not None:
                return self._load_device_store(logical_block_ids, store)
            return self._load_planned(logical_block_ids)

        current_physical, resident_mask, updated_pins, updated_usage = self._inspect_load_requests(logical_block_ids)
        resident_positions = _positions(resident_mask)
        miss_positions = _positions(resident_mask, False)
        hit_slot_ids = current_physical.index_select(0, resident_positions)
        miss_logical_ids = logical_block_ids.index_select(0, miss_positions)
        miss_slot_ids = self._pop_reusable_slots(miss_logical_ids.shape[0], blocked_slot_ids=hit_slot_ids)
        eviction_plan = self._build_eviction_plan(miss_logical_ids, miss_slot_ids)

        if eviction_plan.logical_block_ids.numel() > 0:
            self.backend.save_blocks(eviction_plan.logical_block_ids, eviction_plan.payloads)
        if miss_logical_ids.numel() > 0:
            self.backend.load_blocks(miss_logical_ids, self.actual_blocks, miss_slot_ids)

        if miss_logical_ids.numel() > 0 and hit_slot_ids.numel() > 0:
            hit_usage = _saturating_increment_usage(_slot_meta_usage_counts(_take(self._slot_meta, hit_slot_ids)))
        else:
            hit_usage = _take(updated_usage, resident_positions)
        miss_usage = torch.ones((miss_slot_ids.shape[0],), dtype=USAGE_DTYPE, device=self.actual_blocks.device)
        result_physical = current_physical
        if miss_positions.numel() > 0:
            result_physical = current_physical.clone()
            result_physical.index_copy_(0, miss_positions, miss_slot_ids)
        self._commit_load_metadata(
            evicted_logical_block_ids=eviction_plan.logical_block_ids,
            miss_logical_block_ids=miss_logical_ids,
            miss_physical_slot_ids=miss_slot_ids,
            hit_slot_ids=hit_slot_ids,
            hit_pin_counts=updated_pins.index_select(0, resident_positions),
            hit_usage_counts=hit_usage,
            miss_usage_counts=miss_usage,
        )
        return result_physical

    def release(self, logical_block_ids: torch.Tensor) -> None:
        """adapter.py:309-336: pin - 1 per id (a pin of 0 wraps to the field max)."""
        _require_id_tensor(logical_block_ids, name="logical_block_ids")
        _require_same_device(logical_block_ids, expected_device=self.actual_blocks.device, name="logical_block_ids")
        self._validate_logical_block_ids(logical_block_ids)
        if logical_block_ids.numel() == 0:
            return
        self._native_ext.release_metadata(
            self._logical_to_physical, self._slot_meta, logical_block_ids.contiguous(), check=True)

    def get_actual_block(self, physical_slot_id: int) -> torch.Tensor:
        self._validate_physical_slot_id(physical_slot_id)
        return self.actual_blocks[physical_slot_id]

    def debug_snapshot(self) -> dict[str, object]:
        """A host copy of the adapter's state under the keys the reference's
        snapshot uses (adapter.py:342-357): resident logical id -> slot, the
        unpinned slots in scan order, each slot's state name, pin counts and
        the cache rows."""
        l2p = self._logical_to_physical.detach().cpu()
        mapped = l2p.ge(0).nonzero().flatten()
        snap: dict[str, object] = {"runtime_path": self.runtime_path}
        snap["logical_to_physical"] = dict(zip(mapped.tolist(), l2p[mapped].tolist()))
        snap["lru_unpinned"] = self._ordered_reusable_slots().detach().cpu().tolist()
        snap["slot_state"] = list(map(STATE_NAMES.__getitem__, self._slot_state.cpu().tolist()))
        snap["pin_count"] = self._pin_count.cpu().clone()
        snap["actual_blocks"] = self.actual_blocks.detach().cpu().clone()
        return snap

    def shutdown(self) -> None:
        backend_shutdown = getattr(self.backend, "shutdown", None)
        if callable(backend_shutdown):
            backend_shutdown()
            return
        backend_close = getattr(self.backend, "close", None)
        if callable(backend_close):
            backend_close()

    # -- internals ------------------------------------------------------------

    def _detect_native_extension(self, *, prefer_native_extension: bool, native_ext: Any | None) -> tuple[Any, str]:
        """adapter.py:369-391, CUDA only."""
        if native_ext is not None:
            return native_ext, f"{self._platform}_ext_meta"
        if self._platform == "cuda":
            if not prefer_native_extension:
                raise RuntimeError("CUDA actual_blocks require kv_cache_adapter_cuda; strict CUDA path is disabled")
            ext = _load_cuda_extension_module()
            if ext is None:
                raise RuntimeError("CUDA actual_blocks require kv_cache_adapter_cuda, but the extension is unavailable")
            return ext, "cuda_ext_meta"
        raise RuntimeError(
            f"kv_cache_adapter_b200 serves CUDA actual_blocks; got device {self._platform!r} "
            "(pass native_ext= to supply an op set for other devices)")

    def _plan(self, op: str, ids: torch.Tensor):
        try:
            return getattr(self._native_ext, op)(
                self._logical_to_physical, self._physical_to_logical, self._slot_meta, self._search_start, ids,
                order=self.pop_order)
        except IndexError as exc:
            raise ValueError(f"logical block ids must be inside [0, {self.num_logical_blocks})") from exc

    def _device_store(self):
        """The backend's device-resident store (storage, present, scratch) when
        it offers one for these actual_blocks and the op set drives it."""
        offer = getattr(self.backend, "device_store", None)
        if not callable(offer) or not callable(getattr(self._native_ext, "load_device_store", None)):
            return None
        if not self.actual_blocks.is_contiguous():
            return None
        return offer(self.actual_blocks)

    def _store_session(self, store):
        """The op set's session over (these tables, this store), kept while the
        backend offers the same store tensors; None without sessions."""
        key = tuple(id(t) for t in store)
        if self._session is not None and self._session_key == key:
            return self._session
        make = getattr(self._native_ext, "DeviceStoreSession", None)
        if make is None:
            return None
        self._session = make(self._logical_to_physical, self._physical_to_logical, self._slot_meta,
                             self._search_start, self.actual_blocks, *store, order=self.pop_order)
        self._session_key = key
        return self._session

    def _load_device_store(self, ids: torch.Tensor, store) -> torch.Tensor:
        """load (adapter.py:257-307) with the backend's spill and fill on the
        device: one enqueued sequence and one host read."""
        storage, present, scratch = store
        session = self._store_session(store)
        try:
            if session is not None:
                result, counts = session.load(ids)
            else:
                result, counts = self._native_ext.load_device_store(
                    self._logical_to_physical, self._physical_to_logical, self._slot_meta, self._search_start, ids,
                    self.actual_blocks, storage, present, scratch, order=self.pop_order)
        except IndexError as exc:
            raise ValueError(f"logical block ids must be inside [0, {self.num_logical_blocks})") from exc
        except BlockNotFoundError as exc:
            self.backend.note_device_ops(saved=exc.counts[2] > 0, loaded=True)
            raise
        self.backend.note_device_ops(saved=counts[2] > 0, loaded=counts[1] > 0)
        return result

    def _save_device_store(self, ids: torch.Tensor, block_data: torch.Tensor, store) -> None:
        """save (adapter.py:205-255) with the backend's spill on the device."""
        storage, present, scratch = store
        session = self._store_session(store)
        try:
            if session is not None:
                counts = session.save(ids, block_data.contiguous())
            else:
                counts = self._native_ext.save_device_store(
                    self._logical_to_physical, self._physical_to_logical, self._slot_meta, self._search_start, ids,
                    block_data.contiguous(), self.actual_blocks, storage, present, scratch, order=self.pop_order)
        except IndexError as exc:
            raise ValueError(f"logical block ids must be inside [0, {self.num_logical_blocks})") from exc
        self.backend.note_device_ops(saved=counts[2] > 0, loaded=False)

    def _load_planned(self, ids: torch.Tensor) -> torch.Tensor:
        """load (adapter.py:257-307) with the planning steps in one device call;
        the backend calls, the row movers and the commit follow unchanged."""
        plan = self._plan("plan_load", ids)
        # slots from the plan are in range by construction: the launches below
        # leave their status to the next read (the backend's or the next plan's)
        if plan.evict_ids.numel() > 0:
            self.backend.save_blocks(
                plan.evict_ids, self._native_ext.gather_blocks(self.actual_blocks, plan.evict_slots, check=False))
        if plan.miss_ids.numel() > 0:
            self.backend.load_blocks(plan.miss_ids, self.actual_blocks, plan.victims)
        miss_usage = torch.ones((plan.victims.shape[0],), dtype=USAGE_DTYPE, device=self.actual_blocks.device)
        self._native_ext.commit_load_metadata(
            self._logical_to_physical, self._physical_to_logical, self._slot_meta, plan.evict_ids, plan.miss_ids,
            plan.victims, plan.hit_slots, plan.hit_pins, plan.hit_usage, miss_usage, check=False)
        return plan.result

    def _save_planned(self, ids: torch.Tensor, block_data: torch.Tensor) -> None:
        """save (adapter.py:205-255) with the planning steps in one device call."""
        plan = self._plan("plan_save", ids)
        if plan.evict_ids.numel() > 0:
            self.backend.save_blocks(
                plan.evict_ids, self._native_ext.gather_blocks(self.actual_blocks, plan.evict_slots, check=False))
        self._native_ext.scatter_blocks(self.actual_blocks, plan.move_slots, block_data.contiguous(),
                                        skip_negative=True, check=False)
        self._native_ext.commit_save_metadata(
            self._logical_to_physical, self._physical_to_logical, self._slot_meta, plan.evict_ids, ids,
            plan.selected, plan.final_pins, plan.final_usage, check=False)

    def _inspect_load_requests(self, ids: torch.Tensor):
        try:
            return tuple(self._native_ext.inspect_load_requests(
                self._logical_to_physical, self._slot_meta, ids, check=True))
        except IndexError as exc:
            raise ValueError(f"logical block ids must be inside [0, {self.num_logical_blocks})") from exc

    def _inspect_save_requests(self, ids: torch.Tensor):
        try:
            return tuple(self._native_ext.inspect_save_requests(
                self._logical_to_physical, self._slot_meta, ids, check=True))
        except IndexError as exc:
            raise ValueError(f"logical block ids must be inside [0, {self.num_logical_blocks})") from exc

    def _pop_reusable_slots(self, count: int, *, blocked_slot_ids: torch.Tensor) -> torch.Tensor:
        """adapter.py:472-525 through the native clock sweep."""
        if count == 0:
            return self._logical_to_physical[:0]
        return self._native_ext.pop_reusable_slots(
            self._slot_meta, self._search_start, blocked_slot_ids.contiguous(), count, order=self.pop_order)

    def _build_eviction_plan(self, logical_block_ids: torch.Tensor, physical_slot_ids: torch.Tensor) -> _EvictionPlan:
        """adapter.py:527-544; the payload gather runs in the row mover."""
        if physical_slot_ids.numel() == 0:
            return _EvictionPlan(logical_block_ids[:0], self.actual_blocks[:0])
        previous_logical_ids = self._physical_to_logical.index_select(0, physical_slot_ids)
        eviction_mask = (previous_logical_ids >= 0) & (previous_logical_ids != logical_block_ids)
        eviction_positions = _positions(eviction_mask)
        eviction_logical_ids = previous_logical_ids.index_select(0, eviction_positions)
        eviction_slot_ids = physical_slot_ids.index_select(0, eviction_positions)
        payloads = self._native_ext.gather_blocks(self.actual_blocks, eviction_slot_ids)
        return _EvictionPlan(eviction_logical_ids, payloads)

    def _commit_load_metadata(self, *, evicted_logical_block_ids, miss_logical_block_ids, miss_physical_slot_ids,
                              hit_slot_ids, hit_pin_counts, hit_usage_counts, miss_usage_counts) -> None:
        self._native_ext.commit_load_metadata(
            self._logical_to_physical, self._physical_to_logical, self._slot_meta,
            evicted_logical_block_ids.contiguous(), miss_logical_block_ids.contiguous(),
            miss_physical_slot_ids.contiguous(), hit_slot_ids.contiguous(), hit_pin_counts.contiguous(),
            hit_usage_counts.contiguous(), miss_usage_counts.contiguous(), check=True)

    def _commit_save_metadata(self, *, evicted_logical_block_ids, logical_block_ids, physical_slot_ids,
                              final_pin_counts, final_usage_counts) -> None:
        self._native_ext.commit_save_metadata(
            self._logical_to_physical, self._physical_to_logical, self._slot_meta,
            evicted_logical_block_ids.contiguous(), logical_block_ids.contiguous(), physical_slot_ids.contiguous(),
            final_pin_counts.contiguous(), final_usage_counts.contiguous(), check=True)

    def _copy_into_actual_blocks(self, physical_slot_ids: torch.Tensor, block_data: torch.Tensor) -> None:
        """adapter.py:653-656 through the row mover.  index_copy_ applied in
        order leaves the last row of a repeated slot, so earlier repeats are
        dropped before the (unordered) scatter."""
        if physical_slot_ids.numel() == 0:
            return
        self._native_ext.scatter_blocks(self.actual_blocks, _last_occurrences(physical_slot_ids, self.num_actual_blocks),
                                        block_data.contiguous(), skip_negative=True)

    def _ordered_reusable_slots(self) -> torch.Tensor:
        scan_order = (self._search_start[0] + torch.arange(
            self.num_actual_blocks, device=self.actual_blocks.device, dtype=ID_DTYPE)) % self.num_actual_blocks
        return scan_order[self._reusable_mask.index_select(0, scan_order)]

    def _validate_logical_block_ids(self, logical_block_ids: torch.Tensor) -> None:
        """adapter.py:666-672; device ids are checked by the inspect kernels."""
        if logical_block_ids.numel() == 0 or logical_block_ids.device.type != "cpu":
            return
        if torch.any(logical_block_ids < 0) or torch.any(logical_block_ids >= self.num_logical_blocks):
            raise ValueError(f"logical block ids must be inside [0, {self.num_logical_blocks})")

    def _validate_physical_slot_id(self, physical_slot_id: int) -> None:
        if physical_slot_id < 0 or physical_slot_id >= self.num_actual_blocks:
            raise ValueError(f"physical slot id {physical_slot_id} is outside [0, {self.num_actual_blocks})")


class InMemoryBlockStoreBackend:
    """Dense logical-id-indexed block store (adapter.py:679-833).

    CUDA storage moves bytes with the row-mover kernels (``copy_blocks``
    fuses the reference's index_select + index_copy_ of load_blocks).  A
    store on the host stays a host store: it uses torch host indexing and
    one host<->device copy per call.

    ``host_tier=True`` keeps the rows in pinned host memory instead and moves
    them with the GPU (``device``, else the first CUDA tensor it is given):
    saves scatter device rows straight into the pinned rows and loads copy
    pinned rows straight into ``actual_blocks``, one kernel each, over the
    host link; the present mask stays on the GPU.  Host-side reads of the
    rows (``snapshot``) synchronise with that GPU first.
    """

    def __init__(
        self,
        initial_data: dict[int, torch.Tensor] | torch.Tensor | None = None,
        *,
        num_logical_blocks: int | None = None,
        present_mask: torch.Tensor | None = None,
        save_delay_s: float = 0.0,
        load_delay_s: float = 0.0,
        record_device_ops: bool = False,
        ops: Any | None = None,
        host_tier: bool = False,
        device: torch.device | str | None = None,
    ) -> None:
        self._ops = ops
        self._record_device_ops = record_device_ops
        self._host_tier = host_tier
        self._tier_device = torch.device(device) if device is not None else None
        self._storage, self._present_mask, num_logical_blocks = _initial_store(
            initial_data, num_logical_blocks, present_mask)

        if host_tier:
            if self._tier_device is None and self._storage is not None and self._storage.is_cuda:
                self._tier_device = self._storage.device
            if self._storage is not None:
                self._storage = self._storage.cpu().pin_memory()
            if self._present_mask is not None and self._tier_device is not None:
                self._present_mask = self._present_mask.to(device=self._tier_device)

        self.num_logical_blocks = int(num_logical_blocks)
        self._save_delay_s = save_delay_s
        self._load_delay_s = load_delay_s
        self.save_calls: list[int] = []
        self.load_calls: list[int] = []
        self.operation_log: list[tuple[str, int]] = []
        self._device_scratch: torch.Tensor | None = None
        self._saving = _InFlight()
        self._loading = _InFlight()

    @property
    def max_concurrent_saves(self) -> int:
        return self._saving.peak

    @property
    def max_concurrent_loads(self) -> int:
        return self._loading.peak

    def device_store(self, actual_blocks: torch.Tensor):
        """(storage, present mask, scratch) when loads and saves against this
        store can run on the device without a host round trip: storage on
        actual_blocks' GPU (or, for a host tier, pinned rows that GPU moves)
        with its dtype and block shape, the default op set, no recording of
        device ids and no delays.  None otherwise."""
        st = self._storage
        dev = actual_blocks.device
        if (self._ops is not None or self._record_device_ops or self._save_delay_s > 0 or self._load_delay_s > 0
                or st is None or dev.type != "cuda" or st.dtype != actual_blocks.dtype
                or st.shape[1:] != actual_blocks.shape[1:] or not st.is_contiguous()):
            return None
        if self._host_tier:
            if self._gpu_for(actual_blocks) != dev:
                return None
        elif st.device != dev:
            return None
        self._mask_on(dev)
        scratch = self._device_scratch
        if scratch is None or scratch.device != dev:
            scratch = self._device_scratch = torch.zeros(st.shape[0], dtype=torch.int32, device=dev)
        return st, self._present_mask, scratch

    def note_device_ops(self, *, saved: bool, loaded: bool) -> None:
        """Bookkeeping of a save / load that ran on the device (device ids are
        not recorded, as for ``record_device_ops=False``)."""
        if saved:
            with self._saving:
                pass
        if loaded:
            with self._loading:
                pass

    def _device_ops(self):
        return self._ops if self._ops is not None else _load_cuda_extension_module()

    def save_blocks(self, logical_block_ids: torch.Tensor, block_data: torch.Tensor) -> None:
        """adapter.py:735-756."""
        _require_id_tensor(logical_block_ids, name="logical_block_ids")
        _require_block_data_tensor(block_data, expected_blocks=logical_block_ids.shape[0], name="block_data")
        with self._saving:
            if self._save_delay_s > 0:
                time.sleep(self._save_delay_s)
            if self._host_tier:
                self._save_host_tier(logical_block_ids, block_data)
                return
            if self._storage is None:
                self._storage = block_data.new_zeros((self.num_logical_blocks, *block_data.shape[1:]))
            else:
                _require_trailing_shape(block_data, self._storage, name="block_data")
                _require_same_dtype(block_data, reference=self._storage, name="block_data")
            present = self._mask_on(self._storage.device)
            ids = logical_block_ids.to(device=self._storage.device).contiguous()
            data = block_data.to(device=self._storage.device, dtype=self._storage.dtype).contiguous()
            if self._storage.device.type == "cpu" and self._ops is None:
                self._storage.index_copy_(0, ids, data)
            else:  # a repeated id keeps its last row, as index_copy_ in order does
                self._device_ops().scatter_blocks(self._storage, _last_occurrences(ids, self.num_logical_blocks),
                                                  data, skip_negative=True)
            present.index_fill_(0, ids, True)
            self._log("save", logical_block_ids)

    def load_blocks(self, logical_block_ids: torch.Tensor, actual_blocks: torch.Tensor,
                    physical_slot_ids: torch.Tensor) -> None:
        """adapter.py:758-790."""
        _require_id_tensor(logical_block_ids, name="logical_block_ids")
        _require_id_tensor(physical_slot_ids, name="physical_slot_ids")
        if logical_block_ids.shape[0] != physical_slot_ids.shape[0]:
            raise ValueError("physical_slot_ids leading dimension must match logical_block_ids")
        with self._loading:
            if self._load_delay_s > 0:
                time.sleep(self._load_delay_s)
            if self._storage is None:
                raise BlockNotFoundError("backend storage is empty")
            if self._host_tier:
                self._load_host_tier(logical_block_ids, actual_blocks, physical_slot_ids)
                return
            present = self._mask_on(self._storage.device)
            ids = logical_block_ids.to(device=self._storage.device).contiguous()
            if not bool(present.index_select(0, ids).all()):
                raise BlockNotFoundError("some logical blocks are not in backend")
            _require_trailing_shape(actual_blocks, self._storage, name="actual_blocks")
            slots = physical_slot_ids.to(device=actual_blocks.device).contiguous()
            same_device = self._storage.device == actual_blocks.device
            if same_device and self._storage.dtype == actual_blocks.dtype and (
                    self._storage.device.type != "cpu" or self._ops is not None):
                self._device_ops().copy_blocks(self._storage, ids, actual_blocks, slots)
            else:
                payloads = self._storage.index_select(0, ids).to(device=actual_blocks.device, dtype=actual_blocks.dtype)
                if actual_blocks.device.type == "cpu" and self._ops is None:
                    actual_blocks.index_copy_(0, slots, payloads)
                else:
                    self._device_ops().scatter_blocks(actual_blocks, slots, payloads.contiguous())
            self._log("load", logical_block_ids)

    def _gpu_for(self, t: torch.Tensor) -> torch.device:
        if self._tier_device is None:
            if not t.is_cuda:
                raise ValueError("a host tier moves blocks with a GPU: pass device= or CUDA tensors")
            self._tier_device = t.device
        return self._tier_device

    def _save_host_tier(self, logical_block_ids: torch.Tensor, block_data: torch.Tensor) -> None:
        """save_blocks into pinned rows: one scatter kernel writing host memory."""
        dev = self._gpu_for(block_data)
        if self._storage is None:
            self._storage = torch.zeros((self.num_logical_blocks, *block_data.shape[1:]), dtype=block_data.dtype,
                                        pin_memory=True)
        else:
            _require_trailing_shape(block_data, self._storage, name="block_data")
            _require_same_dtype(block_data, reference=self._storage, name="block_data")
        present = self._mask_on(dev)
        ids = logical_block_ids.to(device=dev).contiguous()
        data = block_data.to(device=dev, dtype=self._storage.dtype).contiguous()
        self._device_ops().scatter_blocks(self._storage, _last_occurrences(ids, self.num_logical_blocks), data,
                                          skip_negative=True)
        present.index_fill_(0, ids, True)
        self._log("save", logical_block_ids)

    def _load_host_tier(self, logical_block_ids: torch.Tensor, actual_blocks: torch.Tensor,
                        physical_slot_ids: torch.Tensor) -> None:
        """load_blocks from pinned rows: one copy kernel reading host memory."""
        dev = self._gpu_for(actual_blocks)
        present = self._mask_on(dev)
        ids = logical_block_ids.to(device=dev).contiguous()
        if not bool(present.index_select(0, ids).all()):
            raise BlockNotFoundError("some logical blocks are not in backend")
        _require_trailing_shape(actual_blocks, self._storage, name="actual_blocks")
        if actual_blocks.is_cuda and actual_blocks.dtype == self._storage.dtype:
            slots = physical_slot_ids.to(device=actual_blocks.device).contiguous()
            self._device_ops().copy_blocks(self._storage, ids, actual_blocks, slots)
        else:
            torch.cuda.synchronize(dev)
            payloads = self._storage.index_select(0, ids.cpu()).to(device=actual_blocks.device,
                                                                    dtype=actual_blocks.dtype)
            actual_blocks.index_copy_(0, physical_slot_ids.to(device=actual_blocks.device), payloads)
        self._log("load", logical_block_ids)

    def snapshot(self) -> dict[int, torch.Tensor]:
        """Each present logical id -> a host copy of its row."""
        rows = self._storage
        if rows is None:
            return {}
        if self._host_tier and self._tier_device is not None:
            torch.cuda.synchronize(self._tier_device)  # rows the GPU wrote into pinned memory
        ids = self._present_mask.nonzero().flatten().to(rows.device)
        copies = rows.index_select(0, ids).detach().cpu()
        return {i: copies[j].clone() for j, i in enumerate(ids.tolist())}

    def shutdown(self) -> None:
        return None

    def _mask_on(self, device: torch.device) -> torch.Tensor:
        """The present mask on ``device`` (all absent when there was none)."""
        mask = self._present_mask
        if mask is None:
            mask = torch.zeros((self.num_logical_blocks,), dtype=torch.bool, device=device)
        elif mask.device != device:
            mask = mask.to(device=device)
        self._present_mask = mask
        return mask

    def _log(self, operation: str, logical_block_ids: torch.Tensor) -> None:
        """The reference backend's call log (adapter.py:825-833).  Ids on a
        device are logged only with ``record_device_ops=True``: reading them
        synchronises with the device."""
        if logical_block_ids.device.type != "cpu" and not self._record_device_ops:
            return
        ids = logical_block_ids.detach().cpu().tolist()
        (self.save_calls if operation == "save" else self.load_calls).extend(ids)
        self.operation_log += [(operation, i) for i in ids]


class _InFlight:
    """Calls of one kind inside a backend right now, and the most seen at once."""

    __slots__ = ("now", "peak")

    def __init__(self) -> None:
        self.now = 0
        self.peak = 0

    def __enter__(self) -> "_InFlight":
        self.now += 1
        self.peak = max(self.peak, self.now)
        return self

    def __exit__(self, *exc) -> None:
        self.now -= 1


def _initial_store(initial, num_logical: int | None, present: torch.Tensor | None):
    """(rows, present mask, number of logical ids) of a new in-memory store.

    A tensor gives one row per logical id, all present unless ``present``
    says otherwise.  A dict gives rows for some ids (the others are absent);
    without ``num_logical`` the largest id sets the size.  No rows yet: the
    first save allocates them."""
    mask = None if present is None else present.detach().clone()
    if isinstance(initial, torch.Tensor):
        if initial.ndim < 1:
            raise ValueError("initial_data tensor must have a leading block dimension")
        rows = initial.detach().clone()
        if num_logical is not None and num_logical != rows.shape[0]:
            raise ValueError("num_logical_blocks must match initial_data.shape[0]")
        if mask is None:
            mask = torch.ones((rows.shape[0],), dtype=torch.bool, device=rows.device)
        return rows, mask.to(device=rows.device), int(rows.shape[0])
    entries = dict(initial) if initial else {}
    if num_logical is None:
        if not entries:
            raise ValueError("num_logical_blocks is required when initial_data is empty")
        num_logical = max(entries) + 1
    if not entries:
        return None, mask, int(num_logical)
    keys = list(entries)
    sample = entries[keys[0]]
    rows = sample.new_zeros((num_logical, *sample.shape))
    ids = torch.tensor(keys, dtype=ID_DTYPE, device=sample.device)
    rows.index_copy_(0, ids, torch.stack([entries[k] for k in keys]))
    mask = (torch.zeros((num_logical,), dtype=torch.bool, device=sample.device) if mask is None
            else mask.to(device=sample.device))
    return rows, mask.index_fill_(0, ids, True), int(num_logical)


@functools.lru_cache(maxsize=1)
def _load_cuda_extension_module() -> Any | None:
    """adapter.py:1347-1367: the op set lives next to this file."""
    try:
        return importlib.import_module(f"{__package__}.kv_cache_adapter_cuda")
    except ImportError:
        return None


def _take(t: torch.Tensor, index: torch.Tensor) -> torch.Tensor:
    """``t.index_select(0, index)``, also for uint16 words (16-bit slot meta),
    which torch's index_select does not take."""
    if t.dtype == torch.uint16:
        return t.to(dtype=torch.int32).index_select(0, index).to(dtype=torch.uint16)
    return t.index_select(0, index)


def _saturating_increment_usage(values: torch.Tensor) -> torch.Tensor:
    """adapter.py:1414-1416."""
    incremented = values.to(dtype=torch.int32) + 1
    return torch.clamp(incremented, max=USAGE_COUNT_MAX).to(dtype=USAGE_DTYPE)


class HostTierBackend(InMemoryBlockStoreBackend):
    """Host tier for evicted blocks: the role of the reference's LMCacheBackend
    (adapter.py:836-1062), whose CUDA path copies one block per
    cudaMemcpyAsync into a pinned memory object and back (:1035-1037,
    :960-966).  Here every block lives in one pinned host arena, row l =
    logical block l (the key's chunk_hash), and a save or load is one kernel
    that gathers or scatters all its blocks over the host link; with
    KVCacheAdapter the whole call is enqueued at once (device-store path).

    The constructor takes LMCacheBackend's arguments.  ``model_name``,
    ``world_size`` and ``worker_id`` complete the key as in
    ``CacheEngineKey`` and are kept for the caller; rows are stored in block
    shape, which for a merged K/V block is byte for byte LMCache's
    ``KV_2TD`` / ``KV_T2D`` transfer layout (``memory_format``,
    ``transfer_view``).  Capacity is the logical id space; it must fit in
    ``max_local_cpu_size_gb``.  Unlike LocalCPUBackend there is no eviction
    inside the tier.
    """

    def __init__(self, *, block_shape: tuple[int, ...] | torch.Size, block_dtype: torch.dtype,
                 num_logical_blocks: int, device: torch.device | str | None = None,
                 model_name: str = "kv_cache_adapter", world_size: int = 1, worker_id: int = 0,
                 max_local_cpu_size_gb: float | None = None, record_device_ops: bool = False) -> None:
        super().__init__(num_logical_blocks=num_logical_blocks, record_device_ops=record_device_ops,
                         host_tier=True, device=device)
        self._block_shape = torch.Size(block_shape)
        self._block_dtype = block_dtype
        self.model_name, self.world_size, self.worker_id = model_name, world_size, worker_id
        nbytes = num_logical_blocks * math.prod(self._block_shape) * torch.empty((), dtype=block_dtype).element_size()
        if max_local_cpu_size_gb is not None and nbytes > max_local_cpu_size_gb * (1 << 30):
            raise ValueError(f"{nbytes} bytes of host tier exceed max_local_cpu_size_gb={max_local_cpu_size_gb}")
        self._storage = torch.zeros((num_logical_blocks, *self._block_shape), dtype=block_dtype, pin_memory=True)
        self.layout = _MergedKVBlockLayout.detect(self._block_shape)

    @property
    def memory_format(self) -> str:
        """LMCache's MemoryFormat name of a stored row (adapter.py:1187-1192)."""
        if self.layout is None:
            return "UNDEFINED"
        return "KV_2TD" if self.layout.token_major else "KV_T2D"

    def transfer_view(self, logical_block_id: int) -> torch.Tensor:
        """Stored row of a block in LMCache's transfer shape (a view, no copy)."""
        row = self._storage[int(logical_block_id)]
        return row if self.layout is None else row.reshape(self.layout.transfer_shape)

    def _require_block_layout(self, t: torch.Tensor, *, name: str) -> None:
        """adapter.py:1126-1130."""
        if t.dtype != self._block_dtype:
            raise TypeError(f"{name} must have dtype {self._block_dtype}")
        if tuple(t.shape[1:]) != tuple(self._block_shape):
            raise ValueError(f"{name} must have trailing shape {tuple(self._block_shape)}")

    def save_blocks(self, logical_block_ids: torch.Tensor, block_data: torch.Tensor) -> None:
        """adapter.py:888-907."""
        _require_id_tensor(logical_block_ids, name="logical_block_ids")
        _require_block_data_tensor(block_data, expected_blocks=logical_block_ids.shape[0], name="block_data")
        self._require_block_layout(block_data, name="block_data")
        if logical_block_ids.numel() == 0:
            return
        super().save_blocks(logical_block_ids, block_data)

    def load_blocks(self, logical_block_ids: torch.Tensor, actual_blocks: torch.Tensor,
                    physical_slot_ids: torch.Tensor) -> None:
        """adapter.py:909-969; a missing block raises BlockNotFoundError."""
        _require_id_tensor(logical_block_ids, name="logical_block_ids")
        _require_id_tensor(physical_slot_ids, name="physical_slot_ids")
        if logical_block_ids.shape[0] != physical_slot_ids.shape[0]:
            raise ValueError("physical_slot_ids leading dimension must match logical_block_ids")
        self._require_block_layout(actual_blocks, name="actual_blocks")
        if logical_block_ids.numel() == 0:
            return
        super().load_blocks(logical_block_ids, actual_blocks, physical_slot_ids)

    def shutdown(self) -> None:
        """adapter.py:971-976: drop every stored block."""
        if self._tier_device is not None:
            torch.cuda.synchronize(self._tier_device)
        self._storage = None
        self._present_mask = None
        self._device_scratch = None


def _last_occurrences(ids: torch.Tensor, size: int) -> torch.Tensor:
    """``ids`` with every occurrence but the last of a repeated id set to -1,
    so that an unordered scatter skipping negatives leaves what index_copy_
    applied in order leaves.  Ids outside [0, size) become ``size``, which the
    row mover rejects, instead of reaching a torch index op."""
    positions = torch.arange(ids.numel(), dtype=ID_DTYPE, device=ids.device)
    valid = (ids >= 0) & (ids < size)
    safe = torch.where(valid, ids, 0)
    last = torch.full((size,), -1, dtype=ID_DTYPE, device=ids.device)
    last.scatter_reduce_(0, safe, torch.where(valid, positions, -1), reduce="amax")
    keep = last.index_select(0, safe) == positions
    return torch.where(valid, torch.where(keep, ids, -1), size).contiguous()


def _slot_meta_pin_counts(slot_meta: torch.Tensor, *, dtype: torch.dtype = PIN_COUNT_DTYPE) -> torch.Tensor:
    """adapter.py:1419-1420."""
    return (slot_meta.to(dtype=torch.int32) & _PIN_COUNT_MASK).to(dtype=dtype)


def _slot_meta_usage_counts(slot_meta: torch.Tensor) -> torch.Tensor:
    """adapter.py:1423-1424."""
    return ((slot_meta.to(dtype=torch.int32) >> _USAGE_COUNT_SHIFT) & _USAGE_COUNT_MASK).to(dtype=USAGE_DTYPE)


def _pack_slot_meta(pin_counts: torch.Tensor, usage_counts: torch.Tensor) -> torch.Tensor:
    """adapter.py:1427-1432."""
    packed = (pin_counts.to(dtype=torch.int32) & _PIN_COUNT_MASK) | (
        (usage_counts.to(dtype=torch.int32) & _USAGE_COUNT_MASK) << _USAGE_COUNT_SHIFT)
    return packed.to(dtype=SLOT_META_DTYPE)


def _positions(mask: torch.Tensor, where: bool = True) -> torch.Tensor:
    """Indices, in order, of the entries of ``mask`` that are true (or, with
    ``where=False``, false): the split of a request into hits and misses."""
    picked = mask.bool() if where else mask.logical_not()
    return picked.nonzero().flatten()


def _require_id_tensor(values: torch.Tensor, *, name: str) -> None:
    if not isinstance(values, torch.Tensor):
        raise TypeError(f"{name} must be torch.Tensor")
    if values.dtype != ID_DTYPE:
        raise TypeError(f"{name} must have dtype torch.int64")
    if values.ndim != 1:
        raise ValueError(f"{name} must have shape (k,)")


def _require_same_device(values: torch.Tensor, *, expected_device: torch.device, name: str) -> None:
    if values.device != expected_device:
        raise ValueError(f"{name} must be on device {expected_device}, got {values.device}")


def _require_same_dtype(block_data: torch.Tensor, *, reference: torch.Tensor, name: str) -> None:
    if block_data.dtype != reference.dtype:
        raise TypeError(f"{name} must have dtype {reference.dtype}")


def _require_block_data_tensor(block_data: torch.Tensor, *, expected_blocks: int, name: str) -> None:
    if not isinstance(block_data, torch.Tensor):
        raise TypeError(f"{name} must be torch.Tensor")
    if block_data.ndim < 1:
        raise ValueError(f"{name} must have a leading block dimension")
    if block_data.shape[0] != expected_blocks:
        raise ValueError(f"{name} leading dimension must match logical_block_ids length")


def _require_trailing_shape(block_data: torch.Tensor, reference: torch.Tensor, *, name: str) -> None:
    if block_data.ndim != reference.ndim or block_data.shape[1:] != reference.shape[1:]:
        raise ValueError(f"{name} must have trailing shape {tuple(reference.shape[1:])}")
