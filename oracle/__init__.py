"""CPU oracle for the adapter hot path -- TEST INFRASTRUCTURE ONLY.

Only the test suite, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this package, and only as the checker (or the timed
CPU baseline).  The product (``kv_cache_adapter_b200``) never imports it.

* ``kvca_oracle.c`` restates the reference's strict slot-metadata path and
  clock sweep in plain C (wrapped here with ctypes).
* ``moves.py`` restates the reference's block and token moves with the same
  torch CPU ops the reference calls (``index_select`` / ``index_copy_``).

Pinning: the reference's known-answer tests (test_adapter_npu_kernels.py:42-194)
and fixtures produced by running the reference itself
(``tests/golden/make_golden.py``) are replayed against this oracle by
``tests/test_oracle_golden.py``.
"""
from __future__ import annotations

import ctypes
import pathlib
import subprocess

import torch

_HERE = pathlib.Path(__file__).resolve().parent
_SRC = _HERE / "kvca_oracle.c"
_LIB = _HERE / "libkvca_oracle.so"

OK, INSUFFICIENT, BAD_INDEX, BAD_ARGUMENT = 0, 1, 2, 3


class OracleInsufficientCapacity(RuntimeError):
    """Too few reusable slots (the reference raises InsufficientCapacityError)."""


class OracleBadIndex(IndexError):
    """An id or slot outside its table (the reference raises IndexError)."""


def build(force: bool = False) -> pathlib.Path:
    """Compile the C restatement with gcc into oracle/libkvca_oracle.so."""
    if force or not _LIB.exists() or _LIB.stat().st_mtime < _SRC.stat().st_mtime:
        subprocess.run(
            ["gcc", "-O2", "-std=c11", "-shared", "-fPIC", str(_SRC), "-o", str(_LIB)],
            check=True,
        )
    return _LIB


_lib: ctypes.CDLL | None = None


def _load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(str(build()))
        for name in (
            "oracle_inspect_load",
            "oracle_inspect_save",
            "oracle_pop",
            "oracle_commit_load",
            "oracle_commit_save",
            "oracle_release",
            "oracle_clock_stream",
            "oracle_clock_stream_traced",
        ):
            getattr(_lib, name).restype = ctypes.c_int
    return _lib


def _p(t: torch.Tensor | None) -> ctypes.c_void_p:
    if t is None or t.numel() == 0:
        return ctypes.c_void_p(0)
    assert t.device.type == "cpu" and t.is_contiguous()
    return ctypes.c_void_p(t.data_ptr())


def _i(x: int) -> ctypes.c_int64:
    return ctypes.c_int64(int(x))


def meta_bits_of(slot_meta: torch.Tensor) -> int:
    if slot_meta.dtype == torch.uint8:
        return 8
    if slot_meta.dtype == torch.uint16:
        return 16
    raise TypeError(f"slot_meta must be uint8 or uint16, got {slot_meta.dtype}")


def _raise(rc: int) -> None:
    if rc == OK:
        return
    if rc == INSUFFICIENT:
        raise OracleInsufficientCapacity("No reusable actual block is available")
    if rc == BAD_INDEX:
        raise OracleBadIndex("index out of range")
    raise ValueError(f"oracle rejected its arguments (code {rc})")


def _cpu(t: torch.Tensor) -> torch.Tensor:
    return t.detach().to("cpu").contiguous()


def inspect_load_requests(l2p, slot_meta, ids):
    l2p, slot_meta, ids = _cpu(l2p), _cpu(slot_meta), _cpu(ids)
    k = ids.numel()
    cur = torch.empty(k, dtype=torch.int64)
    resident = torch.empty(k, dtype=torch.uint8)
    pins = torch.empty(k, dtype=torch.int64)
    usage = torch.empty(k, dtype=slot_meta.dtype)
    _raise(_load().oracle_inspect_load(
        meta_bits_of(slot_meta), _p(l2p), _i(l2p.numel()), _p(slot_meta), _i(slot_meta.numel()),
        _p(ids), _i(k), _p(cur), _p(resident), _p(pins), _p(usage)))
    return cur, resident.bool(), pins, usage


def inspect_save_requests(l2p, slot_meta, ids):
    l2p, slot_meta, ids = _cpu(l2p), _cpu(slot_meta), _cpu(ids)
    k = ids.numel()
    cur = torch.empty(k, dtype=torch.int64)
    existing = torch.empty(k, dtype=torch.uint8)
    usage = torch.empty(k, dtype=slot_meta.dtype)
    _raise(_load().oracle_inspect_save(
        meta_bits_of(slot_meta), _p(l2p), _i(l2p.numel()), _p(slot_meta), _i(slot_meta.numel()),
        _p(ids), _i(k), _p(cur), _p(existing), _p(usage)))
    return cur, existing.bool(), usage


def pop_reusable_slots(slot_meta, search_start, blocked_slot_ids, count, *, order: str = "grouped"):
    """In place on CPU tensors ``slot_meta`` and ``search_start``."""
    assert slot_meta.device.type == "cpu" and slot_meta.is_contiguous()
    assert search_start.device.type == "cpu" and search_start.is_contiguous()
    blocked = _cpu(blocked_slot_ids)
    out = torch.empty(int(count), dtype=torch.int64)
    _raise(_load().oracle_pop(
        meta_bits_of(slot_meta), 0 if order == "grouped" else 1, _p(slot_meta),
        _i(slot_meta.numel()), _p(search_start), _p(blocked), _i(blocked.numel()), _i(count),
        _p(out)))
    return out


def commit_load_metadata(l2p, p2l, slot_meta, evicted, miss_ids, miss_slots, hit_slots,
                         hit_pins, hit_usage, miss_usage):
    for t in (l2p, p2l, slot_meta):
        assert t.device.type == "cpu" and t.is_contiguous()
    evicted, miss_ids, miss_slots = _cpu(evicted), _cpu(miss_ids), _cpu(miss_slots)
    hit_slots, hit_pins = _cpu(hit_slots), _cpu(hit_pins).to(torch.int64)
    hit_usage = _cpu(hit_usage).to(slot_meta.dtype)
    miss_usage = _cpu(miss_usage).to(slot_meta.dtype)
    _raise(_load().oracle_commit_load(
        meta_bits_of(slot_meta), _p(l2p), _i(l2p.numel()), _p(p2l), _p(slot_meta),
        _i(slot_meta.numel()), _p(evicted), _i(evicted.numel()), _p(miss_ids), _p(miss_slots),
        _i(miss_ids.numel()), _p(hit_slots), _p(hit_pins), _p(hit_usage), _i(hit_slots.numel()),
        _p(miss_usage)))


def commit_save_metadata(l2p, p2l, slot_meta, evicted, ids, slots, final_pins, final_usage):
    for t in (l2p, p2l, slot_meta):
        assert t.device.type == "cpu" and t.is_contiguous()
    evicted, ids, slots = _cpu(evicted), _cpu(ids), _cpu(slots)
    final_pins = _cpu(final_pins).to(slot_meta.dtype)
    final_usage = _cpu(final_usage).to(slot_meta.dtype)
    _raise(_load().oracle_commit_save(
        meta_bits_of(slot_meta), _p(l2p), _i(l2p.numel()), _p(p2l), _p(slot_meta),
        _i(slot_meta.numel()), _p(evicted), _i(evicted.numel()), _p(ids), _p(slots),
        _p(final_pins), _p(final_usage), _i(ids.numel())))


def release_metadata(l2p, slot_meta, ids):
    assert slot_meta.device.type == "cpu" and slot_meta.is_contiguous()
    l2p, ids = _cpu(l2p), _cpu(ids)
    _raise(_load().oracle_release(
        meta_bits_of(slot_meta), _p(l2p), _i(l2p.numel()), _p(slot_meta), _i(slot_meta.numel()),
        _p(ids), _i(ids.numel())))


def clock_stream(slot_meta, search_start, num_steps, alloc_per_step, reaccess,
                 reaccess_per_step, *, order: str = "grouped", trace: bool = False):
    """Returns (victims[num_steps * alloc_per_step], steps_done, status code),
    plus with ``trace`` each step's usage class T (int8, -1 past steps_done)."""
    assert slot_meta.device.type == "cpu" and slot_meta.is_contiguous()
    assert search_start.device.type == "cpu" and search_start.is_contiguous()
    reaccess = _cpu(reaccess)
    victims = torch.full((int(num_steps) * int(alloc_per_step),), -1, dtype=torch.int64)
    thresholds = torch.full((int(num_steps),), -1, dtype=torch.int8)
    done = ctypes.c_int64(0)
    rc = _load().oracle_clock_stream_traced(
        meta_bits_of(slot_meta), 0 if order == "grouped" else 1, _p(slot_meta),
        _i(slot_meta.numel()), _p(search_start), _i(num_steps), _i(alloc_per_step),
        _p(reaccess), _i(reaccess_per_step), _p(victims), ctypes.byref(done),
        _p(thresholds) if trace else ctypes.c_void_p(0))
    if trace:
        return victims, int(done.value), rc, thresholds
    return victims, int(done.value), rc
