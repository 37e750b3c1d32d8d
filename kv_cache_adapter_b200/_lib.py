"""ctypes binding of the C ABI in include/kvca.h (libkvca_b200.so).

The shared library is built in-tree by ``kv_cache_adapter_b200.build`` with
nvcc for sm_100a.  Loading fails loudly when it is missing: there is no
fallback implementation.
"""
from __future__ import annotations

import ctypes
import functools
import pathlib

LIB_NAME = "libkvca_b200.so"

KVCA_OK = 0
KVCA_ERR_INSUFFICIENT_CAPACITY = 1
KVCA_ERR_BAD_INDEX = 2
KVCA_ERR_BAD_ARGUMENT = 3
KVCA_ERR_CUDA = 4
KVCA_ERR_SIZE_LIMIT = 5
KVCA_ERR_DEVICE_TIMEOUT = 6
KVCA_ERR_BLOCK_NOT_FOUND = 7
KVCA_NOALLOC_MAX_SLOTS = 1048576

KVCA_POP_ORDER_GROUPED = 0
KVCA_POP_ORDER_PREFIX = 1

KVCA_FLAG_SKIP_NEGATIVE = 1
KVCA_FLAG_HOST_MEMORY = 2
KVCA_FLAG_INPUTS_READY = 4
KVCA_MAX_PLANES = 256

c_i64 = ctypes.c_int64
c_int = ctypes.c_int
c_ptr = ctypes.c_void_p


class PagedDesc(ctypes.Structure):
    """kvca_paged_desc."""

    _fields_ = [
        ("plane_ptrs", ctypes.POINTER(ctypes.c_uint64)),
        ("num_blocks", c_i64),
        ("block_size", c_i64),
        ("block_stride", c_i64),
        ("row_stride", c_i64),
        ("index", c_ptr),
    ]


class ChunkDesc(ctypes.Structure):
    """kvca_chunk_desc."""

    _fields_ = [
        ("base", ctypes.c_uint64),
        ("rows_per_chunk", c_i64),
        ("chunk_stride", c_i64),
        ("row_stride", c_i64),
        ("plane_stride", c_i64),
    ]


class DeviceStore(ctypes.Structure):
    """kvca_device_store."""

    _fields_ = [
        ("storage", ctypes.c_uint64),
        ("storage_row_stride", c_i64),
        ("present", c_ptr),
        ("scratch", c_ptr),
        ("move_flags", ctypes.c_int32),
    ]


class AdapterSession(ctypes.Structure):
    """kvca_adapter_session."""

    _fields_ = [
        ("meta_bits", ctypes.c_int32),
        ("order", ctypes.c_int32),
        ("l2p", c_ptr),
        ("num_logical", c_i64),
        ("p2l", c_ptr),
        ("slot_meta", c_ptr),
        ("num_slots", c_i64),
        ("search_start", c_ptr),
        ("scratch_bitmap", c_ptr),
        ("store", DeviceStore),
        ("actual", ctypes.c_uint64),
        ("actual_row_stride", c_i64),
        ("row_bytes", c_i64),
        ("work", c_ptr),
        ("work_meta", c_ptr),
        ("work_ids", c_i64),
        ("counts", c_ptr),
        ("counts_host", c_ptr),
        ("status", c_ptr),
        ("stream", c_ptr),
        ("sequence", c_i64),
    ]


# name -> (restype, argtypes); one entry per declaration in include/kvca.h
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "kvca_abi_version": (c_int, []),
    "kvca_device_sm_count": (c_int, []),
    "kvca_inspect_load_requests": (
        c_int,
        [c_int, c_ptr, c_i64, c_ptr, c_i64, c_ptr, c_i64, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr],
    ),
    "kvca_inspect_save_requests": (
        c_int,
        [c_int, c_ptr, c_i64, c_ptr, c_i64, c_ptr, c_i64, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr],
    ),
    "kvca_pop_scratch_bytes": (ctypes.c_size_t, [c_i64]),
    "kvca_pop_reusable_slots": (
        c_int,
        [c_int, c_int, c_ptr, c_i64, c_ptr, c_ptr, c_i64, c_i64, c_ptr, c_ptr, c_ptr, c_ptr],
    ),
    "kvca_pop_reusable_slots_noalloc": (
        c_int, [c_int, c_int, c_ptr, c_i64, c_ptr, c_ptr, c_i64, c_i64, c_ptr, c_ptr, c_ptr],
    ),
    "kvca_choose_pop_launch_warps": (c_i64, [c_i64]),
    "kvca_commit_load_metadata": (
        c_int,
        [c_int, c_ptr, c_i64, c_ptr, c_ptr, c_i64, c_ptr, c_i64, c_ptr, c_ptr, c_i64, c_ptr, c_ptr,
         c_ptr, c_i64, c_ptr, c_ptr, c_ptr],
    ),
    "kvca_commit_save_metadata": (
        c_int,
        [c_int, c_ptr, c_i64, c_ptr, c_ptr, c_i64, c_ptr, c_i64, c_ptr, c_ptr, c_ptr, c_ptr, c_i64,
         c_ptr, c_ptr],
    ),
    "kvca_release_metadata": (
        c_int, [c_int, c_ptr, c_i64, c_ptr, c_i64, c_ptr, c_i64, c_ptr, c_ptr],
    ),
    "kvca_clock_stream": (
        c_int,
        [c_int, c_int, c_ptr, c_i64, c_ptr, c_i64, c_i64, c_ptr, c_i64, c_ptr, c_ptr, c_ptr, c_ptr],
    ),
    "kvca_clock_stream_scratch_bytes": (ctypes.c_size_t, [c_i64]),
    "kvca_clock_stream_batched": (
        c_int,
        [c_int, c_int, c_ptr, c_i64, c_ptr, c_i64, c_i64, c_ptr, c_i64, c_ptr, c_ptr, c_ptr, c_int, c_ptr,
         c_ptr],
    ),
    "kvca_plan_load": (
        c_int,
        [c_int, c_int, c_ptr, c_i64, c_ptr, c_ptr, c_i64, c_ptr, c_ptr, c_i64, c_ptr, c_ptr, c_ptr, c_ptr,
         c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr],
    ),
    "kvca_plan_save": (
        c_int,
        [c_int, c_int, c_ptr, c_i64, c_ptr, c_ptr, c_i64, c_ptr, c_ptr, c_i64, c_ptr, c_ptr, c_ptr, c_ptr,
         c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr],
    ),
    "kvca_load_device_store": (
        c_int,
        [c_int, c_int, c_ptr, c_i64, c_ptr, c_ptr, c_i64, c_ptr, c_ptr, c_i64, c_ptr,
         ctypes.POINTER(DeviceStore), ctypes.c_uint64, c_i64, c_i64, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr],
    ),
    "kvca_save_device_store": (
        c_int,
        [c_int, c_int, c_ptr, c_i64, c_ptr, c_ptr, c_i64, c_ptr, c_ptr, c_i64, c_ptr,
         ctypes.POINTER(DeviceStore), ctypes.c_uint64, c_i64, c_i64, ctypes.c_uint64, c_ptr, c_ptr, c_ptr, c_ptr,
         c_ptr],
    ),
    "kvca_session_load": (c_int, [ctypes.POINTER(AdapterSession), c_ptr, c_i64, c_ptr]),
    "kvca_session_save": (c_int, [ctypes.POINTER(AdapterSession), c_ptr, c_i64, ctypes.c_uint64]),
    "kvca_host_memory_usable": (c_int, [c_ptr, c_i64]),
    "kvca_wait_selftest": (c_int, [c_ptr, ctypes.c_uint32, c_ptr, c_ptr]),
    "kvca_append_step": (
        c_int,
        [c_int, c_int, c_ptr, c_i64, c_ptr, c_ptr, c_i64, c_ptr, c_ptr, c_i64, c_ptr, c_ptr, c_ptr, c_i64, c_i64,
         c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr],
    ),
    "kvca_append_steps": (
        c_int,
        [c_int, c_int, c_ptr, c_i64, c_ptr, c_ptr, c_i64, c_ptr, c_ptr, c_ptr, c_i64, c_i64, c_ptr, c_ptr, c_ptr,
         c_i64, c_i64, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr],
    ),
    "kvca_exchange": (
        c_int,
        [ctypes.POINTER(PagedDesc), ctypes.POINTER(PagedDesc), c_ptr, c_i64, c_i64, ctypes.c_int32, c_ptr, c_ptr],
    ),
    "kvca_gather": (
        c_int,
        [ctypes.POINTER(PagedDesc), ctypes.POINTER(ChunkDesc), c_i64, c_i64, c_i64, ctypes.c_int32,
         c_ptr, c_ptr],
    ),
    "kvca_scatter": (
        c_int,
        [ctypes.POINTER(ChunkDesc), ctypes.POINTER(PagedDesc), c_i64, c_i64, c_i64, ctypes.c_int32,
         c_ptr, c_ptr],
    ),
    "kvca_row_ceiling": (c_int, [c_ptr, c_ptr, c_ptr, c_i64, c_i64, c_int, c_int, c_ptr]),
    "kvca_move_cycle_scratch_bytes": (c_i64, [c_i64]),
    "kvca_move_cycle": (
        c_int,
        [ctypes.POINTER(ChunkDesc), ctypes.POINTER(PagedDesc), c_i64, ctypes.POINTER(PagedDesc), c_i64,
         ctypes.POINTER(ChunkDesc), c_i64, c_i64, c_ptr, c_i64, c_i64, c_i64, ctypes.c_int32, c_ptr, c_ptr, c_ptr],
    ),
    "kvca_scatter_gather": (
        c_int,
        [ctypes.POINTER(ChunkDesc), ctypes.POINTER(PagedDesc), c_i64, c_i64, c_i64, ctypes.POINTER(PagedDesc),
         ctypes.POINTER(ChunkDesc), c_i64, c_i64, c_i64, ctypes.c_int32, ctypes.c_int32, c_ptr, c_ptr],
    ),
    "kvca_copy_paged": (
        c_int,
        [ctypes.POINTER(PagedDesc), ctypes.POINTER(PagedDesc), c_i64, c_i64, c_i64, ctypes.c_int32,
         c_ptr, c_ptr],
    ),
}


def lib_path() -> pathlib.Path:
    return pathlib.Path(__file__).resolve().with_name(LIB_NAME)


@functools.lru_cache(maxsize=1)
def load() -> ctypes.CDLL:
    path = lib_path()
    if not path.exists():
        raise ImportError(
            f"{path} is missing: build it with `python -m kv_cache_adapter_b200.build` "
            "(nvcc, sm_100a); there is no fallback implementation"
        )
    lib = ctypes.CDLL(str(path))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return lib
