"""CPU: the C ABI library loads, exports every entry point declared in
include/kvca.h, and rejects bad host-side arguments before touching a device."""
from __future__ import annotations

import ctypes
import re

from conftest import REPO
from kv_cache_adapter_b200 import _lib

HEADER = REPO / "include" / "kvca.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(kvca_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_expected_entry_points():
    names = declared_functions()
    assert names == sorted(_lib.SIGNATURES), "ctypes signatures and include/kvca.h disagree"
    for name in ("kvca_pop_reusable_slots", "kvca_inspect_load_requests", "kvca_inspect_save_requests",
                 "kvca_commit_load_metadata", "kvca_commit_save_metadata", "kvca_release_metadata",
                 "kvca_gather", "kvca_scatter", "kvca_copy_paged", "kvca_clock_stream"):
        assert name in names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_abi_version_and_scratch_sizes():
    lib = _lib.load()
    assert lib.kvca_abi_version() == 1
    assert lib.kvca_pop_scratch_bytes(0) == 0
    assert lib.kvca_pop_scratch_bytes(1) == 4
    assert lib.kvca_pop_scratch_bytes(32) == 4
    assert lib.kvca_pop_scratch_bytes(33) == 8
    # tables of 65,536 to 2^24 slots add the whole-GPU pop's area after the bitmap
    assert lib.kvca_pop_scratch_bytes(65535) == 65536 // 8
    assert lib.kvca_pop_scratch_bytes(1 << 20) == (1 << 20) // 8 + 256 + 160 * 256 * 4
    assert lib.kvca_pop_scratch_bytes((1 << 24) + 1) == ((1 << 24) + 32) // 8
    assert lib.kvca_choose_pop_launch_warps(1) == 1
    assert lib.kvca_choose_pop_launch_warps(1 << 20) == 32


def test_host_side_argument_checks_need_no_device():
    lib = _lib.load()
    null = ctypes.c_void_p(0)
    bad = _lib.KVCA_ERR_BAD_ARGUMENT
    # unsupported slot-meta width
    assert lib.kvca_release_metadata(7, null, 1, null, 1, null, 1, null, null) == bad
    # unknown pop order, empty table, negative count
    assert lib.kvca_pop_reusable_slots(8, 9, null, 4, null, null, 0, 1, null, null, null, null) == bad
    assert lib.kvca_pop_reusable_slots(8, 0, null, 0, null, null, 0, 1, null, null, null, null) == bad
    assert lib.kvca_pop_reusable_slots(8, 0, null, 4, null, null, 0, -1, null, null, null, null) == bad
    # count 0 is a no-op that succeeds without any pointer
    assert lib.kvca_pop_reusable_slots(8, 0, null, 4, null, null, 0, 0, null, null, null, null) == 0
    assert lib.kvca_inspect_load_requests(8, null, 1, null, 1, null, 0, null, null, null, null, null, null) == 0
    # missing pointers with work to do
    assert lib.kvca_inspect_save_requests(8, null, 1, null, 1, null, 3, null, null, null, null, null) == bad
    # too many re-accesses per step for the stream kernel
    assert lib.kvca_clock_stream(8, 0, null, 4, null, 1, 1, null, 9000, null, null, null, null) == bad
    # row movers: plane count and row size limits, missing descriptors
    src = _lib.PagedDesc()
    dst = _lib.ChunkDesc()
    assert lib.kvca_gather(ctypes.byref(src), ctypes.byref(dst), 0, 4, 16, 0, null, null) == bad
    assert lib.kvca_gather(ctypes.byref(src), ctypes.byref(dst), _lib.KVCA_MAX_PLANES + 1, 4, 16, 0, null, null) == bad
    assert lib.kvca_gather(ctypes.byref(src), ctypes.byref(dst), 1, 4, 0, 0, null, null) == bad
    assert lib.kvca_gather(ctypes.byref(src), ctypes.byref(dst), 1, 4, 16, 0, null, null) == bad  # null planes
    assert lib.kvca_gather(ctypes.byref(src), ctypes.byref(dst), 1, 0, 16, 0, null, null) == 0  # nothing to move


def test_decode_loop_entry_points_check_arguments_on_the_host():
    lib = _lib.load()
    null = ctypes.c_void_p(0)
    bad = _lib.KVCA_ERR_BAD_ARGUMENT
    # append_steps: no table, negative step count, missing offsets with steps to run
    assert lib.kvca_append_steps(8, 0, null, 0, null, null, 4, null, null, null, 0, 1, null, null, null, 2, 16,
                                 null, null, null, null, null) == bad
    one = ctypes.c_void_p(16)  # never dereferenced: the call is refused first
    assert lib.kvca_append_steps(8, 0, one, 8, one, one, 4, one, null, null, 0, -1, one, one, one, 2, 16,
                                 one, null, one, one, null) == bad
    assert lib.kvca_append_steps(8, 0, one, 8, one, one, 4, one, null, null, 0, 3, one, one, one, 2, 16,
                                 one, null, one, one, null) == bad
    # zero steps is a no-op
    assert lib.kvca_append_steps(8, 0, one, 8, one, one, 4, one, null, null, 0, 0, one, one, one, 2, 16,
                                 one, null, null, one, null) == 0
    # scatter_gather: plane and row limits on either side, missing descriptors
    c, pdesc = _lib.ChunkDesc(), _lib.PagedDesc()
    args = (ctypes.byref(c), ctypes.byref(pdesc))
    assert lib.kvca_scatter_gather(*args, 0, 4, 16, ctypes.byref(pdesc), ctypes.byref(c), 1, 4, 16, 0, 0, null,
                                   null) == bad
    assert lib.kvca_scatter_gather(*args, 1, 4, 16, ctypes.byref(pdesc), ctypes.byref(c), 1, 4, 0, 0, 0, null,
                                   null) == bad
    assert lib.kvca_scatter_gather(*args, 1, 4, 16, ctypes.byref(pdesc), ctypes.byref(c), 1, 4, 16, 0, 0, null,
                                   null) == bad  # null plane tables
    assert lib.kvca_scatter_gather(*args, 1, 0, 16, ctypes.byref(pdesc), ctypes.byref(c), 1, 0, 16, 0, 0, null,
                                   null) == 0  # nothing to move


def test_move_cycle_checks_arguments_on_the_host():
    lib = _lib.load()
    assert lib.kvca_move_cycle_scratch_bytes(0) == 512
    assert lib.kvca_move_cycle_scratch_bytes(65536) == 512 + 16 * 65536
    assert lib.kvca_move_cycle_scratch_bytes(-1) == -1
    bad = _lib.KVCA_ERR_BAD_ARGUMENT
    one = ctypes.c_void_p(4096)  # never dereferenced: every call below is refused first
    planes = (ctypes.c_uint64 * 2)(1 << 20, 1 << 21)
    others = (ctypes.c_uint64 * 2)(1 << 20, 1 << 22)
    ptr = ctypes.cast(planes, ctypes.POINTER(ctypes.c_uint64))

    def paged(table=ptr, block_size=16, row_stride=256, index=one):
        return _lib.PagedDesc(table, 64, block_size, 4096, row_stride, index)

    tokens = _lib.ChunkDesc(1 << 23, 8, 0, 256, 8 * 256)
    spill = _lib.ChunkDesc(1 << 24, 1, 2 * 4096, 4096, 4096)

    def call(tok=None, blk=None, row=256, block_row=4096, steps=4, seqs=8, offsets=one, scratch=one):
        return lib.kvca_move_cycle(ctypes.byref(tokens), ctypes.byref(tok or paged()), row,
                                   ctypes.byref(blk or paged(block_size=1, row_stride=4096)), 16,
                                   ctypes.byref(spill), block_row, 2, offsets, steps, seqs, 16, 1, scratch, one,
                                   None)

    assert call(steps=0) == bad
    assert call(steps=33) == bad
    assert call(offsets=None) == bad
    assert call(scratch=None) == bad
    assert call(row=264) == bad  # rows of 16-byte vectors only
    assert call(blk=paged(block_size=16, row_stride=4096)) == bad  # block side must be block-granular
    assert call(blk=paged(table=ctypes.cast(others, ctypes.POINTER(ctypes.c_uint64)), block_size=1,
                          row_stride=4096)) == bad  # another cache
    assert call(tok=paged(index=None)) == bad  # no slot mapping
    assert call(block_row=8192) == bad  # a block row past its block
    assert call(tok=paged(row_stride=512)) == bad  # token rows past their block
    assert call(seqs=1 << 27) == _lib.KVCA_ERR_SIZE_LIMIT


def test_row_ceiling_checks_arguments_on_the_host():
    lib = _lib.load()
    bad = _lib.KVCA_ERR_BAD_ARGUMENT
    p = ctypes.c_void_p(1 << 20)  # never dereferenced: every call below is refused first
    assert lib.kvca_row_ceiling(p, p, p, 100, 100, 1, 4, None) == bad  # unsupported width
    assert lib.kvca_row_ceiling(p, p, p, 0, 128, 1, 4, None) == bad
    assert lib.kvca_row_ceiling(p, p, p, 1 << 31, 128, 1, 4, None) == bad
    assert lib.kvca_row_ceiling(p, p, p, 100, 128, 1, 0, None) == bad
    assert lib.kvca_row_ceiling(ctypes.c_void_p(8), p, p, 100, 128, 1, 4, None) == bad  # misaligned
    assert lib.kvca_row_ceiling(None, p, p, 100, 128, 1, 4, None) == bad
