"""GPU: the clock sweep entry point that allocates nothing.

kvca_pop_reusable_slots_noalloc serves callers that may not call cudaMalloc
(a serving loop whose device memory is reserved up front, a host runtime
without a device allocator, an embedding with a fixed memory budget): its
blocked-slot bitmap is a device array inside the library instead of caller
scratch.  Called here through the C ABI, it must give exactly what
kvca_pop_reusable_slots gives (victims, aged slot_meta, search_start) on two
calls in a row, the second with different blocked slots, so that anything the
first call left in the shared array would show.  Its error paths (a blocked id
out of range, too few reusable slots, no status words) must report and change
nothing, and the next call must still be exact, against the allocating pop
and against the oracle.  This file is collected last.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import oracle
from kv_cache_adapter_b200 import _lib

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _p(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr() if t.numel() else 0)


def _table(rng, n: int, bits: int) -> torch.Tensor:
    f = bits // 2
    usage = np.where(rng.random(n) < 0.002, 0, rng.integers(1, 4, n))  # few zeros: full scans and aging
    pins = (rng.random(n) < 0.05).astype(np.int64)
    words = pins | (usage << f)
    return torch.from_numpy(words.astype(np.uint8 if bits == 8 else np.uint16)).to(DEV)


@pytest.mark.parametrize("bits,n,order", [(8, 100_003, 0), (16, 5_000, 0), (8, 1 << 20, 1), (8, 1 << 20, 0)])
def test_noalloc_pop_matches_allocating_pop_twice(bits, n, order):
    lib = _lib.load()
    rng = np.random.default_rng(n + bits + order)
    meta_a = _table(rng, n, bits)
    meta_b = meta_a.clone()
    ss_a = torch.tensor([int(rng.integers(0, n))], dtype=torch.int64, device=DEV)
    ss_b = ss_a.clone()
    bitmap = torch.zeros(int(lib.kvca_pop_scratch_bytes(n)) // 4, dtype=torch.int32, device=DEV)
    st_a = torch.zeros(2, dtype=torch.int64, device=DEV)
    st_b = torch.zeros(2, dtype=torch.int64, device=DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)
    for call, count in enumerate((3000, 257)):
        blocked = torch.from_numpy(rng.integers(0, n, 200 + 50 * call).astype(np.int64)).to(DEV)
        out_a = torch.full((count,), -1, dtype=torch.int64, device=DEV)
        out_b = torch.full((count,), -2, dtype=torch.int64, device=DEV)
        rc_a = lib.kvca_pop_reusable_slots(bits, order, _p(meta_a), n, _p(ss_a), _p(blocked), blocked.numel(),
                                           count, _p(out_a), _p(bitmap), _p(st_a), stream)
        rc_b = lib.kvca_pop_reusable_slots_noalloc(bits, order, _p(meta_b), n, _p(ss_b), _p(blocked),
                                                   blocked.numel(), count, _p(out_b), _p(st_b), stream)
        torch.cuda.synchronize(DEV)
        assert rc_a == 0 and rc_b == 0
        assert st_a.tolist() == [0, 0] and st_b.tolist() == [0, 0]
        assert torch.equal(out_a, out_b), call
        assert torch.equal(meta_a.view(torch.uint8), meta_b.view(torch.uint8)), call
        assert torch.equal(ss_a, ss_b), call


def test_noalloc_pop_rejects_tables_above_its_capacity():
    lib = _lib.load()
    null = ctypes.c_void_p(0)
    rc = lib.kvca_pop_reusable_slots_noalloc(8, 0, null, _lib.KVCA_NOALLOC_MAX_SLOTS + 1, null, null, 0, 1,
                                             null, null, null)
    assert rc == _lib.KVCA_ERR_SIZE_LIMIT


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)


def _noalloc(lib, bits, order, meta, ss, blocked, count, out, st) -> int:
    return lib.kvca_pop_reusable_slots_noalloc(bits, order, _p(meta), meta.numel(), _p(ss), _p(blocked),
                                               blocked.numel(), count, _p(out), _p(st) if st is not None else
                                               ctypes.c_void_p(0), _stream())


@pytest.mark.parametrize("bits,order", [(8, 0), (16, 1)])
def test_noalloc_pop_errors_change_nothing_and_next_call_is_exact(bits, order):
    lib = _lib.load()
    n = 70_000
    rng = np.random.default_rng(77 + bits)
    meta = _table(rng, n, bits)
    ss = torch.tensor([12_345], dtype=torch.int64, device=DEV)
    st = torch.zeros(2, dtype=torch.int64, device=DEV)
    out = torch.full((64,), -7, dtype=torch.int64, device=DEV)
    meta0, ss0 = meta.clone(), ss.clone()

    # 1. a blocked id past the table: KVCA_ERR_BAD_INDEX with that id, no pop
    bad = torch.tensor([5, n + 3, 9], dtype=torch.int64, device=DEV)
    assert _noalloc(lib, bits, order, meta, ss, bad, 64, out, st) == 0
    torch.cuda.synchronize(DEV)
    assert st.tolist() == [_lib.KVCA_ERR_BAD_INDEX, n + 3]
    assert torch.equal(meta, meta0) and torch.equal(ss, ss0)
    assert out.tolist() == [-7] * 64
    neg = torch.tensor([-1], dtype=torch.int64, device=DEV)
    st.zero_()
    assert _noalloc(lib, bits, order, meta, ss, neg, 64, out, st) == 0
    torch.cuda.synchronize(DEV)
    assert st.tolist() == [_lib.KVCA_ERR_BAD_INDEX, -1]
    assert torch.equal(meta, meta0) and torch.equal(ss, ss0)

    # 2. the next call (its blocked ids marked in the array the failed call left) is exact
    st.zero_()
    blocked = torch.from_numpy(rng.integers(0, n, 300).astype(np.int64)).to(DEV)
    assert _noalloc(lib, bits, order, meta, ss, blocked, 64, out, st) == 0
    torch.cuda.synchronize(DEV)
    assert st.tolist() == [0, 0]
    meta_o, ss_o = meta0.cpu(), ss0.cpu()
    want = oracle.pop_reusable_slots(meta_o, ss_o, blocked.cpu(), 64, order="grouped" if order == 0 else "prefix")
    assert torch.equal(out.cpu(), want)
    assert torch.equal(meta.cpu().view(torch.uint8), meta_o.view(torch.uint8)) and torch.equal(ss.cpu(), ss_o)

    # 3. more than the reusable slots: KVCA_ERR_INSUFFICIENT_CAPACITY, slot_meta and search_start untouched
    f = bits // 2
    free = int((((meta.to(torch.int64) & ((1 << f) - 1)) == 0)).sum())
    meta1, ss1 = meta.clone(), ss.clone()
    big = torch.empty(free + 1, dtype=torch.int64, device=DEV)
    st.zero_()
    assert _noalloc(lib, bits, order, meta, ss, blocked[:0], free + 1, big, st) == 0
    torch.cuda.synchronize(DEV)
    assert st.tolist() == [_lib.KVCA_ERR_INSUFFICIENT_CAPACITY, free + 1]
    assert torch.equal(meta, meta1) and torch.equal(ss, ss1)

    # 4. then again exact, against the allocating pop on copies of the same state
    st.zero_()
    meta_a, ss_a = meta.clone(), ss.clone()
    bitmap = torch.zeros(int(lib.kvca_pop_scratch_bytes(n)) // 4, dtype=torch.int32, device=DEV)
    st_a = torch.zeros(2, dtype=torch.int64, device=DEV)
    out_a = torch.empty(500, dtype=torch.int64, device=DEV)
    out_b = torch.empty(500, dtype=torch.int64, device=DEV)
    blocked2 = torch.from_numpy(rng.integers(0, n, 40).astype(np.int64)).to(DEV)
    assert lib.kvca_pop_reusable_slots(bits, order, _p(meta_a), n, _p(ss_a), _p(blocked2), blocked2.numel(), 500,
                                       _p(out_a), _p(bitmap), _p(st_a), _stream()) == 0
    assert _noalloc(lib, bits, order, meta, ss, blocked2, 500, out_b, st) == 0
    torch.cuda.synchronize(DEV)
    assert st.tolist() == [0, 0] and st_a.tolist() == [0, 0]
    assert torch.equal(out_a, out_b)
    assert torch.equal(meta_a.view(torch.uint8), meta.view(torch.uint8)) and torch.equal(ss_a, ss)


def test_noalloc_pop_requires_status_words():
    lib = _lib.load()
    meta = torch.zeros(64, dtype=torch.uint8, device=DEV)
    ss = torch.zeros(1, dtype=torch.int64, device=DEV)
    out = torch.full((4,), -1, dtype=torch.int64, device=DEV)
    empty = torch.empty(0, dtype=torch.int64, device=DEV)
    assert _noalloc(lib, 8, 0, meta, ss, empty, 4, out, None) == _lib.KVCA_ERR_BAD_ARGUMENT
    torch.cuda.synchronize(DEV)
    assert out.tolist() == [-1] * 4 and ss.item() == 0
