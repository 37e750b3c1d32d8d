"""GPU parity: the whole-GPU clock sweep that kvca_pop_reusable_slots runs on
tables of 65,536 to 2^24 slots, against the oracle's restatement of the
reference (adapter.py:472-525 grouped order; kv_adapter_cuda.cu:101-236
prefix order) and against the one-CTA kernel (the no-alloc entry point runs
it), bit for bit: victims, every slot word and search_start.

The cases aim at the places where the scan order is cut into per-CTA ranges:
a scan start inside a 16-byte vector (the vector is split between the first
range and the last), blocked slots on both sides of the start, requests that
CTA 0's range alone satisfies with usage-0 slots and requests just past it,
pops that age every slot, 16-bit words with thresholds far above 15, and the
error paths (bad blocked id, too few reusable slots), which change nothing.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import oracle
from kv_cache_adapter_b200 import _lib
from kv_cache_adapter_b200.errors import InsufficientCapacityError

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
ORDERS = {"grouped": 0, "prefix": 1}


@pytest.fixture(scope="module")
def ops():
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda as m

    return m


def _table(rng, n: int, bits: int, kind: str) -> np.ndarray:
    f = bits // 2
    if kind == "zeros":  # usage U{0..3}: CTA 0's range usually holds the victims
        usage = rng.integers(0, 4, n)
    elif kind == "aging":  # no usage-0 slot: every pop ages
        usage = rng.integers(1, 16, n)
    elif kind == "sparse":  # a few usage-0 slots spread over the table
        usage = np.where(rng.random(n) < 0.001, 0, rng.integers(1, 6, n))
    else:  # wide 16-bit usage
        usage = rng.integers(0, 256 if bits == 16 else 16, n)
    pins = np.where(rng.random(n) < 0.07, rng.integers(1, 4, n), 0)
    return (pins | (usage << f)).astype(np.uint8 if bits == 8 else np.uint16)


def _check_pop(ops, meta_np: np.ndarray, start: int, blocked_np: np.ndarray, count: int, order: str):
    """One pop on the GPU (whole-GPU path), the oracle and the one-CTA kernel."""
    meta = torch.from_numpy(meta_np.copy()).to(DEV)
    ss = torch.tensor([start], dtype=torch.int64, device=DEV)
    blocked = torch.from_numpy(blocked_np.astype(np.int64)).to(DEV)
    meta_o = torch.from_numpy(meta_np.copy())
    ss_o = torch.tensor([start], dtype=torch.int64)
    want = oracle.pop_reusable_slots(meta_o, ss_o, blocked.cpu(), count, order=order)
    got = ops.pop_reusable_slots(meta, ss, blocked, count, order=order)
    torch.cuda.synchronize(DEV)
    assert torch.equal(got.cpu(), want), "victims"
    assert np.array_equal(meta.cpu().numpy(), meta_o.numpy()), "slot words"
    assert int(ss[0]) == int(ss_o[0]), "search_start"
    # the one-CTA kernel on the same input (the no-alloc entry point runs it)
    if meta_np.size <= _lib.KVCA_NOALLOC_MAX_SLOTS:
        lib = _lib.load()
        m1 = torch.from_numpy(meta_np.copy()).to(DEV)
        s1 = torch.tensor([start], dtype=torch.int64, device=DEV)
        o1 = torch.empty(count, dtype=torch.int64, device=DEV)
        st = torch.zeros(2, dtype=torch.int64, device=DEV)
        p = lambda t: ctypes.c_void_p(t.data_ptr() if t.numel() else 0)  # noqa: E731
        bits = 8 if meta_np.dtype == np.uint8 else 16
        assert lib.kvca_pop_reusable_slots_noalloc(bits, ORDERS[order], p(m1), m1.numel(), p(s1), p(blocked),
                                                   blocked.numel(), count, p(o1), p(st),
                                                   ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)) == 0
        torch.cuda.synchronize(DEV)
        assert st.tolist() == [0, 0]
        assert torch.equal(o1, got) and torch.equal(m1, meta) and torch.equal(s1, ss), "one-CTA kernel differs"
    return meta, ss


@pytest.mark.parametrize("bits", [8, 16])
@pytest.mark.parametrize("order", ["grouped", "prefix"])
@pytest.mark.parametrize("n", [65_536, 65_537, 1 << 20])
@pytest.mark.parametrize("kind", ["zeros", "aging", "sparse", "wide"])
def test_grid_pop_matches_oracle_and_one_cta_kernel(ops, bits, order, n, kind):
    rng = np.random.default_rng(n * 31 + bits * 7 + len(kind) + (order == "prefix"))
    meta_np = _table(rng, n, bits, kind)
    spv = 16 if bits == 8 else 8
    free = int(((meta_np.astype(np.int64) & ((1 << (bits // 2)) - 1)) == 0).sum())
    starts = [0, 1, spv - 1, spv, n - 1, int(rng.integers(0, n))]
    for i, start in enumerate(starts):
        v0 = start - start % spv
        blocked = np.concatenate([
            rng.integers(0, n, 40),                                  # anywhere, duplicates allowed
            np.arange(v0, min(v0 + spv, n)),                         # the start vector, both sides of the start
            rng.integers(0, n, 3),
        ])
        counts = [1, 7, 300, 5_000, free // 2, free - len(set(blocked.tolist())) - 1]
        count = max(1, min(counts[i % len(counts)], free - len(np.unique(blocked)) - 1))
        _check_pop(ops, meta_np, start, blocked, count, order)


@pytest.mark.parametrize("order", ["grouped", "prefix"])
def test_grid_pop_sequence_keeps_state(ops, order):
    """A run of pops, each starting where the previous left search_start and
    the aging left the words, with refills in between (a save miss)."""
    n = 300_001
    rng = np.random.default_rng(7 if order == "grouped" else 8)
    meta_np = _table(rng, n, 8, "sparse")
    meta = torch.from_numpy(meta_np.copy()).to(DEV)
    meta_o = torch.from_numpy(meta_np.copy())
    ss = torch.zeros(1, dtype=torch.int64, device=DEV)
    ss_o = torch.zeros(1, dtype=torch.int64)
    for call in range(40):
        count = int(rng.choice([1, 3, 64, 700, 2_500]))
        blocked = torch.from_numpy(rng.integers(0, n, int(rng.integers(0, 50))).astype(np.int64))
        want = oracle.pop_reusable_slots(meta_o, ss_o, blocked, count, order=order)
        got = ops.pop_reusable_slots(meta, ss, blocked.to(DEV), count, order=order)
        assert torch.equal(got.cpu(), want), call
        refill = want[: count // 2]
        meta_o[refill] = (meta_o[refill] & 15) | (1 << 4)
        meta[got[: count // 2]] = (meta[got[: count // 2]] & 15) | (1 << 4)
        torch.cuda.synchronize(DEV)
        assert torch.equal(meta.cpu(), meta_o) and int(ss[0]) == int(ss_o[0]), call


def test_grid_pop_largest_table(ops):
    n = 1 << 24  # the largest table the whole-GPU pop takes
    rng = np.random.default_rng(24)
    meta_np = _table(rng, n, 8, "sparse")
    for start, count in ((0, 1), (n - 5, 20_000)):
        _check_pop(ops, meta_np, start, rng.integers(0, n, 100), count, "grouped")


def test_grid_pop_errors_change_nothing(ops):
    n = 1 << 17
    rng = np.random.default_rng(3)
    meta_np = _table(rng, n, 8, "aging")
    meta = torch.from_numpy(meta_np.copy()).to(DEV)
    ss = torch.tensor([12_345], dtype=torch.int64, device=DEV)
    with pytest.raises(IndexError):
        ops.pop_reusable_slots(meta, ss, torch.tensor([5, n], dtype=torch.int64, device=DEV), 10)
    with pytest.raises(IndexError):
        ops.pop_reusable_slots(meta, ss, torch.tensor([-1], dtype=torch.int64, device=DEV), 10)
    free = int(((meta_np & 15) == 0).sum())
    with pytest.raises(InsufficientCapacityError):
        ops.pop_reusable_slots(meta, ss, torch.empty(0, dtype=torch.int64, device=DEV), free + 1)
    torch.cuda.synchronize(DEV)
    assert np.array_equal(meta.cpu().numpy(), meta_np) and int(ss[0]) == 12_345
    _check_pop(ops, meta_np, 12_345, np.array([], dtype=np.int64), free, "grouped")  # exactly all free slots
