"""GPU parity: the prefix-order clock sweep against the reference's own CUDA
kernel, run on the same device.

The reference's CUDA extension (``csrc/kv_adapter_cuda.cu`` +
``csrc/binding.cpp``) is compiled unchanged into ``oracle/_ref`` by
``oracle/build_ref.py``.  Its ``pop_reusable_slots`` (kernel
``kv_adapter_cuda.cu:64-237``, host side ``:406-450``) takes the unpacked
views the reference adapter derives from ``slot_meta`` (``usage_count`` uint8
and ``reusable_mask = pin == 0``, ``adapter.py:185-195``) and picks the first
``count`` available slots in scan order whose usage is at most the smallest
sufficient threshold -- the rule of ``KVCA_POP_ORDER_PREFIX``.  Each case runs
both on copies of one seeded state and compares the victims, the aged usage
of every slot, the untouched pins and ``search_start`` byte for byte, over
sequences of calls so each call starts from the state the previous one left.

The reference kernel counts thresholds up to its usage maximum 127
(``kv_adapter_cuda.cu:13``), so 16-bit tables keep usage at or below 127.
Blocked ids stay in range: the reference marks them with ``index_fill_``,
which would assert on the device for an out-of-range id.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from kv_cache_adapter_b200.errors import InsufficientCapacityError

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


@pytest.fixture(scope="module")
def ref():
    from oracle import build_ref

    if not build_ref.available():
        pytest.skip("reference CUDA extension not built (python -m oracle.build_ref)")
    return build_ref.load()


@pytest.fixture(scope="module")
def ops():
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda as m

    return m


def _pack(pins: np.ndarray, usage: np.ndarray, bits: int) -> torch.Tensor:
    f = bits // 2
    w = (pins.astype(np.int64) & ((1 << f) - 1)) | (usage.astype(np.int64) << f)
    return torch.from_numpy(w.astype(np.uint8 if bits == 8 else np.uint16)).to(DEV)


def _fields(meta: torch.Tensor, bits: int) -> tuple[torch.Tensor, torch.Tensor]:
    f = bits // 2
    w = meta.to(torch.int64)
    return w & ((1 << f) - 1), w >> f


class Pair:
    """One table held twice: packed words for this library, unpacked views for the reference."""

    def __init__(self, pins: np.ndarray, usage: np.ndarray, bits: int, start: int):
        self.bits = bits
        self.n = pins.size
        self.meta = _pack(pins, usage, bits)
        self.ss = torch.tensor([start], dtype=torch.int64, device=DEV)
        self.pins0 = torch.from_numpy(pins.astype(np.int64)).to(DEV)
        self.usage_ref = torch.from_numpy(usage.astype(np.uint8)).to(DEV)
        self.reusable_ref = self.pins0 == 0
        self.ss_ref = self.ss.clone()

    def pop_both(self, ops, ref, blocked: torch.Tensor, count: int):
        got = ops.pop_reusable_slots(self.meta, self.ss, blocked, count, order="prefix")
        want = ref.pop_reusable_slots(self.usage_ref, self.reusable_ref, self.ss_ref, blocked, count)
        torch.cuda.synchronize(DEV)
        return got, want

    def assert_same(self, got: torch.Tensor, want: torch.Tensor, what: str) -> None:
        pins, usage = _fields(self.meta, self.bits)
        assert torch.equal(got, want), f"{what}: victims differ"
        assert torch.equal(usage, self.usage_ref.to(torch.int64)), f"{what}: aged usage differs"
        assert torch.equal(pins, self.pins0), f"{what}: pins changed"
        assert torch.equal(self.ss, self.ss_ref), f"{what}: search_start differs"


def test_reference_kernel_known_answer_prefix_order(ops, ref):
    # test_adapter_npu_kernels.py:91-115's input: the grouped order gives [3, 0]; the
    # reference CUDA kernel (and KVCA_POP_ORDER_PREFIX) the first two in scan order
    p = Pair(np.array([0, 0, 1, 0]), np.array([1, 0, 0, 0]), 8, 0)
    got, want = p.pop_both(ops, ref, torch.tensor([1], dtype=torch.int64, device=DEV), 2)
    p.assert_same(got, want, "kat")
    assert got.tolist() == [0, 3] and p.ss.item() == 0 and p.usage_ref.tolist() == [0, 0, 0, 0]


CASES = [
    # bits, slots, usage high (exclusive), pinned fraction, blocked per call, calls
    (8, 1, 4, 0.0, 0, 3),
    (8, 2, 4, 0.0, 1, 4),
    (8, 31, 16, 0.2, 3, 12),
    (8, 32, 4, 0.1, 2, 12),
    (8, 33, 16, 0.3, 5, 12),
    (8, 255, 16, 0.1, 7, 10),
    (8, 256, 4, 0.05, 9, 10),
    (8, 257, 16, 0.5, 11, 10),
    (8, 1000, 16, 0.05, 40, 10),
    (8, 4097, 4, 0.05, 64, 8),
    (8, 65_536, 16, 0.05, 16, 6),
    (16, 300, 128, 0.1, 5, 10),
    (16, 5_000, 128, 0.3, 20, 8),
    (16, 70_001, 40, 0.05, 8, 5),
]


@pytest.mark.parametrize("bits,n,uhigh,pinned,nblocked,calls", CASES)
def test_prefix_pop_sequences_match_reference_kernel(ops, ref, bits, n, uhigh, pinned, nblocked, calls):
    rng = np.random.default_rng(1234 + n * 7 + bits)
    pins = np.where(rng.random(n) < pinned, rng.integers(1, 3, n), 0)
    usage = rng.integers(0, uhigh, n)
    p = Pair(pins, usage, bits, int(rng.integers(0, n)))
    for call in range(calls):
        blocked_np = rng.integers(0, n, nblocked)  # duplicates and pinned slots included
        blocked = torch.from_numpy(blocked_np.astype(np.int64)).to(DEV)
        avail = (pins == 0).copy()
        avail[blocked_np] = False
        if avail.sum() == 0:
            break
        # mostly small requests, sometimes all available slots (the largest threshold)
        count = int(avail.sum()) if call % 4 == 3 else int(rng.integers(1, max(2, min(avail.sum(), 3 * n // 4) + 1)))
        count = max(1, min(count, int(avail.sum())))
        got, want = p.pop_both(ops, ref, blocked, count)
        p.assert_same(got, want, f"call {call} count {count}")


@pytest.mark.parametrize("usage_high", [4, 16])
def test_prefix_pop_full_size_table_matches_reference_kernel(ops, ref, usage_high):
    """1,048,576 slots (the clock stress table): usage U{0..3} (a usage-0 slot
    is never far, no aging) and U{0..15} with few zeros; 5% pinned."""
    n = 1 << 20
    rng = np.random.default_rng(99 + usage_high)
    pins = (rng.random(n) < 0.05).astype(np.int64)
    usage = rng.integers(0, usage_high, n)
    if usage_high == 16:
        usage = np.where(usage == 0, rng.integers(1, 16, n), usage)  # no zeros: every call ages
        usage[rng.integers(0, n, 50)] = 0
    p = Pair(pins, usage, 8, int(rng.integers(0, n)))
    for call, (count, nb) in enumerate([(1, 0), (256, 0), (1, 32), (4096, 16), (300_000, 0), (7, 64)]):
        blocked = torch.from_numpy(rng.integers(0, n, nb).astype(np.int64)).to(DEV)
        got, want = p.pop_both(ops, ref, blocked, count)
        p.assert_same(got, want, f"call {call}")


def test_insufficient_capacity_both_refuse_and_change_nothing(ops, ref):
    rng = np.random.default_rng(5)
    n = 513
    pins = np.where(rng.random(n) < 0.9, 1, 0)
    usage = rng.integers(0, 16, n)
    p = Pair(pins, usage, 8, 17)
    free = int((pins == 0).sum())
    meta0, u0 = p.meta.clone(), p.usage_ref.clone()
    empty = torch.empty(0, dtype=torch.int64, device=DEV)
    with pytest.raises(InsufficientCapacityError):
        ops.pop_reusable_slots(p.meta, p.ss, empty, free + 1, order="prefix")
    with pytest.raises(RuntimeError):
        ref.pop_reusable_slots(p.usage_ref, p.reusable_ref, p.ss_ref, empty, free + 1)
    torch.cuda.synchronize(DEV)
    assert torch.equal(p.meta, meta0) and torch.equal(p.usage_ref, u0)
    assert p.ss.item() == 17 and p.ss_ref.item() == 17
    got, want = p.pop_both(ops, ref, empty, free)  # exactly the free slots still works
    p.assert_same(got, want, "after refusal")


@pytest.mark.parametrize("method", ["steps", "batched"])
def test_prefix_clock_stream_matches_reference_pops(ops, ref, method):
    """The device-resident clock stream in prefix order against the same stream
    composed from reference kernel pops: pop (no blocked slots), refill the
    victims with usage 1 (a save miss, adapter.py:647-651), then bump the step's
    re-accessed slots saturating (adapter.py:1414-1416)."""
    n, steps, alloc, reacc = 4096, 120, 3, 4
    rng = np.random.default_rng(4242)
    pins = (rng.random(n) < 0.05).astype(np.int64)
    usage = rng.integers(0, 4, n)
    usage = np.where(rng.random(n) < 0.9, np.maximum(usage, 1), usage)  # few zeros: aging recurs
    reaccess = torch.from_numpy(rng.integers(0, n, steps * reacc).astype(np.int64))
    p = Pair(pins, usage, 8, 0)
    got_v, done = ops.clock_stream(p.meta, p.ss, steps, alloc, reaccess.to(DEV), reacc, order="prefix",
                                   method=method)
    assert int(done) == steps
    empty = torch.empty(0, dtype=torch.int64, device=DEV)
    want_v = []
    for s in range(steps):
        v = ref.pop_reusable_slots(p.usage_ref, p.reusable_ref, p.ss_ref, empty, alloc)
        want_v.append(v)
        p.usage_ref[v] = 1
        r = reaccess[s * reacc:(s + 1) * reacc].to(DEV)
        bumped = torch.clamp(p.usage_ref[r].to(torch.int64) + 1, max=15).to(torch.uint8)
        p.usage_ref[r] = bumped
    torch.cuda.synchronize(DEV)
    assert torch.equal(got_v.reshape(-1), torch.cat(want_v))
    p.assert_same(got_v[:0], torch.cat(want_v)[:0], "stream")
