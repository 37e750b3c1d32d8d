"""GPU: small exhaustive cases of the clock sweep against the oracle: every
table of three slots with pins in {0, 1} and usage in {0..3}, every search
start, request size and blocked set, in both victim orders (including the
requests that must fail with InsufficientCapacityError and change nothing)."""
from __future__ import annotations

import itertools

import pytest
import torch

import oracle
from kv_cache_adapter_b200.errors import InsufficientCapacityError

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("order", ["grouped", "prefix"])
def test_every_three_slot_table(order):
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda as ops

    words = [(pin & 15) | (usage << 4) for pin in (0, 1) for usage in range(4)]
    blocked_sets = [[], [0], [2], [0, 1]]
    cases = 0
    for table in itertools.product(words, repeat=3):
        for start, count, blocked in itertools.product(range(3), (1, 2, 3), blocked_sets):
            meta_h = torch.tensor(table, dtype=torch.uint8)
            ss_h = torch.tensor([start], dtype=torch.int64)
            b_h = torch.tensor(blocked, dtype=torch.int64)
            try:
                want = oracle.pop_reusable_slots(meta_h, ss_h, b_h, count, order=order).tolist()
            except oracle.OracleInsufficientCapacity:
                want = None
            meta_d = torch.tensor(table, dtype=torch.uint8, device=DEV)
            ss_d = torch.tensor([start], dtype=torch.int64, device=DEV)
            if want is None:
                with pytest.raises(InsufficientCapacityError):
                    ops.pop_reusable_slots(meta_d, ss_d, b_h.to(DEV), count, order=order)
                assert meta_d.tolist() == list(table) and int(ss_d[0]) == start
            else:
                got = ops.pop_reusable_slots(meta_d, ss_d, b_h.to(DEV), count, order=order).tolist()
                assert got == want, (table, start, count, blocked)
                assert meta_d.cpu().tolist() == meta_h.tolist(), (table, start, count, blocked)
                assert int(ss_d[0]) == int(ss_h[0])
            cases += 1
    assert cases == 512 * 3 * 3 * 4
    ops.check_status(DEV)


def test_release_wraps_every_pin_value():
    """Release of every 4-bit pin value (0 wraps to 15) and every usage."""
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda as ops

    n = 256
    meta_h = torch.arange(n, dtype=torch.int64).to(torch.uint8)  # every (pin, usage) word once
    l2p_h = torch.arange(n, dtype=torch.int64)
    ids_h = torch.arange(n, dtype=torch.int64)
    oracle.release_metadata(l2p_h, meta_h, ids_h)
    meta_d = torch.arange(n, dtype=torch.int64).to(torch.uint8).to(DEV)
    ops.release_metadata(l2p_h.to(DEV), meta_d, ids_h.to(DEV), check=True)
    assert torch.equal(meta_d.cpu(), meta_h)
    pins = (meta_h.to(torch.int32) & 15).tolist()
    assert pins == [((w & 15) - 1) % 16 for w in range(n)]
