"""GPU edge cases: empty requests on every adapter path and op, one-slot
tables, a batch that asks for every slot, and ids at the edges of the id
space."""
from __future__ import annotations

import pytest
import torch

from kv_cache_adapter_b200 import adapter as adapter_mod
from kv_cache_adapter_b200.errors import InsufficientCapacityError

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _empty():
    return torch.zeros(0, dtype=torch.int64, device=DEV)


@pytest.fixture(scope="module")
def ext():
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda as m

    return m


def _adapter(path, num_actual=4, num_logical=16, host=False):
    init = {i: torch.full((3,), float(i), device=DEV) for i in range(num_logical)}
    backend = adapter_mod.InMemoryBlockStoreBackend(init, num_logical_blocks=num_logical,
                                                    record_device_ops=path == "planned", host_tier=host,
                                                    device=DEV if host else None)
    ad = adapter_mod.KVCacheAdapter(num_actual, num_logical, torch.zeros((num_actual, 3), device=DEV), backend)
    ad._planned = path != "stepwise"
    assert (ad._planned and ad._device_store() is not None) == (path == "device_store")
    return ad


@pytest.mark.parametrize("path", ["device_store", "planned", "stepwise"])
def test_empty_requests_change_nothing(ext, path):
    E = _empty()
    ad = _adapter(path)
    state = [t.clone() for t in (ad._logical_to_physical, ad._physical_to_logical, ad._slot_meta, ad._search_start)]
    assert ad.load(E).numel() == 0
    ad.save(E, torch.zeros((0, 3), device=DEV))
    ad.release(E)
    for a, b in zip(state, (ad._logical_to_physical, ad._physical_to_logical, ad._slot_meta, ad._search_start)):
        assert torch.equal(a, b)
    ext.check_status(DEV)


@pytest.mark.parametrize("host", [False, True])
@pytest.mark.parametrize("path", ["device_store", "planned", "stepwise"])
def test_one_slot_table_and_full_batches(ext, path, host):
    if host and path == "planned":
        pytest.skip("the planned path is covered with a device store")
    ad = _adapter(path, num_actual=1, num_logical=3, host=host)
    assert ad.load(torch.tensor([2], device=DEV)).tolist() == [0]
    with pytest.raises(InsufficientCapacityError):  # the only slot is pinned
        ad.load(torch.tensor([1], device=DEV))
    ad.release(torch.tensor([2], device=DEV))
    assert ad.load(torch.tensor([1], device=DEV)).tolist() == [0]  # evicts 2
    assert ad.actual_blocks[0].tolist() == [1.0, 1.0, 1.0]
    ad.release(torch.tensor([1], device=DEV))
    # a batch that needs every slot of a bigger table, ids at both ends
    ad = _adapter(path, num_actual=4, num_logical=16, host=host)
    assert sorted(ad.load(torch.tensor([0, 15, 7, 8], device=DEV)).tolist()) == [0, 1, 2, 3]
    with pytest.raises(InsufficientCapacityError):
        ad.load(torch.tensor([1], device=DEV))
    with pytest.raises(ValueError):
        ad.load(torch.tensor([16], device=DEV))
    ext.check_status(DEV)


def test_empty_ops(ext):
    E = _empty()
    actual = torch.zeros((4, 8), device=DEV)
    assert ext.gather_blocks(actual, E).shape == (0, 8)
    ext.scatter_blocks(actual, E, torch.zeros((0, 8), device=DEV))
    ext.copy_blocks(actual, E, actual.clone(), E)
    ext.exchange_blocks(actual, E, torch.zeros((4, 8), device=DEV), E, E)
    planes = [torch.zeros((4, 2, 8), device=DEV) for _ in range(2)]
    ext.copy_tokens(planes, E, [p.clone() for p in planes], E)
    meta = torch.zeros(64, dtype=torch.uint8, device=DEV)
    ss = torch.zeros(1, dtype=torch.int64, device=DEV)
    victims, done = ext.clock_stream(meta, ss, 0, 1, E, 0)
    assert victims.numel() == 0 and int(done) == 0
    assert ext.pop_reusable_slots(meta, ss, E, 0).numel() == 0
    ext.check_status(DEV)
