"""GPU parity: KVCacheAdapter on CUDA tensors against the reference.

* 60 recorded reference scenarios (tests/golden/scenarios_u8.json): identical
  results, errors and full adapter/backend state after every op.
* The reference's own adapter tests (test_adapter.py:65-343), run on CUDA.
"""
from __future__ import annotations

import json

import pytest
import torch

import scenario_runner
from kv_cache_adapter_b200 import adapter as adapter_mod

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _ids(v):
    return torch.tensor(v, dtype=torch.int64, device=DEV)


def _payload(rows):
    return torch.tensor(rows, dtype=torch.float32, device=DEV)


@pytest.fixture(scope="module")
def api():
    import kv_cache_adapter_b200 as m

    return m


def make_adapter(api, num_actual=2, num_logical=8, backend=None):
    return api.KVCacheAdapter(
        num_actual, num_logical, torch.zeros((num_actual, 2), dtype=torch.float32, device=DEV),
        backend or api.InMemoryBlockStoreBackend(num_logical_blocks=num_logical, record_device_ops=True))


def backend_with(api, rows: dict[int, list[float]], **kw):
    return api.InMemoryBlockStoreBackend({k: _payload(v) for k, v in rows.items()}, record_device_ops=True, **kw)


@pytest.mark.parametrize("path", ["device_store", "planned", "stepwise"])
@pytest.mark.parametrize("case_index", range(60))
def test_recorded_reference_scenarios(case_index, path):
    """device_store: plan, spill, fill and commit enqueued with one host read
    (the backend's storage lives on the GPU once it has any block); planned:
    one-launch plan, then the backend calls; stepwise: inspect, pop, commit as
    separate launches."""
    case = scenario_runner.load_scenarios()[case_index]
    scenario_runner.run_and_compare(case, DEV, planned=path != "stepwise", record=path != "device_store")
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda

    kv_cache_adapter_cuda.check_status(DEV)  # nothing latched by the unchecked launches


def test_runtime_path_and_native_library_loaded(api):
    ad = make_adapter(api)
    assert ad.runtime_path == "cuda_ext_meta"
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda

    assert ad._native_ext is kv_cache_adapter_cuda
    with pytest.raises(RuntimeError, match="strict CUDA path is disabled"):
        api.KVCacheAdapter(2, 8, torch.zeros((2, 2), device=DEV), api.InMemoryBlockStoreBackend(num_logical_blocks=8),
                           prefer_native_extension=False)


def test_free_slots_are_preloaded_into_reusable_lru(api):
    ad = make_adapter(api, num_actual=3)
    snap = ad.debug_snapshot()
    assert snap["lru_unpinned"] == [0, 1, 2]
    assert snap["actual_blocks"].shape == (3, 2)


def test_load_preserves_order_without_internal_reordering(api):
    backend = backend_with(api, {3: [3, 30], 5: [5, 50]})
    ad = make_adapter(api, backend=backend)
    assert ad.load(_ids([3, 5])).tolist() == [0, 1]
    assert backend.load_calls == [3, 5]
    ad.release(_ids([3, 5]))


def test_lru_evicts_only_unpinned_blocks(api):
    backend = backend_with(api, {0: [0, 10], 1: [1, 11], 2: [2, 12]})
    ad = make_adapter(api, backend=backend)
    physical = ad.load(_ids([0, 1]))
    ad.release(_ids([0]))
    slot_for_2 = ad.load(_ids([2]))
    l2p = ad.debug_snapshot()["logical_to_physical"]
    assert physical.tolist() == [0, 1] and slot_for_2.tolist() == [0]
    assert l2p[1] == 1 and l2p[2] == 0 and 0 not in l2p
    assert backend.save_calls == [0]
    assert backend.operation_log[-2:] == [("save", 0), ("load", 2)]


def test_load_raises_when_all_resident_blocks_are_pinned(api):
    backend = backend_with(api, {0: [0, 10], 1: [1, 11]})
    ad = make_adapter(api, num_actual=1, backend=backend)
    ad.load(_ids([0]))
    with pytest.raises(api.InsufficientCapacityError):
        ad.load(_ids([1]))


def test_updated_payload_is_spilled_when_its_resident_slot_is_eventually_evicted(api):
    backend = backend_with(api, {i: [i, 10 + i] for i in range(6)})
    ad = make_adapter(api, backend=backend)
    updated = _payload([100, 101])
    ad.load(_ids([0]))
    ad.save(_ids([0]), updated.unsqueeze(0))
    ad.release(_ids([0]))
    for lid in [1, 2, 3, 4, 5]:
        ad.load(_ids([lid]))
        if 0 not in ad.debug_snapshot()["logical_to_physical"]:
            break
        ad.release(_ids([lid]))
    else:
        raise AssertionError("logical block 0 never got evicted")
    assert torch.equal(backend.snapshot()[0], updated.cpu())
    assert ("save", 0) in backend.operation_log


def test_load_missing_block_raises_backend_error(api):
    ad = make_adapter(api)
    with pytest.raises(api.BlockNotFoundError):
        ad.load(_ids([4]))


def test_load_fills_multiple_slots_with_batched_copy(api):
    backend = backend_with(api, {i: [i, 10 + i] for i in range(4)})
    ad = make_adapter(api, num_actual=4, backend=backend)
    ad.load(_ids([0, 1, 2, 3]))
    assert torch.equal(ad.debug_snapshot()["actual_blocks"], torch.tensor([[0., 10], [1, 11], [2, 12], [3, 13]]))


def test_save_updates_actual_blocks(api):
    backend = backend_with(api, {i: [i, 10 + i] for i in range(4)})
    ad = make_adapter(api, backend=backend)
    ad.load(_ids([0, 1]))
    ad.save(_ids([0, 1]), _payload([[100, 101], [110, 111]]))
    ad.release(_ids([0, 1]))
    ad.save(_ids([2, 3]), _payload([[200, 201], [300, 301]]))
    assert torch.equal(backend.snapshot()[0], torch.tensor([100., 101.]))
    assert torch.equal(backend.snapshot()[1], torch.tensor([110., 111.]))
    assert torch.equal(ad.debug_snapshot()["actual_blocks"], torch.tensor([[200., 201], [300, 301]]))


def test_save_and_load_round_trip_across_evictions(api):
    """test_adapter.py:272-343 of the reference, on CUDA."""
    ad = make_adapter(api)
    expected = {i: _payload([[10 * (i + 1), 10 * (i + 1) + 1]])[0] for i in range(5)}

    def check(ids):
        slots = ad.load(_ids(ids))
        for lid, slot in zip(ids, slots.tolist()):
            assert torch.equal(ad.get_actual_block(int(slot)), expected[lid])
        ad.release(_ids(ids))

    ad.save(_ids([0, 1]), torch.stack((expected[0], expected[1])))
    check([0, 1])
    ad.save(_ids([2]), expected[2].unsqueeze(0))
    check([1, 2])
    ad.save(_ids([3]), expected[3].unsqueeze(0))
    check([3, 0])
    expected[2] = _payload([[300, 301]])[0]
    ad.save(_ids([2]), expected[2].unsqueeze(0))
    check([2, 1])
    ad.save(_ids([4]), expected[4].unsqueeze(0))
    check([4, 3])


def test_out_of_range_logical_id_raises_value_error(api):
    ad = make_adapter(api)
    with pytest.raises(ValueError):
        ad.load(_ids([8]))
    with pytest.raises(ValueError):
        ad.save(_ids([-1]), _payload([[1, 2]]))


def test_program_transcript_on_cuda(api, golden_dir):
    expected = json.loads((golden_dir / "program.json").read_text())["stdout"]
    backend = api.InMemoryBlockStoreBackend({i: _payload([float(i), 10.0 + i]) for i in range(4)})
    ad = api.KVCacheAdapter(2, 4, torch.zeros((2, 2), device=DEV), backend)
    assert ad.load(_ids([0, 1])).tolist() == [0, 1]
    assert expected[1].endswith("tensor([0, 1])")
    ad.release(_ids([0]))
    assert ad.load(_ids([2])).tolist() == [0]
    ad.save(_ids([2]), _payload([[200.0, 201.0]]))
    ad.release(_ids([1, 2]))
    assert ad.load(_ids([2, 3])).tolist() == [0, 1]
    assert ad.debug_snapshot()["logical_to_physical"] == {2: 0, 3: 1}


@pytest.mark.parametrize("path", ["planned", "stepwise", "device_store"])
def test_save_materializes_cold_block_by_evicting_unpinned_resident(api, path):
    """test_adapter.py:165-199 on CUDA, on each path (the operation log is
    recorded, so compared, on the first two)."""
    record = path != "device_store"
    backend = api.InMemoryBlockStoreBackend({k: _payload(v) for k, v in {0: [0, 10], 1: [1, 11], 2: [2, 12]}.items()},
                                            record_device_ops=record)
    ad = make_adapter(api, backend=backend)
    ad._planned = path != "stepwise"
    updated, inserted = _payload([[100, 101]]), _payload([[200, 201]])
    ad.load(_ids([0, 1]))
    ad.save(_ids([0]), updated)
    ad.release(_ids([0, 1]))
    ad.save(_ids([2]), inserted)
    snap = ad.debug_snapshot()
    l2p = snap["logical_to_physical"]
    assert 2 in l2p
    evicted = {0, 1} - set(l2p)
    assert len(evicted) == 1
    if record:
        assert backend.operation_log[-1] == ("save", next(iter(evicted)))
    assert torch.equal(snap["actual_blocks"][l2p[2]], inserted[0].cpu())
    if 0 in l2p:
        assert torch.equal(snap["actual_blocks"][l2p[0]], updated[0].cpu())
    else:
        assert torch.equal(backend.snapshot()[0], updated[0].cpu())
    ad.shutdown()


@pytest.mark.parametrize("target_device", ["cuda", "cpu"])
def test_host_tier_loads_into_target_slots_in_place(api, target_device):
    """test_adapter.py:346-401 (LMCacheBackend, CPU and CUDA targets) against
    the pinned host tier."""
    backend = api.HostTierBackend(block_shape=(2,), block_dtype=torch.float32, num_logical_blocks=8,
                                  model_name="kv-cache-adapter-test", max_local_cpu_size_gb=0.01, device=DEV)
    target = torch.full((3, 2), -1.0, dtype=torch.float32, device=target_device)
    backend.save_blocks(_ids([1, 3]), _payload([[10, 11], [30, 31]]))
    backend.load_blocks(_ids([3, 1]), target, torch.tensor([0, 2], device=target_device))
    torch.cuda.synchronize()
    assert torch.equal(target.cpu(), torch.tensor([[30.0, 31.0], [-1.0, -1.0], [10.0, 11.0]]))
    backend.shutdown()


def test_host_tier_load_restores_flattened_merged_kv_payload(api):
    """test_adapter.py:452-478: a row stored in LMCache's transfer layout comes
    back as the merged block."""
    block_shape = (2, 4, 2, 3)
    layout = adapter_mod._MergedKVBlockLayout.detect(block_shape)
    backend = api.HostTierBackend(block_shape=block_shape, block_dtype=torch.float32, num_logical_blocks=8,
                                  max_local_cpu_size_gb=0.01, device=DEV)
    payload = torch.arange(1, 1 + 2 * 4 * 2 * 3, dtype=torch.float32).view(block_shape)
    flattened = layout.flatten_block_batch(payload.unsqueeze(0))[0].contiguous()
    backend.save_blocks(_ids([7]), payload.unsqueeze(0).to(DEV))
    assert torch.equal(backend.transfer_view(7), flattened)
    actual = torch.zeros((1,) + block_shape, dtype=torch.float32, device=DEV)
    backend.load_blocks(_ids([7]), actual, _ids([0]))
    assert torch.equal(actual[0].cpu(), payload)
    backend.shutdown()
