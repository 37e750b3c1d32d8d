"""GPU parity: the one-launch load / save planners (plan_load, plan_save)
against the same steps composed from the oracle (inspect -> split -> pop ->
eviction plan, adapter.py:221-243 and :264-305), and the planned adapter
against the oracle-backed adapter over long random programs."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from oracle_ops import OracleOps
from kv_cache_adapter_b200 import adapter as adapter_mod
from kv_cache_adapter_b200.errors import InsufficientCapacityError

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


@pytest.fixture(scope="module")
def ops():
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda as m

    return m


def _pack(pins, usage, bits):
    f = bits // 2
    mask = (1 << f) - 1
    w = (np.asarray(pins, dtype=np.int64) & mask) | ((np.asarray(usage, dtype=np.int64) & mask) << f)
    return torch.from_numpy(w.astype(np.uint8 if bits == 8 else np.uint16))


def _usage(meta: torch.Tensor, bits: int) -> np.ndarray:
    f = bits // 2
    return (meta.numpy().astype(np.int64) >> f) & ((1 << f) - 1)


def _table(rng, n_logical, n_slots, bits, pinned_frac):
    umax = (1 << (bits // 2)) - 1
    resident = rng.permutation(n_logical)[: int(rng.integers(0, n_slots + 1))]
    slots = rng.permutation(n_slots)[: resident.size]
    l2p = np.full(n_logical, -1, np.int64)
    l2p[resident] = slots
    p2l = np.full(n_slots, -1, np.int64)
    p2l[slots] = resident
    # a few stale reverse entries: slots that still name a logical id which has moved on
    stale = np.flatnonzero(p2l < 0)[: max(1, n_slots // 50)]
    p2l[stale] = rng.integers(0, n_logical, stale.size)
    pins = np.where(rng.random(n_slots) < pinned_frac, rng.integers(1, umax + 1, n_slots), 0)
    usage = rng.integers(0, min(umax, 6) + 1, n_slots)
    return torch.from_numpy(l2p), torch.from_numpy(p2l), _pack(pins, usage, bits)


def _request(rng, n_logical, k, dup_frac):
    ids = rng.integers(0, n_logical, k)
    dup = rng.random(k) < dup_frac
    if k > 1:
        ids[dup] = ids[rng.integers(0, k, int(dup.sum()))]
    return torch.from_numpy(ids.astype(np.int64))


def _expected_load(l2p, p2l, meta, ss, ids, order, bits):
    cur, resident, pins, usage = oracle.inspect_load_requests(l2p, meta, ids)
    hit_pos = torch.nonzero(resident.bool()).flatten()
    miss_pos = torch.nonzero(~resident.bool()).flatten()
    hit_slots = cur[hit_pos]
    miss_ids = ids[miss_pos]
    if miss_pos.numel():
        victims = oracle.pop_reusable_slots(meta, ss, hit_slots, miss_pos.numel(), order=order)
    else:
        victims = torch.zeros(0, dtype=torch.int64)
    prev = p2l[victims]
    ev = (prev >= 0) & (prev != miss_ids)
    umax = (1 << (bits // 2)) - 1
    if miss_pos.numel() and hit_pos.numel():
        hit_usage = np.minimum(_usage(meta[hit_slots], bits) + 1, umax)
    else:
        hit_usage = usage[hit_pos].numpy().astype(np.int64)
    result = cur.clone()
    result[miss_pos] = victims
    return dict(result=result.tolist(), hit_slots=hit_slots.tolist(), hit_pins=pins[hit_pos].tolist(),
                hit_usage=hit_usage.tolist(), miss_ids=miss_ids.tolist(), victims=victims.tolist(),
                evict_ids=prev[ev].tolist(), evict_slots=victims[ev].tolist())


def _expected_save(l2p, p2l, meta, ss, ids, order, bits):
    cur, existing, usage = oracle.inspect_save_requests(l2p, meta, ids)
    ex_pos = torch.nonzero(existing.bool()).flatten()
    miss_pos = torch.nonzero(~existing.bool()).flatten()
    if miss_pos.numel():
        allocated = oracle.pop_reusable_slots(meta, ss, cur[ex_pos], miss_pos.numel(), order=order)
    else:
        allocated = torch.zeros(0, dtype=torch.int64)
    selected = cur.clone()
    selected[miss_pos] = allocated
    f = bits // 2
    pins = meta[selected].numpy().astype(np.int64) & ((1 << f) - 1)
    umax = (1 << f) - 1
    final_usage = np.minimum(_usage(meta[selected], bits) + 1, umax)
    final_usage[miss_pos.numpy()] = 1
    prev = p2l[selected]
    ev = (prev >= 0) & (prev != ids)
    sel = selected.tolist()
    ex = existing.tolist()
    move = [s if not ex[i] or s not in sel[i + 1:] else -1 for i, s in enumerate(sel)]
    return dict(selected=sel, move_slots=move, final_pins=pins.tolist(), final_usage=final_usage.tolist(),
                allocated=allocated.tolist(), evict_ids=prev[ev].tolist(), evict_slots=selected[ev].tolist())


def _as_lists(plan, fields):
    return {f: getattr(plan, f).to(torch.int64).tolist() for f in fields}


CASES = [  # n_logical, n_slots, k, pinned_frac, dup_frac
    (8, 4, 3, 0.0, 0.0),
    (64, 16, 8, 0.2, 0.3),
    (5000, 1000, 700, 0.1, 0.1),
    (50000, 20000, 3000, 0.05, 0.05),   # several 1024-id tiles
    (4 << 20, 1 << 20, 4096, 0.05, 0.02),
]


@pytest.mark.parametrize("bits", [8, 16])
@pytest.mark.parametrize("order", ["grouped", "prefix"])
@pytest.mark.parametrize("case", range(len(CASES)))
def test_plans_match_oracle_composition(ops, bits, order, case):
    n_logical, n_slots, k, pinned, dup = CASES[case]
    rng = np.random.default_rng(1000 * case + bits + (7 if order == "prefix" else 0))
    for trial in range(3):
        l2p, p2l, meta = _table(rng, n_logical, n_slots, bits, pinned)
        start = int(rng.integers(0, n_slots))
        ids = _request(rng, n_logical, k, dup)
        for kind in ("load", "save"):
            m_h = meta.clone()
            ss_h = torch.tensor([start], dtype=torch.int64)
            try:
                expect = (_expected_load if kind == "load" else _expected_save)(
                    l2p, p2l, m_h, ss_h, ids, order, bits)
            except oracle.OracleInsufficientCapacity:
                expect = None
            m_d = meta.to(DEV)
            ss_d = torch.tensor([start], dtype=torch.int64, device=DEV)
            args = (l2p.to(DEV), p2l.to(DEV), m_d, ss_d, ids.to(DEV))
            if expect is None:
                with pytest.raises(InsufficientCapacityError):
                    getattr(ops, f"plan_{kind}")(*args, order=order)
            else:
                got = _as_lists(getattr(ops, f"plan_{kind}")(*args, order=order), expect.keys())
                for f in expect:
                    assert got[f] == expect[f], (trial, kind, f)
            assert torch.equal(m_d.cpu(), m_h), (trial, kind)
            assert int(ss_d[0]) == int(ss_h[0])
            assert int(ops._bitmap(DEV, n_slots).count_nonzero()) == 0
    ops.check_status(DEV)


def test_plan_errors_change_nothing(ops):
    bits = 8
    rng = np.random.default_rng(5)
    l2p, p2l, _ = _table(rng, 100, 10, bits, 0.0)
    meta = _pack(np.ones(10, np.int64), np.zeros(10, np.int64), bits)  # every slot pinned
    meta[3] = int(_pack([0], [2], bits)[0])                              # one reusable slot
    L, P, M = l2p.to(DEV), p2l.to(DEV), meta.to(DEV)
    ss = torch.tensor([4], dtype=torch.int64, device=DEV)
    misses = torch.from_numpy(np.flatnonzero(l2p.numpy() < 0)[:2].astype(np.int64)).to(DEV)
    for fn in (ops.plan_load, ops.plan_save):
        with pytest.raises(InsufficientCapacityError):
            fn(L, P, M, ss, misses)
        with pytest.raises(IndexError):
            fn(L, P, M, ss, torch.tensor([0, 100], dtype=torch.int64, device=DEV))
        with pytest.raises(IndexError):
            fn(L, P, M, ss, torch.tensor([-1], dtype=torch.int64, device=DEV))
        assert torch.equal(M.cpu(), meta) and int(ss[0]) == 4
        assert int(ops._bitmap(DEV, 10).count_nonzero()) == 0
    ops.check_status(DEV)
    # one miss fits the one reusable slot
    plan = ops.plan_load(L, P, M, ss, misses[:1])
    assert plan.victims.tolist() == [3]


@pytest.mark.parametrize("bits", [8, 16])
def test_commits_keep_last_occurrence(ops, bits):
    """Repeated ids in the commits: the slot of the last occurrence stays, as
    the reference's index_put_ applied in order leaves it."""
    rng = np.random.default_rng(77 + bits)
    for trial in range(6):
        n_logical, n_slots = 3000, 2500
        l2p, p2l, meta = _table(rng, n_logical, n_slots, bits, 0.0)
        free = np.flatnonzero(l2p.numpy() < 0)
        k = int(rng.integers(2, 2000))
        miss_ids = torch.from_numpy(rng.choice(free[:40], k).astype(np.int64))  # many repeats
        slots = torch.from_numpy(rng.permutation(n_slots)[:k].astype(np.int64))
        evicted = torch.from_numpy(rng.choice(n_logical, 5).astype(np.int64))
        usage = torch.ones(k, dtype=meta.dtype)
        none = torch.zeros(0, dtype=torch.int64)
        host = [l2p.clone(), p2l.clone(), meta.clone()]
        dev = [t.to(DEV) for t in (l2p, p2l, meta)]
        oracle.commit_load_metadata(*host, evicted, miss_ids, slots, none, none, usage[:0], usage)
        ops.commit_load_metadata(*dev, evicted.to(DEV), miss_ids.to(DEV), slots.to(DEV), none.to(DEV),
                                 none.to(DEV), usage[:0].to(DEV), usage.to(DEV))
        for h, d in zip(host, dev):
            assert torch.equal(d.cpu(), h), trial
        host = [l2p.clone(), p2l.clone(), meta.clone()]
        dev = [t.to(DEV) for t in (l2p, p2l, meta)]
        pins = torch.zeros(k, dtype=meta.dtype)
        oracle.commit_save_metadata(*host, evicted, miss_ids, slots, pins, usage)
        ops.commit_save_metadata(*dev, evicted.to(DEV), miss_ids.to(DEV), slots.to(DEV), pins.to(DEV),
                                 usage.to(DEV))
        for h, d in zip(host, dev):
            assert torch.equal(d.cpu(), h), trial
    ops.check_status(DEV)


def test_save_with_repeated_ids_keeps_last_row(api_gpu):
    ad = api_gpu.KVCacheAdapter(8, 32, torch.zeros((8, 4), device=DEV),
                                api_gpu.InMemoryBlockStoreBackend(num_logical_blocks=32))
    for planned in (True, False):
        ad._planned = planned
        ids = torch.tensor([5, 6, 5, 5, 7, 6], dtype=torch.int64, device=DEV)
        rows = torch.arange(24, dtype=torch.float32, device=DEV).reshape(6, 4) + (100 if planned else 0)
        ad.save(ids, rows)  # first save: all missing, each occurrence gets a slot
        ad.save(ids, rows + 1)  # second save: all existing, repeated slots
        slot5 = int(ad._logical_to_physical[5])
        slot6 = int(ad._logical_to_physical[6])
        assert torch.equal(ad.actual_blocks[slot5], rows[3] + 1)
        assert torch.equal(ad.actual_blocks[slot6], rows[5] + 1)
        ad.release(torch.tensor([5, 6, 7], dtype=torch.int64, device=DEV))


@pytest.mark.parametrize("path", ["device_store", "planned"])
@pytest.mark.parametrize("seed,num_actual,num_logical,max_batch,shape", [
    (1, 4, 16, 4, (2, 3)),
    (2, 64, 256, 48, (2, 3)),
    (3, 1000, 4000, 700, (2, 3)),
    (4, 3000, 20000, 2500, (2, 3)),
    # 128 KiB blocks: calls above the one-launch size limit take the
    # multi-launch device-store sequence, small ones the single launch
    (5, 4, 16, 4, (32, 1024)),
    (6, 64, 256, 48, (32, 1024)),
])
def test_planned_adapter_matches_oracle_adapter(api_gpu, seed, num_actual, num_logical, max_batch, shape, path):
    """Random load / save / release programs with duplicates, pin pressure,
    capacity errors and blocks missing from the store: the CUDA adapter (store
    driven on the device, or plan + backend calls) and the oracle-backed CPU
    adapter agree on every result, error and the full state after each op."""
    rng = np.random.default_rng(seed)
    # a few logical blocks are in no store: loading them raises BlockNotFoundError
    init = {i: torch.full(shape, float(i)) for i in range(num_logical) if i % 17 != 5}
    cpu_ops = OracleOps()
    ref = adapter_mod.KVCacheAdapter(
        num_actual, num_logical, torch.zeros((num_actual, *shape)),
        adapter_mod.InMemoryBlockStoreBackend(dict(init), num_logical_blocks=num_logical, ops=cpu_ops),
        native_ext=cpu_ops)
    gpu = adapter_mod.KVCacheAdapter(
        num_actual, num_logical, torch.zeros((num_actual, *shape), device=DEV),
        adapter_mod.InMemoryBlockStoreBackend({k: v.to(DEV) for k, v in init.items()},
                                              num_logical_blocks=num_logical, record_device_ops=path == "planned"))
    assert gpu._planned and not ref._planned
    assert (gpu._device_store() is not None) == (path == "device_store")
    pinned: list[int] = []
    for step in range(60):
        op = rng.choice(["load", "save", "release"], p=[0.45, 0.3, 0.25])
        k = int(rng.integers(1, max_batch + 1))
        if op == "release" and pinned:
            ids = np.asarray(pinned[:k], np.int64)
            pinned = pinned[k:]
        else:
            ids = rng.integers(0, num_logical, k).astype(np.int64)
        outs = []
        for ad, dev in ((ref, torch.device("cpu")), (gpu, DEV)):
            t = torch.from_numpy(ids).to(dev)
            try:
                if op == "load":
                    outs.append(("ok", ad.load(t).tolist()))
                elif op == "save":
                    data = torch.arange(k * shape[0] * shape[1], dtype=torch.float32).reshape(k, *shape) + 1000 * step
                    ad.save(t, data.to(dev))
                    outs.append(("ok", None))
                else:
                    ad.release(t)
                    outs.append(("ok", None))
            except Exception as exc:  # compared by type
                outs.append((type(exc).__name__, None))
        assert outs[0] == outs[1], (step, op)
        if op == "load" and outs[0][0] == "ok":
            pinned.extend(ids.tolist())
        for name in ("_logical_to_physical", "_physical_to_logical", "_slot_meta", "_search_start"):
            assert torch.equal(getattr(gpu, name).cpu(), getattr(ref, name)), (step, op, name)
        assert torch.equal(gpu.actual_blocks.cpu(), ref.actual_blocks), (step, op)
        assert torch.equal(gpu.backend._storage.cpu(), ref.backend._storage), (step, op)
        assert torch.equal(gpu.backend._present_mask.cpu(), ref.backend._present_mask), (step, op)
    if path == "device_store":
        assert int(gpu.backend._device_scratch.count_nonzero()) == 0
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda

    kv_cache_adapter_cuda.check_status(DEV)


def test_device_store_path_runs_one_sequence(api_gpu, monkeypatch):
    """With a store on the GPU, load and save call the device-store entry
    points and nothing else of the op set but release."""
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda as ext

    backend = api_gpu.InMemoryBlockStoreBackend(
        {i: torch.full((2, 4), float(i), device=DEV) for i in range(16)}, num_logical_blocks=16)
    ad = api_gpu.KVCacheAdapter(4, 16, torch.zeros((4, 2, 4), device=DEV), backend)
    called = []
    for name in ("plan_load", "plan_save", "gather_blocks", "scatter_blocks", "copy_blocks",
                 "commit_load_metadata", "commit_save_metadata", "pop_reusable_slots"):
        monkeypatch.setattr(ext, name, lambda *a, _n=name, **k: called.append(_n))
    assert ad.load(torch.tensor([3, 5], device=DEV)).tolist() == [0, 1]
    ad.release(torch.tensor([3, 5], device=DEV))
    ad.save(torch.tensor([7, 3], device=DEV), torch.ones((2, 2, 4), device=DEV))
    assert ad.load(torch.tensor([1, 2, 9, 3], device=DEV)).tolist() == [3, 1, 2, 0]
    assert called == []
    assert torch.equal(ad.actual_blocks[0], torch.ones((2, 4), device=DEV))
    assert torch.equal(backend._storage[5], torch.full((2, 4), 5.0, device=DEV))
    assert backend.max_concurrent_saves == 1 and backend.max_concurrent_loads == 1
    ext.check_status(DEV)


@pytest.fixture(scope="module")
def api_gpu():
    import kv_cache_adapter_b200 as m

    return m


@pytest.mark.parametrize("host_tier", [False, True])
def test_load_that_spills_and_fills_one_id(host_tier):
    """A stale reverse entry (two slots saved for one id) makes a later load
    evict id 1 from one victim while loading id 1 into another: the store
    must take the spilled payload before the fill reads it (the reference's
    save_blocks precedes load_blocks)."""
    prog = [("save", [1, 1]), ("load", [2]), ("release", [2]), ("load", [3]), ("release", [3]),
            ("load", [0, 1])]
    nl, na = 8, 3
    init = {i: torch.full((2,), float(i)) for i in range(nl)}
    cpu_ops = OracleOps()
    ref = adapter_mod.KVCacheAdapter(
        na, nl, torch.zeros((na, 2)),
        adapter_mod.InMemoryBlockStoreBackend(dict(init), num_logical_blocks=nl, ops=cpu_ops), native_ext=cpu_ops)
    backend = adapter_mod.InMemoryBlockStoreBackend({k: v.to(DEV) for k, v in init.items()}, num_logical_blocks=nl,
                                                    host_tier=host_tier, device=DEV)
    gpu = adapter_mod.KVCacheAdapter(na, nl, torch.zeros((na, 2), device=DEV), backend)
    assert gpu._device_store() is not None
    for step, (op, ids) in enumerate(prog):
        for ad, dev in ((ref, torch.device("cpu")), (gpu, DEV)):
            t = torch.tensor(ids, device=dev)
            if op == "load":
                ad.load(t)
            elif op == "save":
                ad.save(t, (torch.arange(2 * len(ids), dtype=torch.float32).reshape(-1, 2) + 100 * step).to(dev))
            else:
                ad.release(t)
        assert torch.equal(gpu.actual_blocks.cpu(), ref.actual_blocks), step
        assert torch.equal(backend._storage.cpu(), ref.backend._storage), step
        assert gpu._logical_to_physical.tolist() == ref._logical_to_physical.tolist(), step
    # the last load filled id 1 with the payload it spilled in the same call
    assert torch.equal(ref.backend._storage[1], torch.tensor([2.0, 3.0]))
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda

    kv_cache_adapter_cuda.check_status(DEV)


def test_plan_save_repeats_across_tiles(ops):
    """Every id resident and named many times across several 1,024-id tiles:
    only the last occurrence of each keeps its slot for the data scatter, and
    the blocked bitmap is left clear."""
    n = 4096
    l2p = torch.randperm(n, generator=torch.Generator().manual_seed(8))
    p2l = torch.empty_like(l2p)
    p2l[l2p] = torch.arange(n)
    meta = torch.zeros(n, dtype=torch.uint8)
    ids = torch.from_numpy(np.random.default_rng(9).choice(30, 5000).astype(np.int64))
    ss = torch.zeros(1, dtype=torch.int64, device=DEV)
    plan = ops.plan_save(l2p.to(DEV), p2l.to(DEV), meta.to(DEV), ss, ids.to(DEV))
    sel = l2p[ids].tolist()
    want = [s if s not in sel[i + 1:] else -1 for i, s in enumerate(sel)]
    assert plan.move_slots.tolist() == want
    assert plan.selected.tolist() == sel
    assert int(ops._bitmap(DEV, n).count_nonzero()) == 0
    ops.check_status(DEV)
