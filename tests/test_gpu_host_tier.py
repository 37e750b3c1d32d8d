"""GPU parity: moves between device blocks and pinned host memory (one kernel
over the host link instead of one cudaMemcpyAsync per block, the reference
LMCacheBackend's CUDA path, adapter.py:960-966 and :1035-1037), and the host
tier behind KVCacheAdapter against the recorded reference scenarios and the
oracle-driven adapter."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import scenario_runner
from oracle_ops import OracleOps
from kv_cache_adapter_b200 import adapter as adapter_mod
from kv_cache_adapter_b200.errors import BlockNotFoundError

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


@pytest.fixture(scope="module")
def ext():
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda as m

    return m


def _cache(n, row_shape, dtype, seed, device=DEV):
    g = torch.Generator().manual_seed(seed)
    if dtype.is_floating_point:
        t = torch.randn((n, *row_shape), generator=g).to(dtype)
    else:
        t = torch.randint(0, 255, (n, *row_shape), generator=g).to(dtype)
    return t.to(device)


def test_host_memory_check(ext):
    pinned = torch.zeros(1000, pin_memory=True)
    assert ext.host_memory_usable(pinned)
    assert ext.host_memory_usable(pinned[10:20])
    assert not ext.host_memory_usable(torch.zeros(1000))
    assert not ext.host_memory_usable(torch.zeros(1000, device=DEV))


def test_pageable_host_sides_are_refused_before_any_launch(ext):
    actual = torch.zeros((8, 64), device=DEV)
    ids = torch.arange(4, device=DEV)
    with pytest.raises(ValueError, match="pinned"):
        ext.gather_blocks(actual, ids, out=torch.empty((4, 64)))
    with pytest.raises(ValueError, match="pinned"):
        ext.scatter_blocks(actual, ids, torch.ones((4, 64)))
    with pytest.raises(ValueError, match="pinned host memory"):
        ext.copy_blocks(torch.zeros((8, 64)), ids, actual, ids)
    with pytest.raises(ValueError):
        ext.gather_layers([torch.zeros((8, 64), pin_memory=True)], ids)
    ext.check_status(DEV)


@pytest.mark.parametrize("row_shape,dtype", [
    ((2,), torch.float32),            # 8 B rows
    ((3,), torch.float16),            # 6 B rows: 2-byte accesses
    ((16, 8, 16), torch.bfloat16),    # 4 KiB rows
    ((2, 16, 8, 128), torch.float16), # 64 KiB merged K/V blocks (Llama-3-8B, bs 16)
    ((64, 576), torch.bfloat16),      # 72 KiB MLA latent blocks
    ((5, 7), torch.uint8),            # odd bytes
])
def test_block_moves_to_and_from_pinned_host(ext, row_shape, dtype):
    n, k = 300, 97
    actual = _cache(n, row_shape, dtype, 1)
    gen = torch.Generator().manual_seed(2)
    slots = torch.randperm(n, generator=gen)[:k].to(DEV)
    # D2H gather straight into pinned rows
    out = torch.empty((k, *row_shape), dtype=dtype, pin_memory=True)
    ext.gather_blocks(actual, slots, out=out)
    torch.cuda.synchronize()
    assert torch.equal(out, actual.index_select(0, slots).cpu())
    # H2D scatter from pinned rows, with padding slots skipped
    src = _cache(k, row_shape, dtype, 3, device="cpu").pin_memory()
    pad = slots.clone()
    pad[::5] = -1
    want = actual.clone()
    keep = pad >= 0
    want.index_copy_(0, pad[keep], src.to(DEV)[keep])
    ext.scatter_blocks(actual, pad, src, skip_negative=True)
    torch.cuda.synchronize()
    assert torch.equal(actual, want)
    # host arena <-> device blocks, random rows on both sides
    arena = _cache(2 * n, row_shape, dtype, 4, device="cpu").pin_memory()
    rows = torch.randperm(2 * n, generator=gen)[:k].to(DEV)
    want = actual.clone()
    want.index_copy_(0, slots, arena.index_select(0, rows.cpu()).to(DEV))
    ext.copy_blocks(arena, rows, actual, slots)
    torch.cuda.synchronize()
    assert torch.equal(actual, want)
    want_arena = arena.clone()
    want_arena.index_copy_(0, rows.cpu(), actual.index_select(0, slots).cpu())
    ext.copy_blocks(actual, slots, arena, rows)
    torch.cuda.synchronize()
    assert torch.equal(arena, want_arena)
    ext.check_status(DEV)


def test_layer_and_token_chunks_in_pinned_host(ext):
    """KV_2LTD chunks ([K/V][layer][rows]) written straight to pinned memory and
    read back from it."""
    L, nb, bs = 4, 64, 16
    planes = [_cache(nb, (bs, 2, 64), torch.bfloat16, 10 + p) for p in range(2 * L)]
    table = ext.PlaneTable(planes, 1)
    slots = torch.randperm(nb, generator=torch.Generator().manual_seed(5))[:32].to(DEV)
    host = torch.empty((4, 2 * L, 8, bs, 2, 64), dtype=torch.bfloat16, pin_memory=True)
    ext.gather_layers(table, slots, out=host, blocks_per_chunk=8)
    torch.cuda.synchronize()
    want = torch.stack([p.index_select(0, slots) for p in planes], 0).reshape(2 * L, 4, 8, bs, 2, 64)
    assert torch.equal(host, want.transpose(0, 1).cpu())
    for p in planes:
        p.zero_()
    ext.scatter_layers(table, slots, host, blocks_per_chunk=8)
    torch.cuda.synchronize()
    for i, p in enumerate(planes):
        assert torch.equal(p.index_select(0, slots).cpu(), want[i].reshape(32, bs, 2, 64).cpu())
    tok = ext.PlaneTable([p.view(nb, bs, 128) for p in planes], 2)
    mapping = torch.randperm(nb * bs, generator=torch.Generator().manual_seed(6))[:256].to(DEV)
    mapping[7] = -1
    hchunks = torch.zeros((1, 2 * L, 256, 128), dtype=torch.bfloat16, pin_memory=True)
    ext.gather_tokens(tok, mapping, out=hchunks)
    torch.cuda.synchronize()
    for i, p in enumerate(planes):
        flat = p.view(nb * bs, 128)
        sel = mapping.clone()
        sel[7] = 0
        got = hchunks[0, i].clone()
        want_rows = flat.index_select(0, sel).cpu()
        got[7] = want_rows[7]
        assert torch.equal(got, want_rows)
    ext.check_status(DEV)


@pytest.mark.parametrize("path", ["device_store", "planned", "stepwise"])
@pytest.mark.parametrize("case_index", range(0, 60, 3))
def test_recorded_scenarios_with_host_tier(ext, case_index, path):
    case = scenario_runner.load_scenarios()[case_index]
    scenario_runner.run_and_compare(case, DEV, planned=path != "stepwise", record=path != "device_store",
                                    host_tier=True)
    ext.check_status(DEV)


def test_host_tier_backend_api():
    b = adapter_mod.HostTierBackend(block_shape=(16, 2, 8, 128), block_dtype=torch.float16, num_logical_blocks=64,
                                    device=DEV)
    assert b.memory_format == "KV_2TD" and b._storage.is_pinned()
    assert adapter_mod.HostTierBackend(block_shape=(2, 16, 8, 128), block_dtype=torch.float16,
                                       num_logical_blocks=4).memory_format == "KV_T2D"
    assert adapter_mod.HostTierBackend(block_shape=(7,), block_dtype=torch.float32,
                                       num_logical_blocks=4).memory_format == "UNDEFINED"
    with pytest.raises(ValueError):
        adapter_mod.HostTierBackend(block_shape=(1024,), block_dtype=torch.float32, num_logical_blocks=1 << 20,
                                    max_local_cpu_size_gb=1.0)
    data = torch.randn((3, 16, 2, 8, 128), device=DEV).half()
    ids = torch.tensor([5, 9, 5], device=DEV)
    with pytest.raises(TypeError):
        b.save_blocks(ids, data.float())
    with pytest.raises(ValueError):
        b.save_blocks(ids, data[:, :8])
    b.save_blocks(ids, data)
    snap = b.snapshot()
    assert sorted(snap) == [5, 9]
    assert torch.equal(snap[5], data[2].cpu()) and torch.equal(snap[9], data[1].cpu())
    assert torch.equal(b.transfer_view(9), data[1].cpu().reshape(16, 2, 1024))
    actual = torch.zeros((4, 16, 2, 8, 128), device=DEV).half()
    b.load_blocks(torch.tensor([9, 5], device=DEV), actual, torch.tensor([3, 0], device=DEV))
    assert torch.equal(actual[3], data[1]) and torch.equal(actual[0], data[2])
    with pytest.raises(BlockNotFoundError):
        b.load_blocks(torch.tensor([6], device=DEV), actual, torch.tensor([1], device=DEV))
    b.shutdown()


@pytest.mark.parametrize("seed,num_actual,num_logical,max_batch,shape", [
    (11, 64, 256, 48, (2, 3)), (12, 1000, 4000, 700, (2, 3)),
    # 32 KiB blocks: most calls exceed the one-launch size limit of a pinned store
    (13, 64, 256, 48, (8, 1024)),
])
def test_adapter_with_host_tier_matches_oracle_adapter(seed, num_actual, num_logical, max_batch, shape):
    """Random programs as in the planner tests, the CUDA adapter spilling to
    and filling from the pinned host tier (device-store path)."""
    rng = np.random.default_rng(seed)
    init = {i: torch.full(shape, float(i)) for i in range(num_logical) if i % 13 != 4}
    cpu_ops = OracleOps()
    ref = adapter_mod.KVCacheAdapter(
        num_actual, num_logical, torch.zeros((num_actual, *shape)),
        adapter_mod.InMemoryBlockStoreBackend(dict(init), num_logical_blocks=num_logical, ops=cpu_ops),
        native_ext=cpu_ops)
    tier = adapter_mod.InMemoryBlockStoreBackend(dict(init), num_logical_blocks=num_logical, host_tier=True,
                                                 device=DEV)
    gpu = adapter_mod.KVCacheAdapter(num_actual, num_logical, torch.zeros((num_actual, *shape), device=DEV), tier)
    assert gpu._device_store() is not None and tier._storage.is_pinned()
    pinned: list[int] = []
    for step in range(50):
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
        assert torch.equal(tier._storage, ref.backend._storage), (step, op)
        assert torch.equal(tier._present_mask.cpu(), ref.backend._present_mask), (step, op)
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda

    kv_cache_adapter_cuda.check_status(DEV)


def _kv_token(actual: torch.Tensor, layout, s: int, kv: int) -> torch.Tensor:
    bs = layout.block_size
    flat = actual.view(actual.shape[0], *layout.transfer_shape)
    return flat[s // bs, s % bs, kv] if layout.token_major else flat[s // bs, kv, s % bs]


def _obj_token(obj: torch.Tensor, layout, t: int, kv: int) -> torch.Tensor:
    return obj[t, kv] if layout.token_major else obj[kv, t]


@pytest.mark.parametrize("token_major", [True, False])
@pytest.mark.parametrize("where", ["host", "device"])
def test_fused_single_layer_kv_transfer(ext, token_major, where):
    """The accelerator host path's fused transfer (adapter.py:1200-1243):
    block_data -> memory objects with the dense slot mapping, memory objects ->
    actual_blocks with the physical slot mapping, and an arbitrary token
    mapping with padding, K and V in one launch."""
    bs, H, D = 16, 8, 128
    block = (bs, 2, H, D) if token_major else (2, bs, H, D)
    layout = adapter_mod._MergedKVBlockLayout.detect(block)
    k, m = 24, 64
    g = torch.Generator().manual_seed(31)
    mk = (lambda shape: torch.zeros(shape, dtype=torch.float16, pin_memory=True)) if where == "host" else \
        (lambda shape: torch.zeros(shape, dtype=torch.float16, device=DEV))
    pool = mk((40, *layout.transfer_shape))
    rows = torch.randperm(40, generator=g)[:k].tolist()
    objs = [pool[r] for r in rows]
    block_data = _cache(k, block, torch.float16, 21)
    ext.batched_fused_single_layer_kv_transfer(objs, None, block_data, layout.dense_slot_mapping(k, device=DEV),
                                               layout.chunk_offsets(k), layout.chunk_sizes(k), True, 1,
                                               token_major, False)
    torch.cuda.synchronize()
    flat = layout.flatten_block_batch(block_data)
    for i, r in enumerate(rows):
        assert torch.equal(pool[r].to(DEV), flat[i]), i
    actual = torch.zeros((m, *block), dtype=torch.float16, device=DEV)
    slots = torch.randperm(m, generator=g)[:k].to(DEV)
    ext.batched_fused_single_layer_kv_transfer(objs, None, actual, layout.physical_slot_mapping(slots),
                                               layout.chunk_offsets(k), layout.chunk_sizes(k), False, 1,
                                               token_major, False)
    torch.cuda.synchronize()
    for i, s_ in enumerate(slots.tolist()):
        assert torch.equal(actual[s_], layout.restore_block_tensor(objs[i].to(DEV))), i
    # arbitrary token mapping: 6 chunks of 8 tokens, offsets out of order, padding slots
    T, n = 8, 6
    mapping = torch.randperm(m * bs, generator=g)[: n * T].to(DEV)
    mapping[5] = -1
    offsets = [T * j for j in (3, 0, 5, 1, 4, 2)]
    tshape = (T, 2, layout.hidden_dim) if token_major else (2, T, layout.hidden_dim)
    pool2 = mk((n, *tshape))
    objs2 = list(pool2.unbind(0))
    ext.batched_fused_single_layer_kv_transfer(objs2, None, actual, mapping, offsets, [T] * n, True, 1, token_major)
    torch.cuda.synchronize()
    mp = mapping.tolist()
    for i, off in enumerate(offsets):
        for t in range(T):
            sl = mp[off + t]
            for kv in (0, 1):
                got = _obj_token(objs2[i], layout, t, kv).to(DEV)
                want = torch.zeros_like(got) if sl < 0 else _kv_token(actual, layout, sl, kv)
                assert torch.equal(got, want), (i, t, kv)
    fresh = torch.zeros_like(actual)
    ext.batched_fused_single_layer_kv_transfer(objs2, None, fresh, mapping, offsets, [T] * n, False, 1, token_major)
    torch.cuda.synchronize()
    for i, off in enumerate(offsets):
        for t in range(T):
            sl = mp[off + t]
            if sl >= 0:
                for kv in (0, 1):
                    assert torch.equal(_kv_token(fresh, layout, sl, kv), _obj_token(objs2[i], layout, t, kv).to(DEV))
    with pytest.raises(ValueError):  # objects that are not rows of one buffer
        ext.batched_fused_single_layer_kv_transfer([mk(tshape), mk(tshape)], None, actual, mapping[: 2 * T],
                                                   [0, T], [T, T], True, 1, token_major)
    with pytest.raises(ValueError):  # wrong token order for the block layout
        ext.batched_fused_single_layer_kv_transfer(objs2, None, actual, mapping, offsets, [T] * n, True, 1,
                                                   not token_major)
    ext.check_status(DEV)


@pytest.mark.parametrize("where", ["host", "device"])
@pytest.mark.parametrize("row_shape,dtype", [((2, 16, 8, 128), torch.float16), ((3,), torch.float16),
                                             ((40,), torch.float32)])
def test_exchange_blocks(ext, where, row_shape, dtype):
    """Spill the old bytes of each slot to one store row and fill it from
    another, in one launch; padding entries skip their part."""
    n, nl, k = 200, 600, 77
    g = torch.Generator().manual_seed(41)
    actual = _cache(n, row_shape, dtype, 42)
    store = _cache(nl, row_shape, dtype, 43, device="cpu")
    store = store.pin_memory() if where == "host" else store.to(DEV)
    slots = torch.randperm(n, generator=g)[:k]
    rows = torch.randperm(nl, generator=g)
    spill, fill = rows[:k].clone(), rows[k:2 * k].clone()
    spill[::7] = -1
    fill[3::9] = -1
    slots[10] = -1
    want_actual, want_store = actual.cpu().clone(), store.cpu().clone()
    for j in range(k):
        s_ = int(slots[j])
        if s_ < 0:
            continue
        if spill[j] >= 0:
            want_store[spill[j]] = want_actual[s_]
        if fill[j] >= 0:
            want_actual[s_] = store.cpu()[fill[j]]
    ext.exchange_blocks(actual, slots.to(DEV), store, spill.to(DEV), fill.to(DEV))
    torch.cuda.synchronize()
    assert torch.equal(actual.cpu(), want_actual)
    assert torch.equal(store.cpu(), want_store)
    ext.check_status(DEV)
