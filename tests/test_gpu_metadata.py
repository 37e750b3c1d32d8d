"""GPU parity: slot-metadata kernels and the clock sweep against the oracle and
the reference's recorded known answers (bit-exact)."""
from __future__ import annotations

import json
import random

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


@pytest.fixture(scope="module")
def ops():
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda as m

    return m


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy()


def _same(a: torch.Tensor, b: torch.Tensor) -> bool:
    a, b = _np(a), _np(b)
    return a.shape == b.shape and a.dtype == b.dtype and bool(np.array_equal(a, b))


def _ids(v, device=DEV):
    return torch.tensor(v, dtype=torch.int64, device=device)


def _meta(v, dtype=torch.uint8, device=DEV):
    return torch.tensor(np.asarray(v, dtype=np.uint8 if dtype == torch.uint8 else np.uint16), device=device)


def pack(pins, usage, bits: int) -> np.ndarray:
    f = bits // 2
    mask = (1 << f) - 1
    w = (np.asarray(pins, dtype=np.int64) & mask) | ((np.asarray(usage, dtype=np.int64) & mask) << f)
    return w.astype(np.uint8 if bits == 8 else np.uint16)


def _gold(golden_dir, name):
    return json.loads((golden_dir / name).read_text())


# known answers recorded with 8-bit slot meta and with the reference's 16-bit mode
KAT_FIXTURES = [("kat_metadata.json", torch.uint8), ("kat_metadata_u16.json", torch.uint16)]


# ---------------------------------------------------------------------------
# the reference's known answers (test_adapter_npu_kernels.py:42-194)
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("fixture,dtype", KAT_FIXTURES)
def test_kat_inspect_save(ops, golden_dir, fixture, dtype):
    c = _gold(golden_dir, fixture)["inspect_save"]
    cur, existing, usage = ops.inspect_save_requests(_ids(c["l2p"]), _meta(c["slot_meta"], dtype), _ids(c["ids"]))
    assert cur.tolist() == c["expect"]["cur"]
    assert existing.dtype == torch.bool and existing.int().tolist() == c["expect"]["existing"]
    assert usage.dtype == dtype and usage.tolist() == c["expect"]["usage"]


@pytest.mark.parametrize("fixture,dtype", KAT_FIXTURES)
def test_kat_inspect_load(ops, golden_dir, fixture, dtype):
    c = _gold(golden_dir, fixture)["inspect_load"]
    cur, resident, pins, usage = ops.inspect_load_requests(_ids(c["l2p"]), _meta(c["slot_meta"], dtype), _ids(c["ids"]))
    assert cur.tolist() == c["expect"]["cur"]
    assert resident.int().tolist() == c["expect"]["resident"]
    assert pins.dtype == torch.int64 and pins.tolist() == c["expect"]["pins"]
    assert usage.tolist() == c["expect"]["usage"]


@pytest.mark.parametrize("fixture,dtype", KAT_FIXTURES)
def test_kat_pop(ops, golden_dir, fixture, dtype):
    c = _gold(golden_dir, fixture)["pop"]
    meta, ss = _meta(c["slot_meta"], dtype), _ids([c["search_start"]])
    sel = ops.pop_reusable_slots(meta, ss, _ids(c["blocked"]), c["count"])
    assert sel.tolist() == c["expect"]["selected"] == [3, 0]
    assert ss.tolist() == [c["expect"]["search_start"]]
    assert meta.tolist() == c["expect"]["slot_meta"]


@pytest.mark.parametrize("fixture,dtype", KAT_FIXTURES)
def test_kat_pop_prefix_order(ops, golden_dir, fixture, dtype):
    c = _gold(golden_dir, fixture)["pop"]
    meta, ss = _meta(c["slot_meta"], dtype), _ids([c["search_start"]])
    sel = ops.pop_reusable_slots(meta, ss, _ids(c["blocked"]), c["count"], order="prefix")
    assert sel.tolist() == [0, 3] and ss.tolist() == [0]


@pytest.mark.parametrize("fixture,dtype", KAT_FIXTURES)
def test_kat_commit_save(ops, golden_dir, fixture, dtype):
    c = _gold(golden_dir, fixture)["commit_save"]
    l2p, p2l, meta = _ids(c["l2p"]), _ids(c["p2l"]), _meta(c["slot_meta"], dtype)
    ops.commit_save_metadata(l2p, p2l, meta, _ids(c["evicted"]), _ids(c["ids"]), _ids(c["slots"]),
                             _meta(c["final_pins"], dtype), _meta(c["final_usage"], dtype))
    assert l2p.tolist() == c["expect"]["l2p"] and p2l.tolist() == c["expect"]["p2l"]
    assert meta.tolist() == c["expect"]["slot_meta"]


@pytest.mark.parametrize("fixture,dtype", KAT_FIXTURES)
def test_kat_commit_load(ops, golden_dir, fixture, dtype):
    c = _gold(golden_dir, fixture)["commit_load"]
    l2p, p2l, meta = _ids(c["l2p"]), _ids(c["p2l"]), _meta(c["slot_meta"], dtype)
    ops.commit_load_metadata(l2p, p2l, meta, _ids(c["evicted"]), _ids(c["miss_ids"]), _ids(c["miss_slots"]),
                             _ids(c["hit_slots"]), _ids(c["hit_pins"]), _meta(c["hit_usage"], dtype),
                             _meta(c["miss_usage"], dtype))
    assert l2p.tolist() == c["expect"]["l2p"] and p2l.tolist() == c["expect"]["p2l"]
    assert meta.tolist() == c["expect"]["slot_meta"]


@pytest.mark.parametrize("fixture,dtype", KAT_FIXTURES)
def test_kat_release(ops, golden_dir, fixture, dtype):
    c = _gold(golden_dir, fixture)["release"]
    meta = _meta(c["slot_meta"], dtype)
    ops.release_metadata(_ids(c["l2p"]), meta, _ids(c["ids"]))
    assert meta.tolist() == c["expect"]["slot_meta"]


# ---------------------------------------------------------------------------
# clock sweep
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("fixture,dtype", [("pop_u8.json", torch.uint8), ("pop_u16.json", torch.uint16)])
def test_pop_reference_cases(ops, golden_dir, fixture, dtype):
    """Cases recorded from the reference's strict path (400 with 8-bit slot
    meta, 200 in its 16-bit mode), bit-exact."""
    from kv_cache_adapter_b200.errors import InsufficientCapacityError

    for i, c in enumerate(_gold(golden_dir, fixture)):
        meta, ss = _meta(c["slot_meta"], dtype), _ids([c["search_start"]])
        try:
            sel, err = ops.pop_reusable_slots(meta, ss, _ids(c["blocked"]), c["count"]).tolist(), None
        except InsufficientCapacityError:
            sel, err = None, "InsufficientCapacityError"
        assert (err, sel) == (c["error"], c["selected"]), i
        assert meta.tolist() == c["after_slot_meta"], i
        assert int(ss[0]) == c["after_search_start"], i


def _random_table(rng: np.random.Generator, n: int, bits: int, kind: str):
    umax = (1 << (bits // 2)) - 1
    if kind == "uniform":
        usage = rng.integers(0, umax + 1, n)
    elif kind == "warm":
        usage = rng.integers(0, 4, n)
    elif kind == "nozero":
        usage = rng.integers(1, umax + 1, n)
    else:  # "sparse": few zeros, T = 0 needs a long scan
        usage = np.where(rng.random(n) < 0.0005, 0, rng.integers(1, 4, n))
    pins = np.where(rng.random(n) < 0.05, rng.integers(1, umax + 1, n), 0)
    return pack(pins, usage, bits)


@pytest.mark.parametrize("bits", [8, 16])
@pytest.mark.parametrize("order", ["grouped", "prefix"])
@pytest.mark.parametrize("n", [1, 15, 16, 17, 1000, 16384, 16385, 100003, 1 << 20])
def test_pop_sequences_match_oracle(ops, bits, order, n):
    """Consecutive pops on one table (search_start and aging carry over),
    every table kind, blocked lists, counts up to thousands."""
    from kv_cache_adapter_b200.errors import InsufficientCapacityError

    rng = np.random.default_rng(n * 7 + bits + (order == "prefix"))
    dtype = torch.uint8 if bits == 8 else torch.uint16
    for kind in ("uniform", "warm", "nozero", "sparse"):
        host = torch.from_numpy(_random_table(rng, n, bits, kind))
        dev = host.to(DEV)
        ss_h = torch.tensor([int(rng.integers(0, n))], dtype=torch.int64)
        ss_d = ss_h.to(DEV)
        for call in range(6):
            count = int(rng.choice([1, 2, 7, 256, 1000, 5000]))
            count = min(count, max(1, n))
            nb = int(rng.choice([0, 0, 1, 5, 64]))
            blocked = torch.from_numpy(rng.integers(0, n, nb).astype(np.int64))
            try:
                want = oracle.pop_reusable_slots(host, ss_h, blocked, count, order=order)
                want_err = None
            except oracle.OracleInsufficientCapacity:
                want, want_err = None, InsufficientCapacityError
            if want_err is None:
                got = ops.pop_reusable_slots(dev, ss_d, blocked.to(DEV), count, order=order)
                assert _same(got, want), (kind, call, count)
            else:
                with pytest.raises(want_err):
                    ops.pop_reusable_slots(dev, ss_d, blocked.to(DEV), count, order=order)
            assert _same(dev, host), (kind, call)
            assert int(ss_d[0]) == int(ss_h[0]), (kind, call)


def test_pop_errors_leave_state_untouched(ops):
    from kv_cache_adapter_b200.errors import InsufficientCapacityError

    meta = _meta(pack([1, 0, 1, 0], [0, 5, 0, 9], 8))
    ss = _ids([2])
    before = meta.clone()
    with pytest.raises(IndexError):
        ops.pop_reusable_slots(meta, ss, _ids([4]), 1)
    with pytest.raises(IndexError):
        ops.pop_reusable_slots(meta, ss, _ids([-1]), 1)
    with pytest.raises(InsufficientCapacityError):
        ops.pop_reusable_slots(meta, ss, _ids([1]), 2)
    assert _same(meta, before) and ss.tolist() == [2]
    # the blocked bitmap was cleared: slot 1 is available again
    assert ops.pop_reusable_slots(meta, ss, _ids([]), 2).tolist() == [1, 3]
    assert ops.pop_reusable_slots(meta, ss, _ids([]), 0).numel() == 0


def test_choose_pop_launch_warps(ops):
    assert ops.choose_pop_launch_warps(4) == 1
    assert ops.choose_pop_launch_warps(1 << 20) == 32
    with pytest.raises(ValueError):
        ops.choose_pop_launch_warps(0)


# ---------------------------------------------------------------------------
# inspect / commit / release against the oracle on random tables
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("bits", [8, 16])
def test_metadata_ops_match_oracle(ops, bits):
    rng = np.random.default_rng(99 + bits)
    dtype = torch.uint8 if bits == 8 else torch.uint16
    umax = (1 << (bits // 2)) - 1
    for trial in range(8):
        n_logical = int(rng.integers(8, 50000))
        n_slots = int(rng.integers(4, min(n_logical, 20000) + 1))
        resident = rng.permutation(n_logical)[: int(rng.integers(0, n_slots + 1))]
        slots = rng.permutation(n_slots)[: resident.size]
        l2p = np.full(n_logical, -1, np.int64)
        l2p[resident] = slots
        p2l = np.full(n_slots, -1, np.int64)
        p2l[slots] = resident
        meta = pack(rng.integers(0, umax + 1, n_slots), rng.integers(0, umax + 1, n_slots), bits)
        k = int(rng.integers(1, min(n_logical, 3000) + 1))
        ids = rng.permutation(n_logical)[:k].astype(np.int64)

        L, M, I = (torch.from_numpy(x) for x in (l2p, meta, ids))
        for fn in ("inspect_load_requests", "inspect_save_requests"):
            want = getattr(oracle, fn)(L, M, I)
            got = getattr(ops, fn)(L.to(DEV), M.to(DEV), I.to(DEV))
            for w, g in zip(want, got):
                assert _same(g, w), (trial, fn)

        # release: only resident ids
        rel = torch.from_numpy(resident[: int(rng.integers(0, resident.size + 1))].astype(np.int64))
        Mh = M.clone()
        oracle.release_metadata(L, Mh, rel)
        Md = M.to(DEV)
        ops.release_metadata(L.to(DEV), Md, rel.to(DEV))
        assert _same(Md, Mh), trial

        # commit_save: evict residents of the chosen slots, map new ids there
        cnt = int(rng.integers(0, min(n_slots, 2000) + 1))
        tslots = rng.permutation(n_slots)[:cnt].astype(np.int64)
        free_ids = np.setdiff1d(np.arange(n_logical), resident)
        new_ids = rng.permutation(free_ids)[: min(cnt, free_ids.size)].astype(np.int64)
        tslots = tslots[: new_ids.size]
        evicted = p2l[tslots][p2l[tslots] >= 0].astype(np.int64)
        fp = pack(0, 0, bits)  # dtype carrier
        final_pins = rng.integers(0, umax + 1, new_ids.size).astype(fp.dtype)
        final_usage = rng.integers(0, umax + 1, new_ids.size).astype(fp.dtype)
        args = [torch.from_numpy(x) for x in (evicted, new_ids, tslots, final_pins, final_usage)]
        Lh, Ph, Mh = L.clone(), torch.from_numpy(p2l.copy()), M.clone()
        oracle.commit_save_metadata(Lh, Ph, Mh, *args)
        Ld, Pd, Md = L.to(DEV), torch.from_numpy(p2l.copy()).to(DEV), M.to(DEV)
        ops.commit_save_metadata(Ld, Pd, Md, *[a.to(DEV) for a in args])
        assert _same(Ld, Lh) and _same(Pd, Ph) and _same(Md, Mh), trial

        # commit_load: hits on some residents, misses mapped to other slots
        hits = rng.permutation(slots)[: int(rng.integers(0, slots.size + 1))].astype(np.int64)
        hit_pins = rng.integers(0, 2 * umax, hits.size).astype(np.int64)
        hit_usage = rng.integers(0, umax + 1, hits.size).astype(fp.dtype)
        others = np.setdiff1d(np.arange(n_slots), hits)
        mslots = rng.permutation(others)[: min(others.size, 1500)].astype(np.int64)
        mids = rng.permutation(free_ids)[: min(mslots.size, free_ids.size)].astype(np.int64)
        mslots = mslots[: mids.size]
        mev = p2l[mslots][p2l[mslots] >= 0].astype(np.int64)
        musage = rng.integers(0, umax + 1, mids.size).astype(fp.dtype)
        args = [torch.from_numpy(x) for x in (mev, mids, mslots, hits, hit_pins, hit_usage, musage)]
        Lh, Ph, Mh = L.clone(), torch.from_numpy(p2l.copy()), M.clone()
        oracle.commit_load_metadata(Lh, Ph, Mh, *args)
        Ld, Pd, Md = L.to(DEV), torch.from_numpy(p2l.copy()).to(DEV), M.to(DEV)
        ops.commit_load_metadata(Ld, Pd, Md, *[a.to(DEV) for a in args])
        assert _same(Ld, Lh) and _same(Pd, Ph) and _same(Md, Mh), trial


def test_metadata_bad_ids_raise_and_change_nothing(ops):
    l2p = _ids([0, 1, -1, 2])
    p2l = _ids([0, 1, 3])
    meta = _meta(pack([1, 2, 1], [3, 4, 5], 8))
    snap = (l2p.clone(), p2l.clone(), meta.clone())
    with pytest.raises(IndexError):
        ops.inspect_load_requests(l2p, meta, _ids([0, 4]))
    with pytest.raises(IndexError):
        ops.inspect_save_requests(l2p, meta, _ids([-3]))
    with pytest.raises(IndexError):  # logical 2 is not resident
        ops.release_metadata(l2p, meta, _ids([0, 2]))
    with pytest.raises(IndexError):
        ops.commit_save_metadata(l2p, p2l, meta, _ids([]), _ids([2]), _ids([7]), _meta([0]), _meta([1]))
    with pytest.raises(IndexError):
        ops.commit_load_metadata(l2p, p2l, meta, _ids([9]), _ids([2]), _ids([1]), _ids([]), _ids([]),
                                 _meta([]), _meta([1]))
    assert _same(l2p, snap[0]) and _same(p2l, snap[1]) and _same(meta, snap[2])


def test_release_wraps_pin_and_counts_duplicates_once(ops):
    """A pin of 0 wraps to the field max (adapter.py:332-336); an id listed
    twice in one call releases one pin, as the strict path's single
    index_put_ does."""
    l2p = _ids([0, 1])
    meta = _meta(pack([0, 3], [7, 2], 8))
    ops.release_metadata(l2p, meta, _ids([0, 1, 1]))
    assert meta.tolist() == pack([15, 2], [7, 2], 8).tolist()


def test_unchecked_errors_latch_until_checked(ops):
    l2p = _ids([0, -1])
    meta = _meta([1, 1])
    ops.release_metadata(l2p, meta, _ids([1]), check=False)
    torch.cuda.synchronize()
    with pytest.raises(IndexError):
        ops.check_status(DEV)
    ops.check_status(DEV)  # cleared
