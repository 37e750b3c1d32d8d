"""CPU: the oracle (and the adapter's host orchestration driven by it) against
the reference's known answers and fixtures recorded from the reference."""
from __future__ import annotations

import json

import pytest
import torch

import oracle
from oracle import moves
from kv_cache_adapter_b200 import adapter as adapter_mod
from kv_cache_adapter_b200 import workloads
from kv_cache_adapter_b200.adapter import _MergedKVBlockLayout

import scenario_runner
from oracle_ops import OracleOps


def _load(golden_dir, name):
    return json.loads((golden_dir / name).read_text())


def _ids(v):
    return torch.tensor(v, dtype=torch.int64)


def _meta(v, dtype=torch.uint8):
    return torch.tensor(v, dtype=torch.int64).to(dtype)


# the reference's known answers and pop cases with 8-bit slot meta, and with
# 16-bit slot meta (KVCA_SLOT_META_BITS=16: 8-bit pin and usage fields)
KAT_FIXTURES = [("kat_metadata.json", torch.uint8), ("kat_metadata_u16.json", torch.uint16)]


# ---------------------------------------------------------------------------
# known-answer tests of the reference (test_adapter_npu_kernels.py:42-194)
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("fixture,dtype", KAT_FIXTURES)
def test_kat_inspect_save(golden_dir, fixture, dtype):
    c = _load(golden_dir, fixture)["inspect_save"]
    cur, existing, usage = oracle.inspect_save_requests(_ids(c["l2p"]), _meta(c["slot_meta"], dtype), _ids(c["ids"]))
    assert cur.tolist() == c["expect"]["cur"]
    assert existing.int().tolist() == c["expect"]["existing"]
    assert usage.tolist() == c["expect"]["usage"]


@pytest.mark.parametrize("fixture,dtype", KAT_FIXTURES)
def test_kat_inspect_load(golden_dir, fixture, dtype):
    c = _load(golden_dir, fixture)["inspect_load"]
    cur, resident, pins, usage = oracle.inspect_load_requests(_ids(c["l2p"]), _meta(c["slot_meta"], dtype), _ids(c["ids"]))
    assert cur.tolist() == c["expect"]["cur"]
    assert resident.int().tolist() == c["expect"]["resident"]
    assert pins.tolist() == c["expect"]["pins"]
    assert usage.tolist() == c["expect"]["usage"]


@pytest.mark.parametrize("fixture,dtype", KAT_FIXTURES)
def test_kat_pop_threshold_scan_and_age(golden_dir, fixture, dtype):
    c = _load(golden_dir, fixture)["pop"]
    meta, ss = _meta(c["slot_meta"], dtype), _ids([c["search_start"]])
    sel = oracle.pop_reusable_slots(meta, ss, _ids(c["blocked"]), c["count"])
    assert sel.tolist() == c["expect"]["selected"] == [3, 0]
    assert ss.tolist() == [c["expect"]["search_start"]]
    assert meta.tolist() == c["expect"]["slot_meta"]


@pytest.mark.parametrize("fixture,dtype", KAT_FIXTURES)
def test_kat_commit_save(golden_dir, fixture, dtype):
    c = _load(golden_dir, fixture)["commit_save"]
    l2p, p2l, meta = _ids(c["l2p"]), _ids(c["p2l"]), _meta(c["slot_meta"], dtype)
    oracle.commit_save_metadata(l2p, p2l, meta, _ids(c["evicted"]), _ids(c["ids"]), _ids(c["slots"]),
                                _meta(c["final_pins"], dtype), _meta(c["final_usage"], dtype))
    assert l2p.tolist() == c["expect"]["l2p"]
    assert p2l.tolist() == c["expect"]["p2l"]
    assert meta.tolist() == c["expect"]["slot_meta"]


@pytest.mark.parametrize("fixture,dtype", KAT_FIXTURES)
def test_kat_commit_load(golden_dir, fixture, dtype):
    c = _load(golden_dir, fixture)["commit_load"]
    l2p, p2l, meta = _ids(c["l2p"]), _ids(c["p2l"]), _meta(c["slot_meta"], dtype)
    oracle.commit_load_metadata(l2p, p2l, meta, _ids(c["evicted"]), _ids(c["miss_ids"]), _ids(c["miss_slots"]),
                                _ids(c["hit_slots"]), _ids(c["hit_pins"]), _meta(c["hit_usage"], dtype),
                                _meta(c["miss_usage"], dtype))
    assert l2p.tolist() == c["expect"]["l2p"]
    assert p2l.tolist() == c["expect"]["p2l"]
    assert meta.tolist() == c["expect"]["slot_meta"]


@pytest.mark.parametrize("fixture,dtype", KAT_FIXTURES)
def test_kat_release(golden_dir, fixture, dtype):
    c = _load(golden_dir, fixture)["release"]
    meta = _meta(c["slot_meta"], dtype)
    oracle.release_metadata(_ids(c["l2p"]), meta, _ids(c["ids"]))
    assert meta.tolist() == c["expect"]["slot_meta"]


# ---------------------------------------------------------------------------
# clock sweep: 400 seeded cases recorded from the reference's strict path
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("fixture,dtype,count", [("pop_u8.json", torch.uint8, 400),
                                                 ("pop_u16.json", torch.uint16, 200)])
def test_pop_cases_match_reference(golden_dir, fixture, dtype, count):
    cases = _load(golden_dir, fixture)
    assert len(cases) == count
    for i, c in enumerate(cases):
        meta = _meta(c["slot_meta"], dtype)
        ss = _ids([c["search_start"]])
        try:
            sel = oracle.pop_reusable_slots(meta, ss, _ids(c["blocked"]), c["count"]).tolist()
            err = None
        except oracle.OracleInsufficientCapacity:
            sel, err = None, "InsufficientCapacityError"
        assert err == c["error"], i
        assert sel == c["selected"], i
        assert meta.tolist() == c["after_slot_meta"], i
        assert int(ss[0]) == c["after_search_start"], i


def test_pop_cases_regenerate_identically(golden_dir):
    """The fixture inputs come from the shared generator: regenerating them
    gives the same cases the GPU tests use."""
    cases = _load(golden_dir, "pop_u8.json")
    regen = list(workloads.pop_case_params(len(cases), 1234, usage_max=15, pin_max=15))
    for c, r in zip(cases, regen):
        assert c["usage"] == r["usage"] and c["pins"] == r["pins"] and c["blocked"] == r["blocked"]
        assert c["count"] == r["count"] and c["search_start"] == r["search_start"]


def test_pop_u16_cases_regenerate_identically(golden_dir):
    cases = _load(golden_dir, "pop_u16.json")
    regen = list(workloads.pop_case_params(len(cases), 4321, usage_max=255, pin_max=255))
    for c, r in zip(cases, regen):
        assert c["usage"] == r["usage"] and c["pins"] == r["pins"] and c["blocked"] == r["blocked"]
        assert c["count"] == r["count"] and c["search_start"] == r["search_start"]
    assert max(max(c["usage"]) for c in cases) == 255  # past the 4-bit field


def test_pop_prefix_order_differs_on_known_answer():
    """The prefix rule of the reference CUDA kernel picks [0, 3] where the
    strict path picks [3, 0] (same input as test_adapter_npu_kernels.py:91-115)."""
    meta = adapter_mod._pack_slot_meta(torch.tensor([0, 0, 1, 0]), torch.tensor([1, 0, 0, 0]))
    ss = _ids([0])
    sel = oracle.pop_reusable_slots(meta, ss, _ids([1]), 2, order="prefix")
    assert sel.tolist() == [0, 3]
    assert ss.tolist() == [0]
    assert adapter_mod._slot_meta_usage_counts(meta).tolist() == [0, 0, 0, 0]


def test_pop_bad_blocked_index_raises_without_mutation():
    meta = _meta([0, 16, 32])
    ss = _ids([1])
    with pytest.raises(oracle.OracleBadIndex):
        oracle.pop_reusable_slots(meta, ss, _ids([5]), 1)
    assert meta.tolist() == [0, 16, 32] and ss.tolist() == [1]


# ---------------------------------------------------------------------------
# clock streams recorded from the reference
# ---------------------------------------------------------------------------


def _pack16(pins, usage):
    """16-bit slot word: 8-bit pin | 8-bit usage << 8."""
    return ((pins.to(torch.int64) & 255) | ((usage.to(torch.int64) & 255) << 8)).to(torch.uint16)


@pytest.mark.parametrize("fixture,pack", [("clock_stream.json", adapter_mod._pack_slot_meta),
                                          ("clock_stream_u16.json", _pack16)])
def test_clock_streams_match_reference(golden_dir, fixture, pack):
    for rec in _load(golden_dir, fixture):
        p = rec["params"]
        meta = workloads.clock_initial_meta(p, pack)
        ss = _ids([0])
        victims, done, rc = oracle.clock_stream(meta, ss, p["num_steps"], p["alloc_per_step"],
                                                workloads.zipf_reaccess(p), p["reaccess_per_step"])
        assert rc == 0 and done == rec["steps_done"]
        assert victims.tolist() == rec["victims"]
        assert workloads.sha256_of(meta) == rec["final_slot_meta_sha256"]
        assert int(ss[0]) == rec["final_search_start"]


# ---------------------------------------------------------------------------
# adapter orchestration on CPU through the oracle op set
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("case_index", range(60))
def test_adapter_scenarios_match_reference(case_index):
    case = scenario_runner.load_scenarios()[case_index]
    ops = OracleOps()
    scenario_runner.run_and_compare(case, torch.device("cpu"), native_ext=ops, backend_ops=ops)


def test_program_transcript(golden_dir):
    """The reference demo (test_program.py:11-54) through this adapter."""
    expected = _load(golden_dir, "program.json")["stdout"]
    ops = OracleOps()
    backend = adapter_mod.InMemoryBlockStoreBackend(
        {i: torch.tensor([float(i), 10.0 + i]) for i in range(4)}, ops=ops)
    ad = adapter_mod.KVCacheAdapter(2, 4, torch.zeros((2, 2)), backend, native_ext=ops)
    assert f"load [0, 1] -> {ad.load(_ids([0, 1]))}" == expected[1]
    ad.release(_ids([0]))
    assert f"after releasing 0, load [2] -> {ad.load(_ids([2]))}" == expected[2]
    ad.save(_ids([2]), torch.tensor([[200.0, 201.0]]))
    ad.release(_ids([1, 2]))
    assert f"load [2, 3] -> {ad.load(_ids([2, 3]))}" == expected[3]
    assert ad.debug_snapshot()["logical_to_physical"] == {2: 0, 3: 1}


def test_cpu_adapter_without_op_set_is_refused():
    backend = adapter_mod.InMemoryBlockStoreBackend(num_logical_blocks=4)
    with pytest.raises(RuntimeError, match="CUDA"):
        adapter_mod.KVCacheAdapter(2, 4, torch.zeros((2, 2)), backend)


# ---------------------------------------------------------------------------
# block layout and slot mapping (adapter.py:81-123, :1266-1295)
# ---------------------------------------------------------------------------


def test_layout_and_slot_mapping_match_reference(golden_dir):
    for rec in _load(golden_dir, "layout.json")["cases"]:
        layout = _MergedKVBlockLayout.detect(tuple(rec["block_shape"]))
        assert (layout is not None) == rec["detected"]
        if layout is None:
            continue
        assert list(layout.transfer_shape) == rec["transfer_shape"]
        assert layout.block_size == rec["block_size"] and layout.hidden_dim == rec["hidden_dim"]
        assert layout.token_major == rec["token_major"]
        slots = _ids(rec["slot_ids"])
        assert layout.physical_slot_mapping(slots).tolist() == rec["physical_slot_mapping"]
        assert moves.physical_slot_mapping(slots, layout.block_size).tolist() == rec["physical_slot_mapping"]
        assert layout.dense_slot_mapping(3, device=torch.device("cpu")).tolist() == rec["dense_slot_mapping"]
        assert layout.chunk_offsets(3) == rec["chunk_offsets"]
        assert layout.chunk_sizes(3) == rec["chunk_sizes"]


@pytest.mark.parametrize(("block_shape", "expected"), [((16, 2, 4, 8), (16, 2, 32)), ((2, 16, 4, 8), (2, 16, 32))])
def test_merged_kv_block_layout_round_trips(block_shape, expected):
    """test_adapter.py:432-449 of the reference."""
    layout = _MergedKVBlockLayout.detect(block_shape)
    assert tuple(layout.transfer_shape) == expected
    payload = torch.arange(1, 1 + int(torch.tensor(block_shape).prod()), dtype=torch.float32).view(block_shape)
    flat = layout.flatten_block_batch(payload.unsqueeze(0))
    assert tuple(flat.shape[1:]) == expected
    assert torch.equal(layout.restore_block_tensor(flat[0]), payload)


def test_token_planes_address_the_merged_block():
    """K/V token planes of a merged cache index the same bytes as the
    transfer-shape view (token-major and kv-major)."""
    for shape in [(4, 2, 3, 5), (2, 4, 3, 5)]:
        layout = _MergedKVBlockLayout.detect(shape)
        cache = torch.arange(6 * int(torch.tensor(shape).prod()), dtype=torch.float32).view(6, *shape)
        k, v = layout.token_planes(cache)
        flat = cache.view(6, *layout.transfer_shape)
        for b in range(6):
            for t in range(layout.block_size):
                if layout.token_major:
                    assert torch.equal(k[b, t], flat[b, t, 0]) and torch.equal(v[b, t], flat[b, t, 1])
                else:
                    assert torch.equal(k[b, t], flat[b, 0, t]) and torch.equal(v[b, t], flat[b, 1, t])


def test_token_moves_round_trip_on_cpu():
    gen = torch.Generator().manual_seed(1234)
    planes = [torch.randn(5, 4, 3, generator=gen) for _ in range(3)]
    mapping = _ids([7, -1, 0, 19, 4, 12])
    chunks = moves.gather_tokens(planes, mapping, tokens_per_chunk=3)
    assert chunks.shape == (2, 3, 3, 3)
    for p, plane in enumerate(planes):
        flat = plane.reshape(20, 3)
        for t, s in enumerate(mapping.tolist()):
            row = chunks[t // 3, p, t % 3]
            assert torch.equal(row, flat[s] if s >= 0 else torch.zeros(3))
    fresh = [torch.zeros_like(p) for p in planes]
    moves.scatter_tokens(fresh, mapping, chunks, tokens_per_chunk=3)
    for p in range(3):
        for s in [7, 0, 19, 4, 12]:
            assert torch.equal(fresh[p].reshape(20, 3)[s], planes[p].reshape(20, 3)[s])
