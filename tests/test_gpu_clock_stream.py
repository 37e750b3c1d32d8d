"""GPU parity: the device-resident clock stream (pop -> refill -> Zipf re-access
bumps) against recorded reference streams and the oracle, up to the full
clock-stress size (1,048,576 slots, 200k allocations)."""
from __future__ import annotations

import json

import numpy as np
import pytest
import torch

import oracle
from kv_cache_adapter_b200 import adapter as adapter_mod
from kv_cache_adapter_b200 import workloads

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


@pytest.fixture(scope="module")
def ops():
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda as m

    return m


def _pack16(pins, usage):
    return ((pins.to(torch.int32) & 255) | ((usage.to(torch.int32) & 255) << 8)).to(torch.uint16)


# "batched" runs on a cooperative grid (one CTA per SM), "batched1" on one CTA
METHODS = ["batched", "batched1", "steps"]


def _method(name):
    return ("batched", 1) if name == "batched1" else (name, 0)


@pytest.mark.parametrize("method", METHODS)
@pytest.mark.parametrize("fixture", ["clock_stream.json", "clock_stream_u16.json"])
def test_recorded_reference_streams(ops, golden_dir, method, fixture):
    """Streams recorded from the reference (8-bit slot meta, and its 16-bit mode)."""
    pack = adapter_mod._pack_slot_meta if fixture == "clock_stream.json" else _pack16
    for rec in json.loads((golden_dir / fixture).read_text()):
        p = rec["params"]
        meta = workloads.clock_initial_meta(p, pack).to(DEV)
        ss = torch.zeros(1, dtype=torch.int64, device=DEV)
        victims, done = ops.clock_stream(meta, ss, p["num_steps"], p["alloc_per_step"],
                                         workloads.zipf_reaccess(p).to(DEV), p["reaccess_per_step"],
                                         method=_method(method)[0], ctas=_method(method)[1])
        assert int(done) == rec["steps_done"]
        assert victims.tolist() == rec["victims"]
        assert workloads.sha256_of(meta) == rec["final_slot_meta_sha256"]
        assert int(ss[0]) == rec["final_search_start"]


def _run_both(ops, p, *, order="grouped", bits=8, method="batched"):
    pack = adapter_mod._pack_slot_meta if bits == 8 else _pack16
    meta_h = workloads.clock_initial_meta(p, pack)
    reacc = workloads.zipf_reaccess(p)
    ss_h = torch.zeros(1, dtype=torch.int64)
    want, done_h, rc = oracle.clock_stream(meta_h, ss_h, p["num_steps"], p["alloc_per_step"], reacc,
                                           p["reaccess_per_step"], order=order)
    meta_d = workloads.clock_initial_meta(p, pack).to(DEV)
    ss_d = torch.zeros(1, dtype=torch.int64, device=DEV)
    name, ctas = _method(method)
    got, done_d = ops.clock_stream(meta_d, ss_d, p["num_steps"], p["alloc_per_step"], reacc.to(DEV),
                                   p["reaccess_per_step"], order=order, method=name, ctas=ctas, check=False)
    torch.cuda.synchronize()
    return (want, done_h, rc, meta_h, ss_h), (got, int(done_d), meta_d, ss_d)


@pytest.mark.parametrize("method", METHODS)
@pytest.mark.parametrize("order", ["grouped", "prefix"])
@pytest.mark.parametrize("bits", [8, 16])
@pytest.mark.parametrize("k,m,usage_hi", [(1, 1, 3), (256, 256, 3), (5, 40, 15), (64, 8, 1)])
def test_streams_match_oracle(ops, method, order, bits, k, m, usage_hi):
    p = workloads.clock_params(65536 + 37, 3000 if k == 1 else 400, k, m, seed=4242 + k + m,
                               usage_hi=usage_hi)
    (want, done_h, rc, meta_h, ss_h), (got, done_d, meta_d, ss_d) = _run_both(ops, p, order=order, bits=bits,
                                                                              method=method)
    assert rc == 0 and done_h == done_d == p["num_steps"]
    assert torch.equal(got.cpu(), want)
    assert np.array_equal(meta_d.cpu().numpy(), meta_h.numpy())
    assert int(ss_d[0]) == int(ss_h[0])
    ops.check_status(DEV)


@pytest.mark.parametrize("method", METHODS)
@pytest.mark.parametrize("k", [1, 256])
def test_full_size_clock_stress_matches_oracle(ops, k, method):
    """1,048,576 slots, usage U{0..3}, 5% pinned, 200k allocations with one
    Zipf(1.1) re-access per allocation: identical victim sequence and final
    usage array."""
    steps = 200_000 // k
    p = workloads.clock_params(1 << 20, steps, k, k, seed=1234)
    (want, done_h, rc, meta_h, ss_h), (got, done_d, meta_d, ss_d) = _run_both(ops, p, method=method)
    assert rc == 0 and done_h == done_d == steps
    assert torch.equal(got.cpu(), want)
    assert workloads.sha256_of(meta_d) == workloads.sha256_of(meta_h)
    assert int(ss_d[0]) == int(ss_h[0])
    ops.check_status(DEV)


@pytest.mark.parametrize("k,m,n,steps,usage_hi,pinned", [
    (1, 4, 4096, 20000, 3, 0.05),      # long stream: the sweep wraps, many aging events
    (3, 64, 1000, 3000, 15, 0.3),      # short epochs: exact stretches between them
    (17, 5, 2048, 2000, 1, 0.0),       # k not dividing the candidate runs
    (1, 0, 777, 5000, 2, 0.5),         # no re-access at all
    (128, 1024, 4096, 300, 7, 0.1),    # heavy re-access with duplicates in each batch
])
@pytest.mark.parametrize("method", ["batched", "batched1"])
def test_batched_stream_with_frequent_aging_matches_oracle(ops, k, m, n, steps, usage_hi, pinned, method):
    p = workloads.clock_params(n, steps, k, m, seed=99 + k + m + n, usage_hi=usage_hi, pinned_frac=pinned)
    (want, done_h, rc, meta_h, ss_h), (got, done_d, meta_d, ss_d) = _run_both(ops, p, method=method)
    assert done_d == done_h
    assert torch.equal(got.cpu()[: done_h * k], want[: done_h * k])
    assert np.array_equal(meta_d.cpu().numpy(), meta_h.numpy())
    assert int(ss_d[0]) == int(ss_h[0])
    if rc == 0:
        ops.check_status(DEV)


@pytest.mark.parametrize("method", METHODS)
def test_stream_stops_on_insufficient_capacity(ops, method):
    from kv_cache_adapter_b200.errors import InsufficientCapacityError

    # 10 slots, 3 pinned: 7 reusable; victims are refilled unpinned, so the
    # stream only fails when a single step asks for more than 7.
    pins = torch.tensor([1, 0, 0, 1, 0, 0, 1, 0, 0, 0])
    meta = adapter_mod._pack_slot_meta(pins, torch.zeros(10, dtype=torch.int64)).to(DEV)
    ss = torch.zeros(1, dtype=torch.int64, device=DEV)
    reacc = torch.zeros(0, dtype=torch.int64, device=DEV)
    name, ctas = _method(method)
    victims, done = ops.clock_stream(meta, ss, 3, 8, reacc, 0, check=False, method=name, ctas=ctas)
    assert int(done) == 0
    with pytest.raises(InsufficientCapacityError):
        ops.check_status(DEV)
    victims, done = ops.clock_stream(meta, ss, 3, 7, reacc, 0, method=name, ctas=ctas)
    assert int(done) == 3


@pytest.mark.parametrize("ctas", [2, 7, 33])
def test_batched_stream_on_odd_grids(ops, ctas):
    """Grids that do not divide the slots, candidates or events evenly."""
    p = workloads.clock_params(100_003, 500, 3, 17, seed=77 + ctas, usage_hi=5, pinned_frac=0.2)
    meta_h = workloads.clock_initial_meta(p, adapter_mod._pack_slot_meta)
    reacc = workloads.zipf_reaccess(p)
    ss_h = torch.zeros(1, dtype=torch.int64)
    want, done_h, rc = oracle.clock_stream(meta_h, ss_h, p["num_steps"], p["alloc_per_step"], reacc,
                                           p["reaccess_per_step"])
    meta_d = workloads.clock_initial_meta(p, adapter_mod._pack_slot_meta).to(DEV)
    ss_d = torch.zeros(1, dtype=torch.int64, device=DEV)
    got, done_d = ops.clock_stream(meta_d, ss_d, p["num_steps"], p["alloc_per_step"], reacc.to(DEV),
                                   p["reaccess_per_step"], ctas=ctas)
    assert int(done_d) == done_h
    assert torch.equal(got.cpu()[: done_h * 3], want[: done_h * 3])
    assert np.array_equal(meta_d.cpu().numpy(), meta_h.numpy())
    assert int(ss_d[0]) == int(ss_h[0])
    ops.check_status(DEV)


def test_batched_stream_replays_from_a_cuda_graph(ops):
    """The cooperative launch (and its scratch clearing) can be captured in a
    CUDA graph: a replay from the same start state gives the same stream."""
    p = workloads.clock_params(65536, 500, 2, 3, seed=31)
    meta0 = workloads.clock_initial_meta(p, adapter_mod._pack_slot_meta).to(DEV)
    reacc = workloads.zipf_reaccess(p).to(DEV)
    meta = meta0.clone()
    ss = torch.zeros(1, dtype=torch.int64, device=DEV)
    victims = torch.empty(p["num_steps"] * 2, dtype=torch.int64, device=DEV)
    want, _ = ops.clock_stream(meta, ss, p["num_steps"], 2, reacc, 3, check=True)
    want_meta, want_ss = meta.clone(), ss.clone()
    meta.copy_(meta0)
    ss.zero_()
    ops.clock_stream(meta, ss, p["num_steps"], 2, reacc, 3, victims=victims)  # scratch and status exist now
    torch.cuda.synchronize()
    side = torch.cuda.Stream(DEV)
    side.wait_stream(torch.cuda.current_stream(DEV))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        ops.clock_stream(meta, ss, p["num_steps"], 2, reacc, 3, victims=victims, check=False)  # warm this stream
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=side):
            ops.clock_stream(meta, ss, p["num_steps"], 2, reacc, 3, victims=victims, check=False)
    torch.cuda.current_stream(DEV).wait_stream(side)
    for _ in range(2):
        meta.copy_(meta0)
        ss.zero_()
        victims.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(victims, want)
        assert torch.equal(meta, want_meta) and torch.equal(ss, want_ss)
    del graph
    ops.check_status(DEV)
