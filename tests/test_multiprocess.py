"""CPU, two gloo ranks: the multi-rank pieces of bench.py.

Each rank owns one KV-head shard and its own block tables, so the data path
has no collective; what crosses ranks is the max-over-ranks timing and the
check that the replicated slot-table sweep picked identical victims on every
rank.  Both are exercised here with the oracle standing in for the GPU sweep.
"""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, results) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench
        import oracle
        from kv_cache_adapter_b200 import adapter as adapter_mod
        from kv_cache_adapter_b200 import workloads

        cpu = torch.device("cpu")
        slowest = bench._max_over_ranks(10.0 + rank, world, cpu)
        fastest = bench._min_over_ranks(10.0 + rank, world, cpu)
        # every rank runs the same clock stream on its replica of the slot table
        p = workloads.clock_params(4096, 300, 2, 2, seed=1234)
        meta = workloads.clock_initial_meta(p, adapter_mod._pack_slot_meta)
        victims, done, rc = oracle.clock_stream(meta, torch.zeros(1, dtype=torch.int64), 300, 2,
                                                workloads.zipf_reaccess(p), 2)
        same = bench._same_on_all_ranks(workloads.sha256_of(victims) + workloads.sha256_of(meta), world)
        differs = bench._same_on_all_ranks(f"rank-{rank}", world)
        # shards own different block tables (seed 1234 + rank)
        w = dict(bench.WORKLOADS["llama8b"], layers=1, seqs=4)
        _, _, table, _ = bench.build_cache(w, cpu, 1234 + rank)
        tables = [None] * world
        dist.all_gather_object(tables, table.tolist())
        results[rank] = (slowest, fastest, same, differs, rc, done, tables[0] != tables[1])
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_two_rank_harness_logic():
    world = 2
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    # both ranks need the same port
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=240)
        assert pr.exitcode == 0
    for rank in range(world):
        slowest, fastest, same, differs, rc, done, tables_differ = results[rank]
        assert slowest == 11.0 and fastest == 10.0
        assert same is True and differs is False
        assert rc == 0 and done == 300
        assert tables_differ


def _failing_worker(rank: int, world: int, port: int, results) -> None:
    import datetime

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    import bench

    if rank == 1:
        # this rank fails between steps: it never joins the next collective
        results[rank] = "left"
        os._exit(0)
    t0 = __import__("time").perf_counter()
    try:
        bench._max_over_ranks(1.0, world, torch.device("cpu"))
        results[rank] = "no error"
    except Exception as exc:  # the surviving rank learns of it instead of hanging
        results[rank] = (type(exc).__name__, __import__("time").perf_counter() - t0)
    os._exit(0)


@pytest.mark.timeout(300)
def test_a_rank_that_leaves_surfaces_as_an_error_not_a_hang():
    """A rank that exits between steps: the other rank's next collective (the
    bench's max-over-ranks timing) ends with an error within the process
    group's timeout."""
    world = 2
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, world, port, results)) for r in range(world)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=240)
        assert pr.exitcode == 0
    assert results[1] == "left"
    name, waited = results[0]
    assert name != "no error" and waited < 120
