"""The decode append + gather mix (reshape-and-cache with clock eviction).

CPU: the driver's host logic through the oracle op set.
GPU: the same driver on the CUDA op set against the oracle, step by step:
spilled blocks, the whole cache, slot_meta, l2p / p2l and search_start must
be identical bytes after every step.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from kv_cache_adapter_b200.workloads import DecodeMix
from oracle_ops import OracleOps

SMALL = dict(layers=2, heads=2, head_dim=32, block_size=16, num_blocks=256, seqs=48, max_steps=200)


def _rows(step: int, mix: DecodeMix) -> torch.Tensor:
    gen = torch.Generator().manual_seed(10_000 + step)
    return torch.randn((1, mix.num_planes, mix.seqs, *mix.row_shape), generator=gen).to(mix.kv.dtype)


def test_decode_mix_host_logic_on_cpu():
    ops = OracleOps()
    mix = DecodeMix(ops, torch.device("cpu"), **SMALL)
    pins0 = int(((mix.slot_meta & 15) != 0).sum())
    assert pins0 == SMALL["seqs"]
    total_new = 0
    for step in range(120):
        need = mix.need_new_blocks().size
        spill = mix.step(_rows(step, mix))
        assert spill.shape[0] == need
        total_new += need
        # one pinned block per sequence, all of them distinct
        pinned = torch.nonzero((mix.slot_meta & 15) != 0).flatten().sort().values
        assert torch.equal(pinned, mix.cur_block_dev.sort().values)
        # l2p and p2l stay inverse on the resident blocks
        assert torch.equal(mix.l2p[mix.p2l], torch.arange(mix.num_blocks))
    assert total_new == mix.evictions > 0
    assert mix.tokens == 120 * SMALL["seqs"]


@pytest.mark.gpu
@pytest.mark.parametrize("pipelined", [False, True])
def test_decode_mix_matches_oracle_step_by_step(pipelined):
    """Unpipelined, and with each step's bookkeeping on its own stream
    overlapping the previous step's moves: identical bytes either way."""
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda as cuda_ops

    dev = torch.device("cuda", 0)
    gpu = DecodeMix(cuda_ops, dev, **SMALL)
    gpu.pipelined = pipelined
    assert gpu.pipelined == pipelined
    cpu = DecodeMix(OracleOps(), torch.device("cpu"), **SMALL)
    cpu.kv.copy_(gpu.kv.cpu())
    for step in range(150):
        rows = _rows(step, cpu)
        spill_g = gpu.step(rows.to(dev), check=True)
        spill_c = cpu.step(rows)
        assert torch.equal(spill_g.cpu().view(torch.int16), spill_c.view(torch.int16)), step
        assert torch.equal(gpu.slot_meta.cpu(), cpu.slot_meta), step
        assert torch.equal(gpu.l2p.cpu(), cpu.l2p) and torch.equal(gpu.p2l.cpu(), cpu.p2l), step
        assert int(gpu.search_start[0]) == int(cpu.search_start[0]), step
        for name in ("cur_block_dev", "cur_logical_dev", "pos_dev", "next_logical_dev"):
            assert torch.equal(getattr(gpu, name).cpu(), getattr(cpu, name)), (step, name)
    assert gpu._append is not None  # the one-launch bookkeeping ran on the GPU
    assert torch.equal(gpu.kv.cpu().view(torch.int16), cpu.kv.view(torch.int16))
    assert gpu.evictions == cpu.evictions > 100


@pytest.mark.gpu
@pytest.mark.parametrize("pipelined", [False, True])
def test_decode_mix_graph_replay_matches_eager(pipelined):
    """A captured cycle of block_size steps, replayed, leaves exactly the state
    that running the same steps eagerly (unpipelined) leaves; pipelined, the
    capture forks the bookkeeping stream inside the graph, and eager steps
    after the replays still line up."""
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda as cuda_ops

    dev = torch.device("cuda", 0)
    eager = DecodeMix(cuda_ops, dev, **SMALL)
    graphed = DecodeMix(cuda_ops, dev, **SMALL)
    graphed.pipelined = pipelined
    rows = _rows(0, eager).to(dev)
    for _ in range(SMALL["block_size"] + 1):  # one full cycle eagerly, then step 1 of the next
        eager.step(rows)
        graphed.step(rows)
    graph, per_cycle = graphed.capture_cycle(rows)
    assert per_cycle == SMALL["seqs"]
    for _ in range(5):
        for _ in range(SMALL["block_size"]):
            eager.step(rows)
        graph.replay()
    for step in range(7):  # eager steps after the replays
        eager.step(_rows(step, eager).to(dev))
        graphed.step(_rows(step, eager).to(dev))
    torch.cuda.synchronize()
    cuda_ops.check_status(dev)
    assert torch.equal(eager.kv.view(torch.int16), graphed.kv.view(torch.int16))
    assert torch.equal(eager.slot_meta, graphed.slot_meta)
    assert torch.equal(eager.l2p, graphed.l2p) and torch.equal(eager.p2l, graphed.p2l)
    assert torch.equal(eager.search_start, graphed.search_start)
    assert torch.equal(eager.cur_block_dev, graphed.cur_block_dev)
    assert torch.equal(eager.next_logical_dev, graphed.next_logical_dev)


@pytest.mark.gpu
def test_append_step_errors_change_nothing():
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda as ops
    from kv_cache_adapter_b200.errors import InsufficientCapacityError

    dev = torch.device("cuda", 0)
    mix = DecodeMix(ops, dev, **SMALL)
    state = [t.clone() for t in (mix.slot_meta, mix.l2p, mix.p2l, mix.search_start, mix.cur_block_dev,
                                 mix.cur_logical_dev, mix.pos_dev, mix.next_logical_dev)]
    need = torch.tensor([0, 1], dtype=torch.int64, device=dev)
    victims = torch.empty(2, dtype=torch.int64, device=dev)
    sm = torch.empty(mix.seqs, dtype=torch.int64, device=dev)
    args = (mix.slot_meta, mix.search_start, mix.l2p, mix.p2l)
    tail = (mix.cur_block_dev, mix.cur_logical_dev, mix.pos_dev, mix.block_size, mix.next_logical_dev, victims, sm)
    with pytest.raises(IndexError):  # a sequence index outside [0, seqs)
        ops.append_step(*args, torch.tensor([0, mix.seqs], dtype=torch.int64, device=dev), *tail, check=True)
    pinned = mix.slot_meta | 1  # every slot pinned: no victim
    with pytest.raises(InsufficientCapacityError):
        ops.append_step(pinned, *args[1:], need, *tail, check=True)
    for before, after in zip(state, (mix.slot_meta, mix.l2p, mix.p2l, mix.search_start, mix.cur_block_dev,
                                     mix.cur_logical_dev, mix.pos_dev, mix.next_logical_dev)):
        assert torch.equal(before, after)
    ops.check_status(dev)
