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
# more sequences needing a block in one step than the bookkeeping CTA has threads
WIDE = dict(layers=1, heads=1, head_dim=16, block_size=4, num_blocks=8192, seqs=1500, max_steps=60)
# more sequences than the multi-step booking keeps in shared memory
HUGE = dict(layers=1, heads=1, head_dim=8, block_size=4, num_blocks=16384, seqs=5000, max_steps=40)


def _rows(step: int, mix: DecodeMix) -> torch.Tensor:
    gen = torch.Generator().manual_seed(10_000 + step)
    return torch.randn((1, mix.num_planes, mix.seqs, *mix.row_shape), generator=gen).to(mix.kv.dtype)


def test_decode_mix_host_logic_on_cpu():
    ops = OracleOps()
    mix = DecodeMix(ops, torch.device("cpu"), **SMALL)
    pins0 = int(((mix.slot_meta & 15) != 0).sum())
    assert pins0 == SMALL["seqs"]
    total_new = 0
    written = set()  # blocks the previous step's scatter wrote
    for step in range(120):
        need_set = mix.need_new_blocks()
        need = need_set.size
        spill = mix.step(_rows(step, mix))
        assert spill.shape[0] == need
        total_new += need
        # this step's victims were not written by the previous step's scatter
        # (the pop of a step precedes its release of the full blocks)
        victims = set(mix.cur_block_dev[torch.from_numpy(need_set)].tolist())
        assert not victims & written, step
        written = set(mix.cur_block_dev.tolist())
        # one pinned block per sequence, all of them distinct
        pinned = torch.nonzero((mix.slot_meta & 15) != 0).flatten().sort().values
        assert torch.equal(pinned, mix.cur_block_dev.sort().values)
        # l2p and p2l stay inverse on the resident blocks
        assert torch.equal(mix.l2p[mix.p2l], torch.arange(mix.num_blocks))
    assert total_new == mix.evictions > 0
    assert mix.tokens == 120 * SMALL["seqs"]


@pytest.mark.gpu
@pytest.mark.parametrize("pipelined,cfg", [(False, SMALL), (True, SMALL), (True, WIDE)])
def test_decode_mix_matches_oracle_step_by_step(pipelined, cfg):
    """Unpipelined, and with each step's bookkeeping on its own stream
    overlapping the previous step's moves: identical bytes either way."""
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda as cuda_ops

    dev = torch.device("cuda", 0)
    gpu = DecodeMix(cuda_ops, dev, **cfg)
    gpu.pipelined = pipelined
    assert gpu.pipelined == pipelined
    cpu = DecodeMix(OracleOps(), torch.device("cpu"), **cfg)
    cpu.kv.copy_(gpu.kv.cpu())
    steps = min(150, cfg["max_steps"])
    wide = 0
    for step in range(steps):
        wide = max(wide, cpu.need_new_blocks().size)
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
    if cfg is WIDE:
        assert wide > 256


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


def _state(mix: DecodeMix):
    return [t.clone() for t in (mix.kv, mix.slot_meta, mix.l2p, mix.p2l, mix.search_start, mix.cur_block_dev,
                                mix.cur_logical_dev, mix.pos_dev, mix.next_logical_dev)]


def _assert_same_state(a: DecodeMix, b: DecodeMix):
    torch.cuda.synchronize()
    for x, y in zip(_state(a), _state(b)):
        assert torch.equal(x.view(torch.uint8) if x.dtype != torch.int64 else x,
                           y.view(torch.uint8) if y.dtype != torch.int64 else y)
    assert (a.evictions, a.tokens) == (b.evictions, b.tokens)


@pytest.mark.gpu
@pytest.mark.parametrize("one_launch", [False, True])
@pytest.mark.parametrize("cfg", [SMALL, WIDE, HUGE])
def test_cycle_booking_matches_single_steps(cfg, one_launch):
    """Whole-cycle booking (one append_steps launch per cycle, one cycle ahead
    of the moves), eager and replayed from a graph, leaves the same cache
    bytes and metadata as the same number of single unpipelined steps; the
    moves of a cycle are paired launches or one move_cycle launch, whose
    spill then holds every victim of the cycle (checked against the single
    steps' spills)."""
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda as cuda_ops

    dev = torch.device("cuda", 0)
    bs = cfg["block_size"]
    ref = DecodeMix(cuda_ops, dev, **cfg)
    cyc = DecodeMix(cuda_ops, dev, **cfg)
    rows = _rows(0, ref).to(dev)
    for _ in range(bs + 1):  # past the first step: positions periodic
        ref.step(rows)
        cyc.step(rows)
    cyc.start_cycles(one_launch=one_launch)
    cyc.run_cycle(rows)
    cyc.run_cycle(rows)
    cyc.stop_cycles(rows)
    spills = []
    for i in range(3 * bs):
        spill = ref.step(rows)
        if i >= 2 * bs:  # the last cycle's victims, step by step
            spills.append(spill.clone())
    _assert_same_state(ref, cyc)
    if one_launch:
        last = torch.cat(spills)
        assert torch.equal(cyc.spill[: last.shape[0]].view(torch.uint8), last.view(torch.uint8))
    # graph replays of two cycles each, then single steps again
    cyc.start_cycles(one_launch=one_launch)
    cyc.run_cycle(rows)
    graph, per_replay = cyc.capture_cycles(rows)
    cpr = cyc.CYCLE_BUFFERS
    assert per_replay == cpr * cfg["seqs"]
    replays = 2 if cfg is SMALL else 1
    for _ in range(replays):
        graph.replay()
    cyc.stop_cycles(rows)
    for _ in range(3):
        cyc.step(rows)
    for _ in range((2 + cpr * replays) * bs + 3):
        ref.step(rows)
    torch.cuda.synchronize()
    cuda_ops.check_status(dev)
    cyc.evictions += replays * per_replay  # graph replays are not counted on the host
    cyc.tokens += replays * cpr * bs * cfg["seqs"]
    _assert_same_state(ref, cyc)


@pytest.mark.gpu
@pytest.mark.parametrize("bits", [8, 16])
def test_append_steps_equals_single_steps_across_launches(bits):
    """300 steps in one append_steps call (two launches of at most 256 steps,
    the slot table copied into shared memory) against 300 append_step calls
    (table in global memory): victims, slot mappings and state, with 8- and
    16-bit slot words."""
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda as ops

    dev = torch.device("cuda", 0)
    cfg = dict(layers=1, heads=1, head_dim=8, block_size=4, num_blocks=2048, seqs=100, max_steps=320)
    a = DecodeMix(ops, dev, **cfg)
    b = DecodeMix(ops, dev, **cfg)
    if bits == 16:  # the same pins and usage counts in 16-bit words (8-bit fields)
        w = a.slot_meta.cpu().numpy().astype(np.uint16)
        w16 = torch.from_numpy((w & 15) | ((w >> 4) << 8))
        a.slot_meta = w16.to(dev)
        b.slot_meta = w16.to(dev)
    steps = 300
    pos = a.pos.copy()
    needs, offs = [], [0]
    for _ in range(steps):
        need = np.nonzero(pos == cfg["block_size"])[0]
        needs.append(need)
        offs.append(offs[-1] + need.size)
        pos[need] = 0
        pos += 1
    need_all = torch.tensor(np.concatenate(needs), dtype=torch.int64, device=dev)
    offsets = torch.tensor(offs, dtype=torch.int64, device=dev)
    victims = torch.full((offs[-1],), -1, dtype=torch.int64, device=dev)
    sm = torch.full((steps, cfg["seqs"]), -1, dtype=torch.int64, device=dev)
    ops.append_steps(a.slot_meta, a.search_start, a.l2p, a.p2l, need_all, offsets, a.cur_block_dev,
                     a.cur_logical_dev, a.pos_dev, a.block_size, a.next_logical_dev, victims, sm, check=True)
    for s in range(steps):
        v = torch.empty(offs[s + 1] - offs[s], dtype=torch.int64, device=dev)
        one = torch.empty(cfg["seqs"], dtype=torch.int64, device=dev)
        ops.append_step(b.slot_meta, b.search_start, b.l2p, b.p2l, need_all[offs[s]:offs[s + 1]], b.cur_block_dev,
                        b.cur_logical_dev, b.pos_dev, b.block_size, b.next_logical_dev, v, one, check=True)
        assert torch.equal(v, victims[offs[s]:offs[s + 1]]), s
        assert torch.equal(one, sm[s]), s
    for x, y in zip(_state(a)[1:], _state(b)[1:]):
        assert torch.equal(x, y)
    assert offs[-1] > cfg["num_blocks"] // 4  # enough evictions to age the table


@pytest.mark.gpu
def test_append_steps_errors():
    """Bad offsets change nothing; too few reusable slots at step s leave the
    earlier steps done and step s unchanged."""
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda as ops
    from kv_cache_adapter_b200.errors import InsufficientCapacityError

    dev = torch.device("cuda", 0)
    cfg = dict(layers=1, heads=1, head_dim=8, block_size=4, num_blocks=64, seqs=8, max_steps=64)
    mix = DecodeMix(ops, dev, **cfg)
    state = _state(mix)
    need = torch.arange(8, dtype=torch.int64, device=dev)
    victims = torch.empty(8, dtype=torch.int64, device=dev)
    sm = torch.empty((2, 8), dtype=torch.int64, device=dev)
    args = (mix.slot_meta, mix.search_start, mix.l2p, mix.p2l, need)
    tail = (mix.cur_block_dev, mix.cur_logical_dev, mix.pos_dev, mix.block_size, mix.next_logical_dev, victims, sm)
    for bad in ([0, 5, 3], [0, 3, 9], [-1, 2, 4]):  # decreasing, past the need list, negative
        with pytest.raises(IndexError):
            ops.append_steps(*args, torch.tensor(bad, dtype=torch.int64, device=dev), *tail, check=True)
    for before, after in zip(state, _state(mix)):
        assert torch.equal(before, after)
    # all but 3 unpinned slots pinned: step 0 takes those 3 and releases the
    # 3 full blocks; step 1 needs 5
    meta = mix.slot_meta.clone()
    free = torch.nonzero((meta & 15) == 0).flatten()
    keep = free[:3]
    pinned = meta | 1
    pinned[keep] = meta[keep]
    mix.slot_meta.copy_(pinned)
    with pytest.raises(InsufficientCapacityError):
        ops.append_steps(*args, torch.tensor([0, 3, 8], dtype=torch.int64, device=dev), *tail, check=True)
    assert set(victims[:3].tolist()) == set(keep.tolist())
    assert int(mix.next_logical_dev[0]) == int(state[-1][0]) + 3  # step 0 committed, step 1 not
    ops.check_status(dev)
