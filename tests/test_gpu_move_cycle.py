"""GPU parity for move_cycle (kvca_move_cycle): a booked cycle's spill gathers
and token scatters in one launch, against the same steps run one after the
other with the oracle's torch CPU moves (gather_layers, then scatter_tokens,
per step), byte for byte: the spill rows and the whole cache.

Schedules are built to hit every ordering the launch has to keep:
  - decode-like: sequences append one token per step; a full block is
    released and a new one popped, preferring blocks released earlier in the
    same call (a gather of bytes this launch wrote, then new tokens into the
    same block: the same slots written again after the gather);
  - random: distinct random slots and random victims, among them blocks
    written before and after the step that evicts them, and repeated victims;
plus padding (-1) slots and victims, rows of 256 B, 576 B and 2 KiB (block
rows of 4 KiB to 32 KiB: rows cut into item pieces, several rows per item,
division by non-powers of two), steps without victims, several launches on
one scratch, and the argument errors."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from kv_cache_adapter_b200 import _lib
from oracle import moves

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


@pytest.fixture(scope="module")
def ops():
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda as m

    return m


def _decode_schedule(rng, nb: int, bs: int, steps: int, seqs: int):
    cur = rng.choice(nb, seqs, replace=False).astype(np.int64)
    pos = rng.integers(0, bs, seqs).astype(np.int64)
    free = [b for b in rng.permutation(nb).tolist() if b not in set(cur.tolist())]
    released: list[int] = []
    slot_mapping = np.empty((steps, seqs), np.int64)
    victims: list[int] = []
    offs = [0]
    for q in range(steps):
        now_released = []
        for s in np.nonzero(pos == bs)[0]:
            if released and rng.random() < 0.6:  # a block whose tokens this call wrote
                v = released.pop(int(rng.integers(len(released))))
            else:
                v = free.pop()
            victims.append(v)
            now_released.append(int(cur[s]))
            cur[s], pos[s] = v, 0
        released.extend(now_released)  # a step pops before it releases
        offs.append(len(victims))
        slot_mapping[q] = cur * bs + pos
        pos += 1
    return slot_mapping, np.array(victims, np.int64), np.array(offs, np.int64)


def _random_schedule(rng, nb: int, bs: int, steps: int, seqs: int):
    slots = rng.permutation(nb * bs)[: steps * seqs].reshape(steps, seqs).astype(np.int64)
    counts = rng.integers(0, 7, steps)
    if steps > 1:
        counts[1] = 0  # a step without victims
    offs = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
    victims = rng.integers(0, nb, int(offs[-1])).astype(np.int64)
    # blocks written at the previous step, and blocks the next step writes
    for q in range(1, steps - 1):
        if counts[q] >= 2:
            victims[offs[q]] = slots[q - 1, rng.integers(seqs)] // bs
            victims[offs[q] + 1] = slots[q + 1, rng.integers(seqs)] // bs
    if offs[-1] > 3:
        victims[1] = victims[0]  # the same block twice
    return slots, victims, offs


def _rows_of(spill: torch.Tensor) -> torch.Tensor:
    """Spill chunks (n, P, cb, *block) as rows (n * cb, P, *block): row e is
    block e % cb of chunk e // cb."""
    n, P, cb = spill.shape[:3]
    return spill.transpose(1, 2).reshape(n * cb, P, *spill.shape[3:])


def _reference(planes, bs, slot_mapping, victims, offs, token_rows, spill_rows):
    """The steps one after the other on CPU planes (modified in place);
    spill_rows (rows, P, *block) is updated in place."""
    steps, seqs = slot_mapping.shape
    tok_planes = [p.view(p.shape[0], bs, -1) for p in planes]
    for q in range(steps):
        a, b = int(offs[q]), int(offs[q + 1])
        vq = victims[a:b]
        live = vq >= 0
        if live.any():
            got = moves.gather_layers(planes, vq[live], blocks_per_chunk=1)  # (k, P, 1, *block)
            spill_rows[torch.nonzero(live).flatten() + a] = got[:, :, 0]
        rows = token_rows[q if token_rows.shape[0] > 1 else 0][None]
        moves.scatter_tokens(tok_planes, slot_mapping[q], rows, tokens_per_chunk=seqs)


def _run(ops, planes_cpu, bs, slot_mapping, victims, offs, token_rows, *, spill_chunks=None, cb=1):
    planes = [p.to(DEV) for p in planes_cpu]
    tok_table = ops.PlaneTable([p.view(p.shape[0], bs, -1) for p in planes], 2)
    blk_table = ops.PlaneTable(planes, 1)
    V = int(offs[-1])
    n_spill = spill_chunks if spill_chunks is not None else max(1, -(-V // cb))
    spill0 = torch.from_numpy(np.random.default_rng(V).integers(0, 256, (n_spill, len(planes), cb, *planes[0].shape[1:]),
                                                                  dtype=np.uint8))
    spill = spill0.to(DEV)
    ops.move_cycle(tok_table, torch.from_numpy(slot_mapping).to(DEV), token_rows.to(DEV), blk_table,
                   torch.from_numpy(victims).to(DEV), torch.from_numpy(offs).to(DEV), spill, blocks_per_chunk=cb,
                   check=True)
    torch.cuda.synchronize(DEV)
    return [p.cpu() for p in planes], spill.cpu(), spill0


def _check(ops, rng, nb, bs, P, row, steps, seqs, kind, cb=1, shared_rows=False, pad=False):
    planes = [torch.from_numpy(rng.integers(0, 256, (nb, bs, row), dtype=np.uint8)) for _ in range(P)]
    sched = _decode_schedule if kind == "decode" else _random_schedule
    slot_mapping, victims, offs = sched(rng, nb, bs, steps, seqs)
    if pad:
        slot_mapping[rng.integers(0, steps, 5), rng.integers(0, seqs, 5)] = -1
        if offs[-1]:
            victims[rng.integers(0, int(offs[-1]), 2)] = -1
    token_rows = torch.from_numpy(rng.integers(0, 256, (1 if shared_rows else steps, P, seqs, row), dtype=np.uint8))
    got_planes, got_spill, spill0 = _run(ops, planes, bs, slot_mapping, victims, offs, token_rows, cb=cb)
    want_spill = _rows_of(spill0).clone()
    _reference(planes, bs, torch.from_numpy(slot_mapping), torch.from_numpy(victims), offs, token_rows, want_spill)
    assert torch.equal(_rows_of(got_spill), want_spill), "spill"
    for p in range(P):
        assert torch.equal(got_planes[p], planes[p]), f"plane {p}"
    return slot_mapping, victims, offs


@pytest.mark.parametrize("row,bs", [(2048, 16), (256, 16), (576, 16), (2048, 4)])
@pytest.mark.parametrize("kind", ["decode", "random"])
def test_move_cycle_matches_steps_one_after_another(ops, row, bs, kind):
    rng = np.random.default_rng(row + bs + len(kind))
    nb = 96 if kind == "decode" else 160
    sm, victims, offs = _check(ops, rng, nb, bs, 8, row, 16, 24, kind)
    if kind == "decode":  # the schedule did evict blocks written earlier in the call
        written = set()
        raw = 0
        for q in range(16):
            raw += len(set(victims[offs[q]:offs[q + 1]].tolist()) & written)
            written |= set((sm[q] // bs).tolist())
        assert raw > 0


@pytest.mark.parametrize("shared_rows,pad,cb", [(True, False, 1), (False, True, 1), (False, False, 2)])
def test_move_cycle_layouts_and_padding(ops, shared_rows, pad, cb):
    rng = np.random.default_rng(11 + cb + 2 * pad)
    _check(ops, rng, 128, 8, 6, 1024, 12, 20, "decode" if cb == 1 else "random", cb=cb, shared_rows=shared_rows,
           pad=pad)


def test_move_cycle_longest_call_and_scratch_reuse(ops):
    """32 steps (the most one call takes), then more calls on the same
    scratch: each launch starts from the words the previous one left."""
    rng = np.random.default_rng(5)
    for kind, steps in (("decode", 32), ("random", 7), ("decode", 16), ("random", 1)):
        _check(ops, rng, 200, 8, 4, 512, steps, 30, kind)


def test_move_cycle_argument_errors(ops):
    rng = np.random.default_rng(9)
    nb, bs, P, row, steps, seqs = 32, 4, 2, 256, 4, 6
    planes = [torch.from_numpy(rng.integers(0, 256, (nb, bs, row), dtype=np.uint8)).to(DEV) for _ in range(P)]
    tok = ops.PlaneTable([p.view(nb, bs, -1) for p in planes], 2)
    blk = ops.PlaneTable(planes, 1)
    sm = torch.from_numpy(rng.permutation(nb * bs)[: steps * seqs].reshape(steps, seqs).astype(np.int64)).to(DEV)
    rows = torch.zeros((steps, P, seqs, row), dtype=torch.uint8, device=DEV)
    victims = torch.arange(4, dtype=torch.int64, device=DEV)
    spill = torch.zeros((4, P, 1, bs, row), dtype=torch.uint8, device=DEV)
    before = [p.clone() for p in planes]
    # offsets that do not start at 0, that decrease, or that pass the spill rows: nothing moves
    for bad in ([1, 1, 2, 3, 4], [0, 2, 1, 3, 4], [0, 1, 2, 3, 5]):
        spill5 = torch.zeros((5, P, 1, bs, row), dtype=torch.uint8, device=DEV)
        v = torch.arange(5, dtype=torch.int64, device=DEV)
        with pytest.raises(ValueError):
            ops.move_cycle(tok, sm, rows, blk, v, torch.tensor(bad, device=DEV), spill5 if bad[-1] < 5 else spill,
                           check=True)
        assert all(torch.equal(a, b) for a, b in zip(planes, before))
    # a slot past the cache: that row is refused, the others move
    sm2 = sm.clone()
    sm2[2, 3] = nb * bs + 1
    with pytest.raises(IndexError):
        ops.move_cycle(tok, sm2, rows, blk, victims, torch.tensor([0, 1, 2, 3, 4], device=DEV), spill, check=True)
    # host-side refusals: too many steps, other planes, misaligned rows
    lib = _lib.load()
    assert lib.kvca_move_cycle_scratch_bytes(1000) == 512 + 16 * 1000
    with pytest.raises(ValueError):
        ops.move_cycle(tok, torch.zeros((33, seqs), dtype=torch.int64, device=DEV),
                       torch.zeros((33, P, seqs, row), dtype=torch.uint8, device=DEV), blk, victims,
                       torch.zeros(34, dtype=torch.int64, device=DEV), spill, check=True)
    other = ops.PlaneTable([p.clone() for p in planes], 1)
    with pytest.raises(ValueError):
        ops.move_cycle(tok, sm, rows, other, victims, torch.tensor([0, 1, 2, 3, 4], device=DEV), spill, check=True)
