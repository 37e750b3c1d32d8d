"""GPU parity of the paired move (kvca_scatter_gather through
scatter_tokens_gather_layers): a token scatter and a block gather over
disjoint blocks of one cache in one launch must give the bytes of the
oracle's torch CPU indexing (scatter_tokens, then gather_layers), for every
body the pair kernel can run on each side (rows under 128 B, 128 B to
1.5 KiB, larger), rows that force narrower vectors (two launches), an empty
side, padding tokens and bad ids."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import moves

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


@pytest.fixture(scope="module")
def ops():
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda as m

    return m


def _same(a: torch.Tensor, b: torch.Tensor) -> bool:
    a = a.detach().contiguous().cpu().view(torch.uint8).numpy()
    b = b.detach().contiguous().cpu().view(torch.uint8).numpy()
    return a.shape == b.shape and np.array_equal(a, b)


def _case(planes: int, num_blocks: int, bs: int, row: int, tokens: int, gathered: int, seed: int):
    gen = torch.Generator().manual_seed(seed)
    kv = torch.randint(0, 256, (planes, num_blocks, bs, row), generator=gen, dtype=torch.uint8)
    perm = torch.randperm(num_blocks, generator=gen)
    a_blocks, b_blocks = perm[: num_blocks // 2], perm[num_blocks // 2:]
    # token slots inside the scatter's half, distinct, some padding
    slots = (a_blocks.reshape(-1, 1) * bs + torch.arange(bs).reshape(1, -1)).reshape(-1)
    tokens = min(tokens, slots.numel())
    slots = slots[torch.randperm(slots.numel(), generator=gen)][:tokens].clone()
    if tokens > 4:
        slots[torch.randperm(tokens, generator=gen)[: tokens // 8]] = -1
    ids = b_blocks[torch.randint(0, b_blocks.numel(), (gathered,), generator=gen)]
    rows = torch.randint(0, 256, (1, planes, tokens, row), generator=gen, dtype=torch.uint8)
    return kv, slots, ids, rows


def _run(ops, kv, slots, ids, rows, bs, row, blocks_per_chunk):
    kv_d = kv.to(DEV)
    token_planes = [kv_d[p] for p in range(kv.shape[0])]
    block_planes = [kv_d[p].reshape(kv.shape[1], bs * row) for p in range(kv.shape[0])]
    k = ids.numel()
    out = torch.full((k // blocks_per_chunk if k else 0, kv.shape[0], blocks_per_chunk, bs * row), 7,
                     dtype=torch.uint8, device=DEV)
    ops.scatter_tokens_gather_layers(token_planes, slots.to(DEV), rows.to(DEV), block_planes, ids.to(DEV), out,
                                     tokens_per_chunk=max(slots.numel(), 1), blocks_per_chunk=blocks_per_chunk,
                                     check=True)
    # oracle: the two moves one after the other on CPU tensors
    ref = kv.clone()
    if slots.numel():
        moves.scatter_tokens([ref[p] for p in range(ref.shape[0])], slots, rows, tokens_per_chunk=slots.numel())
    want = moves.gather_layers([ref[p].reshape(ref.shape[1], bs * row) for p in range(ref.shape[0])], ids,
                               blocks_per_chunk=blocks_per_chunk) if k else out.cpu()
    return kv_d, out, ref, want


@pytest.mark.parametrize("row,bs", [(64, 16), (256, 16), (576, 4), (1552, 4), (2048, 16), (2064, 2), (1024, 1),
                                    (100, 8), (48, 2)])
def test_pair_matches_oracle(ops, row, bs):
    planes, nb = 6, 96
    kv, slots, ids, rows = _case(planes, nb, bs, row, tokens=200 if bs > 1 else 40, gathered=24, seed=row * 31 + bs)
    kv_d, out, ref, want = _run(ops, kv, slots, ids, rows, bs, row, blocks_per_chunk=4)
    assert _same(kv_d, ref)
    assert _same(out, want)


@pytest.mark.parametrize("row", [256, 2048])
def test_pair_decode_step_shapes(ops, row):
    """Decode steps with 1 and 8 KV heads: 256 token rows of 256 B / 2 KiB over
    64 planes and 16 spilled blocks of 4 / 32 KiB (one launch; two above
    32 MiB)."""
    planes, nb, bs = 64, 512, 16
    kv, slots, ids, rows = _case(planes, nb, bs, row, tokens=256, gathered=16, seed=5)
    kv_d, out, ref, want = _run(ops, kv, slots, ids, rows, bs, row, blocks_per_chunk=1)
    assert _same(kv_d, ref)
    assert _same(out, want)


@pytest.mark.parametrize("tokens,gathered", [(0, 12), (64, 0), (0, 0)])
def test_pair_with_an_empty_side(ops, tokens, gathered):
    kv, slots, ids, rows = _case(4, 64, 16, 256, tokens=max(tokens, 1), gathered=max(gathered, 1), seed=11)
    slots, ids = slots[:tokens], ids[:gathered]
    rows = rows[:, :, :tokens].contiguous() if tokens else torch.empty((0, 4, 1, 256), dtype=torch.uint8)
    kv_d, out, ref, want = _run(ops, kv, slots, ids, rows, 16, 256, blocks_per_chunk=1)
    assert _same(kv_d, ref)
    if gathered:
        assert _same(out, want)


def test_pair_bad_gather_id_raises(ops):
    kv, slots, ids, rows = _case(4, 64, 16, 256, tokens=32, gathered=4, seed=13)
    ids = ids.clone()
    ids[2] = 64  # one past the last block
    with pytest.raises(IndexError):
        _run(ops, kv, slots, ids, rows, 16, 256, blocks_per_chunk=1)
    ops.check_status(DEV)  # the error was consumed by the raise


@pytest.mark.parametrize("row,planes,per", [(256, 8, 4), (64, 8, 4), (2048, 8, 4), (2048, 64, 16)])
def test_pair_chain_with_inputs_ready(ops, row, planes, per):
    """A chain of paired launches with inputs_ready (each reads its indices and
    token rows while the previous one drains): launch k + 1's gather reads the
    blocks launch k's scatter just wrote, so its paged reads must wait; the
    bytes must equal the oracle's moves applied in order.  Groups of `per`
    blocks; 64 planes x 16 blocks of 2 KiB rows moves 64 MiB per launch
    (every CTA in both moves, the decode step with 8 KV heads)."""
    gen = torch.Generator().manual_seed(row)
    nb, bs, launches = 16 * per, 16, 8
    kv = torch.randint(0, 256, (planes, nb, bs, row), generator=gen, dtype=torch.uint8)
    groups = torch.randperm(nb, generator=gen)[: per * (launches + 1)].reshape(launches + 1, per)
    slots = [(g.reshape(-1, 1) * bs + torch.arange(bs).reshape(1, -1)).reshape(-1) for g in groups]
    rows = [torch.randint(0, 256, (1, planes, per * bs, row), generator=gen, dtype=torch.uint8)
            for _ in range(launches)]
    kv_d = kv.to(DEV)
    token_planes = [kv_d[p] for p in range(planes)]
    block_planes = [kv_d[p].reshape(nb, bs * row) for p in range(planes)]
    slots_d = [s.to(DEV) for s in slots]
    ids_d = [g.to(DEV) for g in groups]
    rows_d = [r.to(DEV) for r in rows]
    outs = [torch.empty((per, planes, 1, bs * row), dtype=torch.uint8, device=DEV) for _ in range(launches)]
    torch.cuda.synchronize()
    for k in range(launches):  # scatter into group k, gather group k (written by launch k - 1's scatter)
        ops.scatter_tokens_gather_layers(token_planes, slots_d[k], rows_d[k],
                                         block_planes, ids_d[k - 1] if k else ids_d[launches], outs[k],
                                         tokens_per_chunk=per * bs, blocks_per_chunk=1, inputs_ready=True)
    torch.cuda.synchronize()
    ops.check_status(DEV)
    ref = kv.clone()
    for k in range(launches):
        gid = groups[k - 1] if k else groups[launches]
        want = moves.gather_layers([ref[p].reshape(nb, bs * row) for p in range(planes)], gid, blocks_per_chunk=1)
        moves.scatter_tokens([ref[p] for p in range(planes)], slots[k], rows[k], tokens_per_chunk=per * bs)
        assert _same(outs[k], want), k
    assert _same(kv_d, ref)
