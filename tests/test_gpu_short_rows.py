"""GPU parity for rows under 4 KiB in 16-byte vectors, which take the
small-row mover (rows under 128 bytes: up to 8 lanes and four rows per lane
group and iteration), the warp-cooperative stream mover (128 bytes to
1.5 KiB: a warp's 32 x 9 vector slots tile a batch of rows) or the SIMT
mover (past 1.5 KiB), against the oracle's torch CPU indexing, byte for
byte: row widths from 16 bytes to just under 4 KiB, plane counts that make
one iteration's rows straddle tokens, work ranges that end inside a batch,
chunks shorter than a batch, padding tokens, out-of-range ids, and
block-granular moves of short blocks."""
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


def _rand_bytes(shape, gen) -> torch.Tensor:
    return torch.randint(0, 256, shape, generator=gen, dtype=torch.uint8)


ROW_BYTES = [16, 32, 48, 64, 112, 128, 144, 240, 256, 272, 512, 576, 1040, 1152, 1536, 1552, 2048, 2064, 3072, 4080]


@pytest.mark.parametrize("row", ROW_BYTES)
@pytest.mark.parametrize("planes", [1, 3, 7])
def test_token_gather_scatter_short_rows(ops, row, planes):
    gen = torch.Generator().manual_seed(row * 31 + planes)
    nblk, bs = 29, 16
    caches_h = [_rand_bytes((nblk, bs, row), gen) for _ in range(planes)]
    caches_d = [c.to(DEV) for c in caches_h]
    for t in (1, 2, 5, 61, 300):
        tpc = t if t < 61 else (61 if t == 61 else 100)
        mapping = torch.randperm(nblk * bs, generator=gen)[:t]
        if t > 4:
            mapping[torch.randperm(t, generator=gen)[: t // 5]] = -1
        out = torch.zeros((t // tpc, planes, tpc, row), dtype=torch.uint8, device=DEV)
        ops.gather_tokens(caches_d, mapping.to(DEV), out, tokens_per_chunk=tpc)
        assert _same(out, moves.gather_tokens(caches_h, mapping, tokens_per_chunk=tpc)), t
        src_h = _rand_bytes((t // tpc, planes, tpc, row), gen)
        moves.scatter_tokens(caches_h, mapping, src_h, tokens_per_chunk=tpc)
        ops.scatter_tokens(caches_d, mapping.to(DEV), src_h.to(DEV), tokens_per_chunk=tpc)
        for a, b in zip(caches_d, caches_h):
            assert _same(a, b), t


@pytest.mark.parametrize("row", [128, 256, 576, 1152])
@pytest.mark.parametrize("tpc,t", [(1, 7), (3, 60), (7, 301), (17, 34), (256, 512)])
def test_token_chunk_sizes_short_rows(ops, row, tpc, t):
    """Chunk lengths below, at and above the rows one warp moves per batch
    (18 rows of 256 B, 8 of 576 B, 4 of 1,152 B), so the chunk position
    carries across chunks inside a batch, and row counts below a batch, so
    the row position wraps into the next plane more than once."""
    gen = torch.Generator().manual_seed(row + 7 * tpc + t)
    planes = 5
    nblk, bs = 40, 16
    caches_h = [_rand_bytes((nblk, bs, row), gen) for _ in range(planes)]
    caches_d = [c.to(DEV) for c in caches_h]
    table = torch.randperm(nblk, generator=gen)
    mapping = (table.view(-1, 1) * bs + torch.arange(bs).view(1, -1)).reshape(-1)[:t].clone()
    if t > 10:
        mapping[torch.randperm(t, generator=gen)[: t // 9]] = -1
    out = torch.zeros((t // tpc, planes, tpc, row), dtype=torch.uint8, device=DEV)
    ops.gather_tokens(caches_d, mapping.to(DEV), out, tokens_per_chunk=tpc)
    assert _same(out, moves.gather_tokens(caches_h, mapping, tokens_per_chunk=tpc))
    src_h = _rand_bytes((t // tpc, planes, tpc, row), gen)
    moves.scatter_tokens(caches_h, mapping, src_h, tokens_per_chunk=tpc)
    ops.scatter_tokens(caches_d, mapping.to(DEV), src_h.to(DEV), tokens_per_chunk=tpc)
    for a, b in zip(caches_d, caches_h):
        assert _same(a, b)


@pytest.mark.parametrize("row", [32, 144, 256, 576, 1536])
def test_token_copy_short_rows(ops, row):
    gen = torch.Generator().manual_seed(row)
    src_h = [_rand_bytes((13, 8, row), gen) for _ in range(5)]
    dst_h = [_rand_bytes((21, 4, row), gen) for _ in range(5)]
    dst_d = [d.to(DEV) for d in dst_h]
    t = 77
    src_map = torch.randint(0, 13 * 8, (t,), generator=gen)
    dst_map = torch.randperm(21 * 4, generator=gen)[:t]
    src_map[3] = -1
    dst_map[40] = -1
    ops.copy_tokens([s.to(DEV) for s in src_h], src_map.to(DEV), dst_d, dst_map.to(DEV))
    keep = (src_map >= 0) & (dst_map >= 0)
    rows = moves.gather_tokens(src_h, src_map[keep])
    moves.scatter_tokens(dst_h, dst_map[keep], rows)
    for a, b in zip(dst_d, dst_h):
        assert _same(a, b)


@pytest.mark.parametrize("shape,dtype", [((128,), torch.float16), ((4, 16), torch.bfloat16),
                                         ((3, 16), torch.float32), ((16,), torch.uint8),
                                         ((2, 4, 32), torch.float16), ((9, 64), torch.uint8),
                                         ((16, 24), torch.float32)])
def test_block_moves_short_rows(ops, shape, dtype):
    """Whole blocks of 16 bytes to 1.5 KiB (block-granular gather / scatter /
    fused copy, the backend's index_select + index_copy_)."""
    gen = torch.Generator().manual_seed(sum(shape))
    m = 300
    cache_h = _rand_bytes((m, *shape[:-1], shape[-1] * torch.empty((), dtype=dtype).element_size()), gen).view(dtype)
    cache_d = cache_h.to(DEV)
    for k in (1, 3, 4, 5, 255):
        ids = torch.randint(0, m, (k,), generator=gen)
        assert _same(ops.gather_blocks(cache_d, ids.to(DEV)), moves.gather_blocks(cache_h, ids))
    ids = torch.randperm(m, generator=gen)[:203]
    data = _rand_bytes((203, *cache_h.shape[1:-1], cache_h.shape[-1] * cache_h.element_size()), gen).view(dtype)
    moves.scatter_blocks(cache_h, ids, data)
    ops.scatter_blocks(cache_d, ids.to(DEV), data.to(DEV))
    assert _same(cache_d, cache_h)
    store_h = _rand_bytes(tuple(cache_h.shape[:-1]) + (cache_h.shape[-1] * cache_h.element_size(),), gen).view(dtype)
    src = torch.randint(0, m, (97,), generator=gen)
    dst = torch.randperm(m, generator=gen)[:97]
    moves.copy_blocks(store_h, src, cache_h, dst)
    ops.copy_blocks(store_h.to(DEV), src.to(DEV), cache_d, dst.to(DEV))
    assert _same(cache_d, cache_h)


@pytest.mark.parametrize("cols", [16, 64, 144])  # int32 rows of 64 B (small mover), 256 B and 576 B (stream)
def test_short_rows_out_of_range_raise_and_skip(ops, cols):
    cache = torch.arange(64 * cols, dtype=torch.int32, device=DEV).reshape(64, cols)
    before = cache.clone()
    with pytest.raises(IndexError):
        ops.scatter_blocks(cache, torch.tensor([3, 64, 5], device=DEV), torch.ones((3, cols), dtype=torch.int32, device=DEV))
    want = before.clone()
    want[3] = 1
    want[5] = 1
    assert torch.equal(cache, want)
    planes = [cache.reshape(16, 4, cols), cache.reshape(16, 4, cols)]
    with pytest.raises(IndexError):
        ops.gather_tokens(planes, torch.tensor([0, 1, 2, 3, 64], device=DEV))
    with pytest.raises(IndexError):
        ops.scatter_tokens(planes, torch.tensor([0, 64], device=DEV),
                           torch.zeros((1, 2, 2, cols), dtype=torch.int32, device=DEV), tokens_per_chunk=2)
    assert int(cache[0].abs().sum()) == 0  # the valid token was written, the bad one skipped
    got = torch.full((1, 2, 5, cols), -7, dtype=torch.int32, device=DEV)
    ops.gather_tokens(planes, torch.tensor([0, -1, 63, -1, 7], device=DEV), got)
    for p in range(2):
        assert torch.equal(got[0, p, 2], planes[p][15, 3]) and torch.equal(got[0, p, 4], planes[p][1, 3])
        assert bool((got[0, p, 1] == -7).all()) and bool((got[0, p, 3] == -7).all())  # padding untouched


@pytest.mark.parametrize("row,P,nblk,bs", [(128, 64, 4096, 16), (288, 8, 4096, 64)])
def test_short_rows_large_random_round_trip(ops, row, P, nblk, bs):
    """256-byte rows over 64 planes (one KV head of a 70B-shaped cache, fp16)
    and 576-byte rows over 8 planes (an fp8 MLA latent), half of all token
    slots through a random slot mapping: gather, scatter into zeroed planes,
    gather again; three planes checked byte for byte against the oracle, all
    of them by the round trip on the device."""
    gen = torch.Generator().manual_seed(5 + row)
    base = torch.randint(-30000, 30000, (P, nblk, bs, row), generator=gen, dtype=torch.int16).to(DEV)
    caches = [base[p] for p in range(P)]
    t = nblk * bs // 2
    mapping_h = torch.randperm(nblk * bs, generator=gen)[:t]
    mapping = mapping_h.to(DEV)
    chunks = ops.gather_tokens(caches, mapping, tokens_per_chunk=256)
    for p in (0, P // 3, P - 1):
        want = moves.gather_tokens([base[p].cpu()], mapping_h, tokens_per_chunk=256)
        assert _same(chunks[:, p:p + 1], want)
    fresh = torch.zeros_like(base)
    ops.scatter_tokens([fresh[p] for p in range(P)], mapping, chunks, tokens_per_chunk=256)
    flat = mapping.view(-1)
    assert torch.equal(fresh.view(P, -1, row)[:, flat], base.view(P, -1, row)[:, flat])
    untouched = torch.ones(nblk * bs, dtype=torch.bool, device=DEV)
    untouched[flat] = False
    assert int(fresh.view(P, -1, row)[:, untouched].abs().sum()) == 0
    again = ops.gather_tokens([fresh[p] for p in range(P)], mapping, tokens_per_chunk=256)
    assert torch.equal(again, chunks)
