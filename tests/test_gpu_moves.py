"""GPU parity: the row mover (block and token gathers/scatters) against the
reference's torch CPU indexing (oracle/moves.py), byte for byte."""
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


def _bytes(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.uint8).numpy()


def _same_bytes(a: torch.Tensor, b: torch.Tensor) -> bool:
    return (tuple(a.shape) == tuple(b.shape) and a.element_size() == b.element_size()
            and np.array_equal(_bytes(a), _bytes(b)))


def _o(t):
    """Host tensors for the oracle: fp8 moves as its raw bytes (torch has no
    CPU indexing kernels for float8)."""
    if isinstance(t, (list, tuple)):
        return [_o(x) for x in t]
    return t.view(torch.uint8) if t.dtype == torch.float8_e4m3fn else t


def _rand(shape, dtype, gen):
    if dtype in (torch.uint8, torch.float8_e4m3fn):
        return torch.randint(0, 256, shape, generator=gen, dtype=torch.uint8).view(dtype)
    if dtype == torch.int16:
        return torch.randint(-30000, 30000, shape, generator=gen, dtype=torch.int16)
    return torch.randn(shape, generator=gen, dtype=torch.float32).to(dtype)


BLOCK_CASES = [
    ((2,), torch.float32),           # 8-byte rows (reference unit tests)
    ((3,), torch.float16),           # 6-byte rows: 2-byte accesses
    ((5,), torch.uint8),             # 5-byte rows: byte accesses
    ((16, 8, 128), torch.float16),   # 32 KiB: one layer's K block of the Llama-3-8B cache
    ((16, 1, 128), torch.bfloat16),  # 4 KiB: one KV head of the Llama-3-70B cache
    ((64, 576), torch.bfloat16),     # MLA latent block, 72 KiB
    ((64, 576), torch.float8_e4m3fn),
    ((2, 16, 4, 8), torch.float16),  # merged K/V block
    ((7, 3), torch.float32),
]


@pytest.mark.parametrize("block,dtype", BLOCK_CASES)
def test_gather_scatter_copy_blocks(ops, block, dtype):
    gen = torch.Generator().manual_seed(1234)
    m = 37
    cache_h = _rand((m, *block), dtype, gen)
    cache_d = cache_h.to(DEV)
    for k in (0, 1, 5, 37, 100):
        ids_h = torch.randint(0, m, (k,), generator=gen)  # duplicates allowed for a gather
        got = ops.gather_blocks(cache_d, ids_h.to(DEV))
        assert _same_bytes(got, moves.gather_blocks(_o(cache_h), ids_h))
    # scatter with unique slots
    ids_h = torch.randperm(m, generator=gen)[:23]
    data_h = _rand((23, *block), dtype, gen)
    want = _o(cache_h.clone())
    moves.scatter_blocks(want, ids_h, _o(data_h))
    ops.scatter_blocks(cache_d, ids_h.to(DEV), data_h.to(DEV))
    assert _same_bytes(cache_d, want)
    # fused paged -> paged copy (backend load path)
    store_h = _rand((50, *block), dtype, gen)
    src_ids = torch.randint(0, 50, (19,), generator=gen)
    dst_ids = torch.randperm(m, generator=gen)[:19]
    moves.copy_blocks(_o(store_h), src_ids, want, dst_ids)
    ops.copy_blocks(store_h.to(DEV), src_ids.to(DEV), cache_d, dst_ids.to(DEV))
    assert _same_bytes(cache_d, want)


@pytest.mark.parametrize("cb", [None, 1, 4, 16])
def test_gather_scatter_layers(ops, cb):
    gen = torch.Generator().manual_seed(7 + (cb or 0))
    planes_h = [_rand((40, 16, 2, 64), torch.bfloat16, gen) for _ in range(6)]
    planes_d = [p.to(DEV) for p in planes_h]
    ids_h = torch.randperm(40, generator=gen)[:32]
    got = ops.gather_layers(planes_d, ids_h.to(DEV), blocks_per_chunk=cb)
    want = moves.gather_layers(planes_h, ids_h, blocks_per_chunk=cb)
    assert _same_bytes(got, want)
    fresh_h = [torch.zeros_like(p) for p in planes_h]
    fresh_d = [p.to(DEV) for p in fresh_h]
    moves.scatter_layers(fresh_h, ids_h, want, blocks_per_chunk=cb)
    ops.scatter_layers(fresh_d, ids_h.to(DEV), got, blocks_per_chunk=cb)
    for a, b in zip(fresh_d, fresh_h):
        assert _same_bytes(a, b)


def test_layers_on_strided_planes(ops):
    """Planes that are views of one vLLM-style (L, 2, num_blocks, ...) tensor."""
    gen = torch.Generator().manual_seed(11)
    kv = _rand((4, 2, 30, 16, 1, 128), torch.float16, gen)
    kv_d = kv.to(DEV)
    planes_h = [kv[l, s] for l in range(4) for s in range(2)]
    planes_d = [kv_d[l, s] for l in range(4) for s in range(2)]
    ids = torch.randperm(30, generator=gen)[:16]
    assert _same_bytes(ops.gather_layers(planes_d, ids.to(DEV), blocks_per_chunk=16),
                       moves.gather_layers(planes_h, ids, blocks_per_chunk=16))


TOKEN_CASES = [
    ((16, 8, 128), torch.float16, 16),   # reshape-and-cache rows, 2 KiB
    ((16, 1, 128), torch.bfloat16, 16),  # 256-byte rows (one head)
    ((64, 576), torch.bfloat16, 64),     # MLA latent rows, 1152 B
    ((64, 576), torch.float8_e4m3fn, 64),  # fp8 byte view, 576 B
    ((4, 3), torch.float32, 4),          # 12-byte rows
]


@pytest.mark.parametrize("block,dtype,bs", TOKEN_CASES)
def test_gather_scatter_tokens(ops, block, dtype, bs):
    gen = torch.Generator().manual_seed(bs + block[-1])
    nblk = 23
    planes_h = [_rand((nblk, *block), dtype, gen) for _ in range(3)]
    planes_d = [p.to(DEV) for p in planes_h]
    t = 48
    mapping = torch.randperm(nblk * bs, generator=gen)[:t]
    mapping[torch.randperm(t, generator=gen)[:5]] = -1  # padding tokens
    out = torch.zeros((3, 3, 16, *block[1:]), dtype=dtype, device=DEV)
    ops.gather_tokens(planes_d, mapping.to(DEV), out, tokens_per_chunk=16)
    assert _same_bytes(out, moves.gather_tokens(_o(planes_h), mapping, tokens_per_chunk=16))
    src_h = _rand((3, 3, 16, *block[1:]), dtype, gen)
    planes_o = _o(planes_h)
    moves.scatter_tokens(planes_o, mapping, _o(src_h), tokens_per_chunk=16)
    ops.scatter_tokens(planes_d, mapping.to(DEV), src_h.to(DEV), tokens_per_chunk=16)
    for a, b in zip(planes_d, planes_o):
        assert _same_bytes(a, b)


@pytest.mark.parametrize("shape", [(16, 2, 4, 32), (2, 16, 4, 32)])
def test_tokens_on_merged_kv_layout(ops, shape):
    """slot_mapping transfer into a merged (bs,2,H,D) / (2,bs,H,D) cache
    (adapter.py:1200-1243 with the mapping of adapter.py:1275-1285)."""
    from kv_cache_adapter_b200.adapter import _MergedKVBlockLayout

    layout = _MergedKVBlockLayout.detect(shape)
    gen = torch.Generator().manual_seed(3)
    cache_h = _rand((12, *shape), torch.float16, gen)
    cache_d = cache_h.to(DEV)
    slots = torch.tensor([5, 0, 11], dtype=torch.int64)
    mapping = layout.physical_slot_mapping(slots)
    planes_h = [p.reshape(12, layout.block_size, layout.hidden_dim) for p in layout.token_planes(cache_h)]
    planes_d = layout.token_planes(cache_d)
    got = ops.gather_tokens(planes_d, mapping.to(DEV), tokens_per_chunk=layout.block_size)
    assert _same_bytes(got, moves.gather_tokens(planes_h, mapping, tokens_per_chunk=layout.block_size))
    # the gathered chunk of one block is that block's (2, bs, hidden) content
    for i, s in enumerate(slots.tolist()):
        kv = cache_h[s].reshape(layout.transfer_shape)
        k_rows = kv[:, 0] if layout.token_major else kv[0]
        assert _same_bytes(got[i, 0].cpu(), k_rows)
    fresh_d = torch.zeros_like(cache_d)
    ops.scatter_tokens(layout.token_planes(fresh_d), mapping.to(DEV), got, tokens_per_chunk=layout.block_size)
    for s in slots.tolist():
        assert _same_bytes(fresh_d[s], cache_h[s])


def test_out_of_range_rows_raise_and_are_skipped(ops):
    cache = torch.arange(40, dtype=torch.float32, device=DEV).reshape(10, 4)
    with pytest.raises(IndexError):
        ops.gather_blocks(cache, torch.tensor([1, 10], device=DEV))
    with pytest.raises(IndexError):
        ops.gather_blocks(cache, torch.tensor([-1], device=DEV))
    before = cache.clone()
    with pytest.raises(IndexError):
        ops.scatter_blocks(cache, torch.tensor([3, 12], device=DEV), torch.ones((2, 4), device=DEV))
    # the valid row was written, the bad one skipped; nothing outside the table
    assert torch.equal(cache[3], torch.ones(4, device=DEV))
    mask = torch.ones(10, dtype=torch.bool)
    mask[3] = False
    assert torch.equal(cache[mask.to(DEV)], before[mask.to(DEV)])
    planes = [cache.reshape(5, 2, 4)]
    with pytest.raises(IndexError):
        ops.gather_tokens(planes, torch.tensor([0, 10], device=DEV))
    ops.gather_tokens(planes, torch.tensor([0, -1], device=DEV))  # padding is fine


def test_argument_checks(ops):
    cache = torch.zeros((4, 8), dtype=torch.float16, device=DEV)
    with pytest.raises(TypeError):
        ops.gather_blocks(cache, torch.tensor([0], dtype=torch.int32, device=DEV))
    with pytest.raises(ValueError):
        ops.gather_blocks(cache, torch.tensor([0]))  # ids on the host
    with pytest.raises(ValueError):
        ops.scatter_blocks(cache, torch.tensor([0], device=DEV), torch.zeros((1, 8), device=DEV))  # dtype
    with pytest.raises(ValueError):
        ops.gather_layers([cache, cache[:2]], torch.tensor([0], device=DEV))
    with pytest.raises(ValueError):
        ops.gather_layers([cache.t()], torch.tensor([0], device=DEV))  # row not contiguous
    with pytest.raises(ValueError):
        ops.gather_layers([cache], torch.tensor([0, 1, 2], device=DEV), blocks_per_chunk=2)


def test_llama8b_cache_round_trip_full_size(ops):
    """32 layers x K/V, 8 KV heads, head_dim 128, block 16, fp16, 1024 blocks
    per layer (2 GiB): gather every block through a seeded permutation into
    256-token chunks, scatter back through the same table into an empty cache,
    and compare every byte; two planes are also checked against index_select."""
    L, nblk = 32, 1024
    gen = torch.Generator(device=DEV).manual_seed(1234)
    planes = [torch.randn((nblk, 16, 8, 128), generator=gen, device=DEV, dtype=torch.float16)
              for _ in range(2 * L)]
    perm = torch.randperm(nblk, generator=torch.Generator().manual_seed(1234))
    chunks = ops.gather_layers(planes, perm.to(DEV), blocks_per_chunk=16)
    for p in (0, 2 * L - 1):
        want = moves.gather_layers([planes[p].cpu()], perm, blocks_per_chunk=16)
        assert _same_bytes(chunks[:, p:p + 1], want)
    fresh = [torch.empty_like(p).zero_() for p in planes]
    ops.scatter_layers(fresh, perm.to(DEV), chunks, blocks_per_chunk=16)
    for a, b in zip(fresh, planes):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))
