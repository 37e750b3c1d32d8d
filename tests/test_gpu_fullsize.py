"""GPU parity at the full sizes of the benchmark configurations.

Only full-size cases reach byte offsets past 2^31 within one chunk tensor and
the largest block tables, so every byte is compared here, not a sample:

* the Llama-3-70B KV-head shard (80 layers x K/V, 1 KV head, head_dim 128,
  block 16, bf16, 32,768 blocks = 21.47 GB of cache), gathered into 256-token
  chunks through a random block table and scattered back into a zeroed cache
  through another, block-granular and token-granular (slot_mapping =
  block x 16 + offset, adapter.py:1275-1285);
* the MLA latent cache of one GPU's layer range (8 of 61 layers, 576-wide
  rows, block 64, 128k tokens), bf16 and the fp8-e4m3 byte view;
* the decode append + gather mix with 8 KV heads over whole 16-step cycles,
  step by step against the same steps composed from the oracle.

The checker is the reference's own op: torch ``index_select`` on the device
(adapter.py:543) per plane, and the inverse property of the round trip for
the scatter (adapter.py:653-656).
"""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


@pytest.fixture(scope="module")
def ops():
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda as m

    return m


@pytest.fixture(autouse=True)
def _release_memory():
    yield
    torch.cuda.synchronize(DEV)
    torch.cuda.empty_cache()


def _bytes(t: torch.Tensor) -> torch.Tensor:
    return t.view(torch.uint8) if t.element_size() == 1 else t.view(torch.int16)


def _cache(layers: int, kv: int, blocks: int, block: int, heads: int, dim: int, dtype, seed: int):
    gen = torch.Generator(device=DEV).manual_seed(seed)
    shape = (layers, kv, blocks, block, heads, dim)
    if dtype == torch.float8_e4m3fn:
        c = torch.empty(shape, dtype=torch.uint8, device=DEV)
        c.random_(0, 256, generator=gen)
        return c.view(dtype)
    c = torch.empty(shape, dtype=dtype, device=DEV)
    c.normal_(generator=gen)
    return c


def _planes(cache: torch.Tensor) -> list[torch.Tensor]:
    L, K = cache.shape[0], cache.shape[1]
    return [cache[l, h] for h in range(K) for l in range(L)]  # K of every layer, then V


def _check_rows(chunks: torch.Tensor, planes, index: torch.Tensor, rows_per_block: bool) -> None:
    """chunks[:, p] against plane p's rows ``index`` (index_select on the device)."""
    n = index.numel()
    for p, plane in enumerate(planes):
        src = plane.reshape(plane.shape[0], -1) if rows_per_block else plane.reshape(plane.shape[0] * plane.shape[1], -1)
        want = _bytes(src).index_select(0, index)
        got = _bytes(chunks[:, p].reshape(n, -1))
        assert torch.equal(got, want), f"plane {p}"


def _slot_mapping(table: torch.Tensor, block_size: int) -> torch.Tensor:
    off = torch.arange(block_size, dtype=torch.int64, device=table.device)
    return (table.view(-1, 1) * block_size + off.view(1, -1)).reshape(-1)


def test_llama70b_shard_full_gather_scatter_blocks_and_tokens(ops):
    nb, cb = 32768, 16  # 16 x 32k tokens; 256-token chunks
    cache = _cache(80, 2, nb, 16, 1, 128, torch.bfloat16, 1234)
    planes = _planes(cache)
    assert cache.numel() * 2 == 21_474_836_480
    table = torch.randperm(nb, generator=torch.Generator().manual_seed(1)).to(DEV)
    chunks = ops.gather_layers(planes, table, blocks_per_chunk=cb, check=True)
    assert chunks.numel() * 2 > 2**34
    _check_rows(chunks, planes, table, rows_per_block=True)
    # scatter into a zeroed cache through another permutation: every block is
    # written once, so the result is the source permuted
    back = torch.zeros_like(cache)
    table2 = torch.randperm(nb, generator=torch.Generator().manual_seed(2)).to(DEV)
    ops.scatter_layers(_planes(back), table2, chunks, blocks_per_chunk=cb, check=True)
    inv = torch.empty_like(table2)
    inv[table2] = torch.arange(nb, device=DEV)
    # back[:, :, table2[r]] == cache[:, :, table[r]]  <=>  back == cache[:, :, table[inv]]
    for h in range(2):
        for l in range(80):
            assert torch.equal(_bytes(back[l, h]), _bytes(cache[l, h].index_select(0, table[inv]))), (l, h)
    del back, chunks
    torch.cuda.empty_cache()

    # token-granular: one 256-byte row per token and plane through a slot mapping
    mapping = _slot_mapping(table, 16)
    tok = ops.gather_tokens(planes, mapping, tokens_per_chunk=256, check=True)
    assert tok.shape == (nb * 16 // 256, 160, 256, 1, 128)
    _check_rows(tok, planes, mapping, rows_per_block=False)
    back = torch.zeros_like(cache)
    ops.scatter_tokens(_planes(back), _slot_mapping(table2, 16), tok, tokens_per_chunk=256, check=True)
    for h in range(2):
        for l in range(80):
            assert torch.equal(_bytes(back[l, h]), _bytes(cache[l, h].index_select(0, table[inv]))), (l, h)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float8_e4m3fn])
def test_mla_layer_range_full_gather_scatter(ops, dtype):
    nb, bs = 2048, 64  # 128k tokens, block 64
    cache = _cache(8, 1, nb, bs, 1, 576, dtype, 4321)
    planes = _planes(cache)
    table = torch.randperm(nb, generator=torch.Generator().manual_seed(3)).to(DEV)
    chunks = ops.gather_layers(planes, table, blocks_per_chunk=256 // bs, check=True)
    _check_rows(chunks, planes, table, rows_per_block=True)
    back = torch.zeros_like(cache)
    ops.scatter_layers(_planes(back), table, chunks, blocks_per_chunk=256 // bs, check=True)
    assert torch.equal(_bytes(back), _bytes(cache))
    # random half of the token slots, gathered and scattered as 576-wide rows
    gen = torch.Generator().manual_seed(4)
    mapping = torch.randperm(nb * bs, generator=gen)[: nb * bs // 2].to(DEV)
    tok = ops.gather_tokens(planes, mapping, tokens_per_chunk=256, check=True)
    _check_rows(tok, planes, mapping, rows_per_block=False)
    back.zero_()
    ops.scatter_tokens(_planes(back), mapping, tok, tokens_per_chunk=256, check=True)
    flat_b = _bytes(back).reshape(8, nb * bs, -1)
    flat_c = _bytes(cache).reshape(8, nb * bs, -1)
    assert torch.equal(flat_b[:, mapping], flat_c[:, mapping])
    untouched = torch.ones(nb * bs, dtype=torch.bool, device=DEV)
    untouched[mapping] = False
    assert int(flat_b[:, untouched].count_nonzero()) == 0


@pytest.mark.parametrize("one_launch", [False, True])
def test_decode_mix_eight_heads_cycles_match_oracle(ops, one_launch):
    """32 layers x K/V, 8 KV heads, head_dim 128, fp16, 256 sequences: 17 eager
    steps, then whole-cycle bookings with paired moves or one move_cycle launch
    per cycle (three cycles, a new token rows tensor per step), against the
    oracle composition on CPU (a 1,024-block pool, 4.3 GB)."""
    from oracle_ops import OracleOps
    from kv_cache_adapter_b200.workloads import DecodeMix

    cfg = dict(layers=32, heads=8, head_dim=128, block_size=16, num_blocks=1024, seqs=256, max_steps=120,
               dtype=torch.float16)
    gpu = DecodeMix(ops, DEV, **cfg)
    cpu = DecodeMix(OracleOps(), torch.device("cpu"), **cfg)
    cpu.kv.copy_(gpu.kv.cpu())
    gen = torch.Generator().manual_seed(77)
    rows = torch.randn((1, gpu.num_planes, gpu.seqs, *gpu.row_shape), generator=gen).to(torch.float16)
    rows_d = rows.to(DEV)
    for step in range(17):
        spill_g = gpu.step(rows_d, check=True)
        spill_c = cpu.step(rows)
        assert torch.equal(spill_g.cpu().view(torch.int16), spill_c.view(torch.int16)), step
    cycle_rows = [torch.randn((16, gpu.num_planes, gpu.seqs, *gpu.row_shape), generator=gen).to(torch.float16)
                  for _ in range(3)]
    gpu.start_cycles(one_launch=one_launch)
    gpu.run_cycle(cycle_rows[0].to(DEV))
    gpu.run_cycle(cycle_rows[1].to(DEV))
    gpu.stop_cycles(cycle_rows[2].to(DEV))
    spills = []
    for c in range(3):  # the three booked cycles
        for i in range(16):
            spills.append(cpu.step(cycle_rows[c][i:i + 1]).clone())
    if one_launch:  # the last cycle's victims, in step order
        last = torch.cat(spills[32:])
        assert torch.equal(gpu.spill[: last.shape[0]].cpu().view(torch.int16), last.view(torch.int16))
    torch.cuda.synchronize(DEV)
    ops.check_status(DEV)
    assert gpu.tokens == cpu.tokens and gpu.evictions == cpu.evictions > 0
    assert torch.equal(gpu.slot_meta.cpu(), cpu.slot_meta)
    assert torch.equal(gpu.l2p.cpu(), cpu.l2p) and torch.equal(gpu.p2l.cpu(), cpu.p2l)
    assert int(gpu.search_start[0]) == int(cpu.search_start[0])
    assert torch.equal(gpu.kv.cpu().view(torch.int16), cpu.kv.view(torch.int16))
