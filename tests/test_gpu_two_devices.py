"""GPU: one process driving two devices.  The kernels that need more than
48 KB of dynamic shared memory (the bulk block mover, the staged token
gather, the cycle-booking kernel with its copy of the slot table) have that
limit raised per device, so the same calls must work on the second device
after the first one has run them.  Skipped with fewer than two devices."""
from __future__ import annotations

import pytest
import torch

from oracle import moves

pytestmark = pytest.mark.gpu

needs_two = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                               reason="needs two visible GPUs")


def _gathers_match(ops, dev: torch.device) -> None:
    gen = torch.Generator().manual_seed(dev.index + 7)
    # 4 KiB block rows: the bulk mover
    planes = [torch.randn((256, 16, 1, 128), generator=gen).to(torch.bfloat16) for _ in range(4)]
    ids = torch.randperm(256, generator=gen)[:128]
    planes_d = [p.to(dev) for p in planes]
    got = ops.gather_layers(planes_d, ids.to(dev), blocks_per_chunk=16, check=True)
    want = moves.gather_layers(planes, ids, blocks_per_chunk=16)
    assert torch.equal(got.cpu().view(torch.int16), want.view(torch.int16))
    # 256-byte token rows into dense chunks: the staged gather
    tokens = [p.reshape(256, 16, 128) for p in planes]
    tokens_d = [p.reshape(256, 16, 128) for p in planes_d]
    mapping = torch.randperm(256 * 16, generator=gen)[:1024]
    got = ops.gather_tokens(tokens_d, mapping.to(dev), tokens_per_chunk=256, check=True)
    want = moves.gather_tokens(tokens, mapping, tokens_per_chunk=256)
    assert torch.equal(got.cpu().view(torch.int16), want.view(torch.int16))


def _booking_matches_single_steps(dev: torch.device) -> None:
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda as ops
    from kv_cache_adapter_b200.workloads import DecodeMix

    # 256 sequences and 16,384 slots: staged state and table copy over 48 KB
    cfg = dict(layers=1, heads=1, head_dim=8, block_size=16, num_blocks=16384, seqs=256, max_steps=120)
    with torch.cuda.device(dev):
        ref = DecodeMix(ops, dev, **cfg)
        cyc = DecodeMix(ops, dev, **cfg)
        rows = torch.randn((1, ref.num_planes, ref.seqs, *ref.row_shape), dtype=torch.float16, device=dev)
        for _ in range(17):
            ref.step(rows)
            cyc.step(rows)
        cyc.start_cycles()
        cyc.run_cycle(rows)
        cyc.stop_cycles(rows)
        for _ in range(32):
            ref.step(rows)
        torch.cuda.synchronize(dev)
        ops.check_status(dev)
        for a, b in zip((ref.kv, ref.slot_meta, ref.l2p, ref.p2l, ref.search_start, ref.cur_block_dev),
                        (cyc.kv, cyc.slot_meta, cyc.l2p, cyc.p2l, cyc.search_start, cyc.cur_block_dev)):
            assert torch.equal(a.view(torch.uint8) if a.dtype != torch.int64 else a,
                               b.view(torch.uint8) if b.dtype != torch.int64 else b)


@needs_two
def test_large_shared_memory_kernels_on_both_devices():
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda as ops

    for index in (0, 1):
        dev = torch.device("cuda", index)
        torch.cuda.set_device(dev)
        _gathers_match(ops, dev)
        _booking_matches_single_steps(dev)
    torch.cuda.set_device(torch.device("cuda", 0))
