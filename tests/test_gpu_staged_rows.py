"""GPU parity for token-row moves through the C ABI, where the calls the
Python API never makes are possible: a last chunk shorter than the others,
chunks shorter than a tile and longer than several tiles, padding and
out-of-range ids in the same call, against the oracle's torch CPU indexing,
byte for byte.  Gathers of rows of 128 to 576 bytes take the staged mover
(shared-memory tiles filled by cp.async and written by one bulk store), the
others the stream mover.  A padded or refused row of a gather leaves its
chunk row as it was; of a scatter, its cache row."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from kv_cache_adapter_b200 import _lib

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


@pytest.fixture(scope="module")
def ops():
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda as m

    return m


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)


@pytest.mark.parametrize("row", [128, 144, 576, 1152, 1536])
@pytest.mark.parametrize("rpc,rows", [(256, 1000), (3, 50), (1000, 2500), (64, 64)])
def test_staged_gather_scatter_c_abi(ops, row, rpc, rows):
    rng = np.random.default_rng(row * 7 + rpc + rows)
    planes_n, nblk, bs = 3, 200, 16
    cache = torch.from_numpy(rng.integers(0, 256, (planes_n, nblk, bs, row), dtype=np.uint8)).to(DEV)
    mapping = torch.from_numpy(rng.permutation(nblk * bs)[:rows].astype(np.int64))
    mapping[rng.integers(0, rows, rows // 10)] = -1  # padding
    lib = _lib.load()
    table = ops.PlaneTable([cache[p] for p in range(planes_n)], 2)
    n_chunks = -(-rows // rpc)  # the last chunk may be short
    chunks = torch.from_numpy(rng.integers(0, 256, (n_chunks, planes_n, rpc, row), dtype=np.uint8)).to(DEV)
    before = chunks.clone()
    idx = mapping.to(DEV)
    st = torch.zeros(2, dtype=torch.int64, device=DEV)
    cd = _lib.ChunkDesc(chunks.data_ptr(), rpc, planes_n * rpc * row, row, rpc * row)
    pd = table.desc(idx)
    assert lib.kvca_gather(ctypes.byref(pd), ctypes.byref(cd), planes_n, rows, row, _lib.KVCA_FLAG_SKIP_NEGATIVE,
                           ctypes.c_void_p(st.data_ptr()), _stream()) == 0
    torch.cuda.synchronize(DEV)
    assert st.tolist() == [0, 0]
    flat = cache.view(planes_n, nblk * bs, row).cpu()
    got = chunks.cpu().permute(1, 0, 2, 3).reshape(planes_n, n_chunks * rpc, row)[:, :rows]
    old = before.cpu().permute(1, 0, 2, 3).reshape(planes_n, n_chunks * rpc, row)[:, :rows]
    live = mapping >= 0
    assert torch.equal(got[:, live], flat[:, mapping[live]])
    assert torch.equal(got[:, ~live], old[:, ~live])  # padding rows untouched
    tail = chunks.cpu().permute(1, 0, 2, 3).reshape(planes_n, n_chunks * rpc, row)[:, rows:]
    assert torch.equal(tail, before.cpu().permute(1, 0, 2, 3).reshape(planes_n, n_chunks * rpc, row)[:, rows:])

    # scatter new rows back through the same mapping: live rows land, padding rows are skipped
    src = torch.from_numpy(rng.integers(0, 256, (n_chunks, planes_n, rpc, row), dtype=np.uint8)).to(DEV)
    cache_before = cache.cpu()
    cs = _lib.ChunkDesc(src.data_ptr(), rpc, planes_n * rpc * row, row, rpc * row)
    assert lib.kvca_scatter(ctypes.byref(cs), ctypes.byref(pd), planes_n, rows, row, _lib.KVCA_FLAG_SKIP_NEGATIVE,
                            ctypes.c_void_p(st.data_ptr()), _stream()) == 0
    torch.cuda.synchronize(DEV)
    assert st.tolist() == [0, 0]
    want = cache_before.view(planes_n, nblk * bs, row).clone()
    rows_src = src.cpu().permute(1, 0, 2, 3).reshape(planes_n, n_chunks * rpc, row)[:, :rows]
    want[:, mapping[live]] = rows_src[:, live]
    assert torch.equal(cache.view(planes_n, nblk * bs, row).cpu(), want)


@pytest.mark.parametrize("row", [128, 576])
def test_staged_bad_ids_reported_and_skipped(ops, row):
    rng = np.random.default_rng(row)
    planes_n, nblk, bs, rows = 2, 50, 16, 512
    cache = torch.from_numpy(rng.integers(0, 256, (planes_n, nblk, bs, row), dtype=np.uint8)).to(DEV)
    table = ops.PlaneTable([cache[p] for p in range(planes_n)], 2)
    mapping = torch.from_numpy(rng.permutation(nblk * bs)[:rows].astype(np.int64))
    mapping[17] = nblk * bs + 5  # past the table
    mapping[300] = -3            # negative without the padding flag
    out = torch.zeros((rows // 256, planes_n, 256, row), dtype=torch.uint8, device=DEV)
    with pytest.raises(IndexError):
        ops.gather_tokens(table, mapping.to(DEV), out, tokens_per_chunk=256, check=True)
    # every other row moved; the refused ones kept their (zero) chunk bytes
    flat = cache.view(planes_n, nblk * bs, row).cpu()
    got = out.cpu().permute(1, 0, 2, 3).reshape(planes_n, rows, row)
    ok = torch.ones(rows, dtype=torch.bool)
    ok[[17, 300]] = False
    assert torch.equal(got[:, ok], flat[:, mapping[ok]])
    assert int(got[:, ~ok].count_nonzero()) == 0
