"""GPU: the adapter's device-store calls through a DeviceStoreSession
(kvca_session_load / kvca_session_save), against the oracle-driven adapter on
CPU, on whichever stream is current at each call: calls of one launch, whose
kernel writes its counts and a sequence number into pinned host memory for
the host to wait on, and calls above the one-launch size, which copy the
counts and wait for the stream; errors raised with the reference's types;
the session's work arrays growing with the largest request."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from kv_cache_adapter_b200 import _lib
from kv_cache_adapter_b200 import adapter as adapter_mod
from oracle_ops import OracleOps

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("shape", [(2, 64), (32, 1024)])  # 512 B (one launch) and 128 KiB rows
def test_session_calls_on_changing_streams_match_oracle_adapter(shape):
    num_actual, num_logical = 64, 300
    rng = np.random.default_rng(shape[1])
    init = {i: torch.full(shape, float(i)) for i in range(num_logical) if i % 13 != 4}
    cpu_ops = OracleOps()
    ref = adapter_mod.KVCacheAdapter(
        num_actual, num_logical, torch.zeros((num_actual, *shape)),
        adapter_mod.InMemoryBlockStoreBackend(dict(init), num_logical_blocks=num_logical, ops=cpu_ops),
        native_ext=cpu_ops)
    gpu = adapter_mod.KVCacheAdapter(
        num_actual, num_logical, torch.zeros((num_actual, *shape), device=DEV),
        adapter_mod.InMemoryBlockStoreBackend({k: v.to(DEV) for k, v in init.items()}, num_logical_blocks=num_logical))
    streams = [torch.cuda.current_stream(DEV), torch.cuda.Stream(DEV), torch.cuda.Stream(DEV)]
    pinned: list[int] = []
    for step in range(90):
        op = rng.choice(["load", "save", "release"], p=[0.45, 0.3, 0.25])
        k = int(rng.integers(1, 80 if step > 60 else 20))  # the last steps grow the work arrays
        ids = (np.asarray(pinned[:k], np.int64) if op == "release" and pinned
               else rng.integers(0, num_logical, k).astype(np.int64))
        if op == "release" and pinned:
            pinned = pinned[len(ids):]
        outs = []
        for ad, dev in ((ref, torch.device("cpu")), (gpu, DEV)):
            ctx = torch.cuda.stream(streams[step % 3]) if dev.type == "cuda" else torch.autograd.no_grad()
            with ctx:
                t = torch.from_numpy(ids).to(dev)
                try:
                    if op == "load":
                        outs.append(("ok", ad.load(t).tolist()))
                    elif op == "save":
                        data = torch.arange(len(ids) * shape[0] * shape[1], dtype=torch.float32)
                        ad.save(t, (data.reshape(len(ids), *shape) + 1000 * step).to(dev))
                        outs.append(("ok", None))
                    else:
                        ad.release(t)
                        outs.append(("ok", None))
                except Exception as exc:  # compared by type
                    outs.append((type(exc).__name__, None))
        assert outs[0] == outs[1], (step, op)
        if op == "load" and outs[0][0] == "ok":
            pinned.extend(ids.tolist())
        torch.cuda.synchronize(DEV)
        for name in ("_logical_to_physical", "_physical_to_logical", "_slot_meta", "_search_start"):
            assert torch.equal(getattr(gpu, name).cpu(), getattr(ref, name)), (step, op, name)
        assert torch.equal(gpu.actual_blocks.cpu(), ref.actual_blocks), (step, op)
        assert torch.equal(gpu.backend._storage.cpu(), ref.backend._storage), (step, op)
    assert gpu._session is not None and gpu._session.s.sequence > 0
    assert gpu._session.s.work_ids >= 79


def test_session_refuses_requests_above_its_work_arrays():
    backend = adapter_mod.InMemoryBlockStoreBackend(
        {i: torch.full((4,), float(i), device=DEV) for i in range(8)}, num_logical_blocks=8)
    ad = adapter_mod.KVCacheAdapter(4, 8, torch.zeros((4, 4), device=DEV), backend)
    ad.load(torch.tensor([1], device=DEV))
    sess = ad._session
    lib = _lib.load()
    ids = torch.arange(int(sess.s.work_ids) + 1, dtype=torch.int64, device=DEV) % 8
    out = torch.empty_like(ids)
    assert lib.kvca_session_load(sess.ref, ids.data_ptr(), ids.numel(), out.data_ptr()) == _lib.KVCA_ERR_BAD_ARGUMENT
    assert lib.kvca_session_load(sess.ref, ids.data_ptr(), -1, out.data_ptr()) == _lib.KVCA_ERR_BAD_ARGUMENT
    assert ad.load(torch.tensor([2, 1], device=DEV)).tolist() == [1, 0]  # the session still works
