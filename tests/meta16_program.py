"""Runs KVCacheAdapter with 16-bit slot metadata (KVCA_SLOT_META_BITS=16, the
reference's adapter.py:23-26 mode: 8-bit pin and usage fields).

The width is read when the adapter module is imported, so the tests run this
file in a child process with the variable set:

    KVCA_SLOT_META_BITS=16 python tests/meta16_program.py cpu   # oracle op set only
    KVCA_SLOT_META_BITS=16 python tests/meta16_program.py gpu   # CUDA paths vs the oracle
    KVCA_SLOT_META_BITS=16 python tests/meta16_program.py golden      # reference scenarios, oracle op set
    KVCA_SLOT_META_BITS=16 python tests/meta16_program.py golden-gpu  # reference scenarios, CUDA paths

Exit status 0 when every check holds.
"""
from __future__ import annotations

import os
import pathlib
import sys

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
sys.path.insert(0, str(HERE))

import numpy as np  # noqa: E402
import torch  # noqa: E402

from oracle_ops import OracleOps  # noqa: E402
from kv_cache_adapter_b200 import adapter as adapter_mod  # noqa: E402


def _oracle_adapter(num_actual, num_logical, shape, init):
    ops = OracleOps()
    backend = adapter_mod.InMemoryBlockStoreBackend(dict(init), num_logical_blocks=num_logical, ops=ops)
    return adapter_mod.KVCacheAdapter(num_actual, num_logical, torch.zeros((num_actual, *shape)), backend,
                                      native_ext=ops)


def check_cpu() -> None:
    """Pins count past the 4-bit field (they wrap only at 256) and usage
    saturates at 255, through the oracle-driven adapter."""
    assert adapter_mod.SLOT_META_DTYPE == torch.uint16 and adapter_mod.PIN_COUNT_MAX == 255
    init = {i: torch.full((2,), float(i)) for i in range(8)}
    ad = _oracle_adapter(2, 8, (2,), init)
    for _ in range(20):
        assert ad.load(torch.tensor([3])).tolist() == [0]
    pins = adapter_mod._slot_meta_pin_counts(ad._slot_meta)
    usage = adapter_mod._slot_meta_usage_counts(ad._slot_meta)
    assert int(pins[0]) == 20 and int(usage[0]) == 20, (pins, usage)
    for _ in range(300):
        ad.load(torch.tensor([3]))
    usage = adapter_mod._slot_meta_usage_counts(ad._slot_meta)
    assert int(usage[0]) == 255  # saturated
    assert int(adapter_mod._slot_meta_pin_counts(ad._slot_meta)[0]) == 320 % 256


def check_gpu() -> None:
    """Random load / save / release programs: the CUDA adapter on each of its
    paths (device store, planner + backend calls, step by step) against the
    oracle-driven adapter, 16-bit metadata throughout."""
    dev = torch.device("cuda", 0)
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda

    for path in ("device_store", "planned", "stepwise"):
        rng = np.random.default_rng(16)
        num_actual, num_logical, max_batch = 48, 200, 40
        shape = (2, 3)
        init = {i: torch.full(shape, float(i)) for i in range(num_logical) if i % 11 != 3}
        ref = _oracle_adapter(num_actual, num_logical, shape, init)
        backend = adapter_mod.InMemoryBlockStoreBackend({k: v.to(dev) for k, v in init.items()},
                                                        num_logical_blocks=num_logical,
                                                        record_device_ops=path != "device_store")
        gpu = adapter_mod.KVCacheAdapter(num_actual, num_logical, torch.zeros((num_actual, *shape), device=dev),
                                         backend)
        gpu._planned = path != "stepwise"
        assert gpu._slot_meta.dtype == torch.uint16
        assert (gpu._device_store() is not None) == (path == "device_store")
        pinned: list[int] = []
        for step in range(80):
            op = rng.choice(["load", "save", "release"], p=[0.5, 0.25, 0.25])
            k = int(rng.integers(1, max_batch + 1))
            if op == "release" and pinned:
                ids = np.asarray(pinned[:k], np.int64)
                pinned = pinned[k:]
            else:
                ids = rng.integers(0, num_logical, k).astype(np.int64)
            outs = []
            for ad, d in ((ref, torch.device("cpu")), (gpu, dev)):
                t = torch.from_numpy(ids).to(d)
                try:
                    if op == "load":
                        outs.append(("ok", ad.load(t).tolist()))
                    elif op == "save":
                        data = torch.arange(k * 6, dtype=torch.float32).reshape(k, *shape) + 1000 * step
                        ad.save(t, data.to(d))
                        outs.append(("ok", None))
                    else:
                        ad.release(t)
                        outs.append(("ok", None))
                except Exception as exc:  # compared by type
                    outs.append((type(exc).__name__, None))
            assert outs[0] == outs[1], (path, step, op, outs)
            if op == "load" and outs[0][0] == "ok":
                pinned.extend(ids.tolist())
            for name in ("_logical_to_physical", "_physical_to_logical", "_slot_meta", "_search_start"):
                assert torch.equal(getattr(gpu, name).cpu(), getattr(ref, name)), (path, step, name)
            assert torch.equal(gpu.actual_blocks.cpu(), ref.actual_blocks), (path, step)
            assert torch.equal(backend._storage.cpu(), ref.backend._storage), (path, step)
        kv_cache_adapter_cuda.check_status(dev)


def check_golden() -> None:
    """The scenarios recorded from the reference in its 16-bit mode, through
    this repository's adapter driven by the oracle op set."""
    import scenario_runner

    cases = scenario_runner.load_scenarios("scenarios_u16.json")
    assert len(cases) == 30
    for case in cases:
        ops = OracleOps()
        scenario_runner.run_and_compare(case, torch.device("cpu"), native_ext=ops, backend_ops=ops)


def check_golden_gpu() -> None:
    """The same scenarios through the CUDA adapter on each of its paths, and
    against a pinned host store."""
    import scenario_runner
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda

    dev = torch.device("cuda", 0)
    for case in scenario_runner.load_scenarios("scenarios_u16.json"):
        for path in ("device_store", "planned", "stepwise"):
            scenario_runner.run_and_compare(case, dev, planned=path != "stepwise", record=path != "device_store")
        # the store in pinned host memory (the host tier's device-store path)
        scenario_runner.run_and_compare(case, dev, planned=True, record=False, host_tier=True)
    kv_cache_adapter_cuda.check_status(dev)


if __name__ == "__main__":
    if os.environ.get("KVCA_SLOT_META_BITS") != "16":
        sys.exit("run with KVCA_SLOT_META_BITS=16")
    {"cpu": check_cpu, "gpu": check_gpu, "golden": check_golden, "golden-gpu": check_golden_gpu}[sys.argv[1]]()
    print("meta16 ok:", sys.argv[1])
