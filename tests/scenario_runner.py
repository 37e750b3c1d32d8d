"""Replays recorded reference scenarios (tests/golden/scenarios_u*.json) through
this repository's KVCacheAdapter and compares the full state after every op."""
from __future__ import annotations

import json
import pathlib

import torch

from kv_cache_adapter_b200 import InMemoryBlockStoreBackend, KVCacheAdapter

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"


def load_scenarios(name: str = "scenarios_u8.json") -> list[dict]:
    """scenarios_u8.json (8-bit slot meta) or scenarios_u16.json (recorded
    with KVCA_SLOT_META_BITS=16; replay those in a process with the same
    setting)."""
    return json.loads((GOLDEN / name).read_text())


def _flat(t: torch.Tensor | None):
    if t is None:
        return None
    return t.detach().cpu().reshape(t.shape[0], -1)


def run_and_compare(case: dict, device: torch.device, *, native_ext=None, backend_ops=None,
                    planned: bool | None = None, record: bool = True, host_tier: bool = False) -> None:
    """Replays a recorded reference scenario and compares results, errors and
    the full adapter / backend state after every step.  ``record=False`` runs
    the backend without recording device ids (the operation log is then not
    compared), which lets a device-resident store take the fused path."""
    spec = case["spec"]
    shape = tuple(spec["block_shape"])
    init = {int(k): torch.tensor(v, dtype=torch.float32, device=device).reshape(shape)
            for k, v in spec["initial"].items()}
    if init:
        backend = InMemoryBlockStoreBackend(init, num_logical_blocks=spec["num_logical"],
                                            record_device_ops=record, ops=backend_ops,
                                            host_tier=host_tier, device=device if host_tier else None)
    else:
        backend = InMemoryBlockStoreBackend(num_logical_blocks=spec["num_logical"],
                                            record_device_ops=record, ops=backend_ops,
                                            host_tier=host_tier, device=device if host_tier else None)
    ad = KVCacheAdapter(spec["num_actual"], spec["num_logical"],
                        torch.zeros((spec["num_actual"], *shape), dtype=torch.float32, device=device),
                        backend, native_ext=native_ext)
    if planned is not None:  # force the one-launch planners on or off
        assert ad._planned or not planned
        ad._planned = planned
    for i, step in enumerate(case["steps"]):
        where = f"case {spec['case']} step {i} {step['op']} {step['ids']}"
        ids = torch.tensor(step["ids"], dtype=torch.int64, device=device)
        result, error = None, None
        try:
            if step["op"] == "load":
                result = ad.load(ids).tolist()
            elif step["op"] == "save":
                data = torch.tensor(step["data"], dtype=torch.float32, device=device).reshape(len(step["ids"]), *shape)
                ad.save(ids, data)
            else:
                ad.release(ids)
        except Exception as exc:  # compared by type name with the reference's
            error = type(exc).__name__
        assert error == step["error"], f"{where}: error {error!r} != reference {step['error']!r}"
        assert result == step["result"], f"{where}: result {result} != reference {step['result']}"
        st = step["state"]
        assert ad._logical_to_physical.tolist() == st["l2p"], f"{where}: l2p"
        assert ad._physical_to_logical.tolist() == st["p2l"], f"{where}: p2l"
        assert ad._slot_meta.tolist() == st["slot_meta"], f"{where}: slot_meta"
        assert int(ad._search_start[0]) == st["search_start"], f"{where}: search_start"
        assert torch.equal(_flat(ad.actual_blocks), torch.tensor(st["actual_blocks"], dtype=torch.float32)), \
            f"{where}: actual_blocks"
        storage = backend._storage
        if st["storage"] is None:
            assert storage is None, f"{where}: storage"
        else:
            assert torch.equal(_flat(storage), torch.tensor(st["storage"], dtype=torch.float32)), f"{where}: storage"
        present = backend._present_mask
        got_present = None if present is None else present.int().cpu().tolist()
        assert got_present == st["present"], f"{where}: present mask"
        if record:
            assert [list(x) for x in backend.operation_log] == st["operation_log"], f"{where}: operation log"
