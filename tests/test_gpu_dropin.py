"""GPU: the reference's own adapter.py driving this library (the drop-in).

``tests/golden/dropin_u8.json`` holds every call that the reference's
``KVCacheAdapter`` -- its own code, with INTEGRATION.md's Option B edits --
made to its CUDA extension while replaying recorded load / save / release
scenarios (``tests/golden/make_dropin.py``; those runs reproduced the
reference strict path's state after every step).  Here the same calls, in
the same order and with the same arguments, go to
``kv_cache_adapter_b200.kv_cache_adapter_cuda`` on CUDA tensors.  The
adapter's state (l2p, p2l, slot_meta, search_start, actual_blocks) lives on
the GPU and changes only through this library's ops, except for the rows the
reference's in-memory backend writes between calls, which are applied as it
wrote them.  Every call must give the recorded results (or the recorded
error type) and leave the recorded state.
"""
from __future__ import annotations

import json

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
DTYPES = {"int64": torch.int64, "uint8": torch.uint8, "bool": torch.bool, "float32": torch.float32,
          "int32": torch.int32, "uint16": torch.uint16}
META = ("l2p", "p2l", "slot_meta", "search_start")


@pytest.fixture(scope="module")
def ops():
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda as m

    return m


@pytest.fixture(scope="module")
def cases(golden_dir):
    return json.loads((golden_dir / "dropin_u8.json").read_text())


def _tensor(v: dict) -> torch.Tensor:
    return torch.tensor(v["t"], dtype=DTYPES[v["dtype"]]).reshape(v["shape"]).to(DEV)


def _same(got: torch.Tensor, want: dict) -> bool:
    return (str(got.dtype).replace("torch.", "") == want["dtype"] and list(got.shape) == want["shape"]
            and got.detach().cpu().reshape(-1).tolist() == want["t"])


@pytest.mark.parametrize("case", range(16))
def test_reference_adapter_calls_replayed_on_cuda(ops, cases, case):
    sc = cases[case]
    spec = sc["spec"]
    shape = (spec["num_actual"], *spec["block_shape"])
    first = sc["calls"][0]["before"]
    state = {
        "l2p": torch.tensor(first["l2p"], dtype=torch.int64, device=DEV),
        "p2l": torch.tensor(first["p2l"], dtype=torch.int64, device=DEV),
        "slot_meta": torch.tensor(first["slot_meta"], dtype=torch.uint8, device=DEV),
        "search_start": torch.tensor(first["search_start"], dtype=torch.int64, device=DEV),
        "actual_blocks": torch.zeros(shape, dtype=torch.float32, device=DEV),
    }
    for i, c in enumerate(sc["calls"]):
        where = f"case {spec['case']} call {i} {c['op']}"
        # rows the reference's backend wrote since the previous call (load_blocks)
        state["actual_blocks"].copy_(torch.tensor(c["before"]["actual_blocks"], dtype=torch.float32).reshape(shape))
        for k in META:  # metadata changes only through the ops replayed here
            assert state[k].cpu().tolist() == c["before"][k], f"{where}: {k} before"
        args = [state[a["state"]] if isinstance(a, dict) and "state" in a else
                _tensor(a) if isinstance(a, dict) else a for a in c["args"]]
        error, out = None, None
        try:
            out = getattr(ops, c["op"])(*args)
        except Exception as exc:
            error = type(exc).__name__
        torch.cuda.synchronize(DEV)
        assert error == c["error"], f"{where}: error {error!r}, reference adapter saw {c['error']!r}"
        if error is None and c["out"] is not None:
            if isinstance(c["out"], list):
                assert len(out) == len(c["out"]), where
                for j, (g, w) in enumerate(zip(out, c["out"])):
                    assert _same(g, w), f"{where}: result {j}"
            else:
                assert _same(out, c["out"]), f"{where}: result"
        for k, t in state.items():
            assert t.cpu().reshape(-1).tolist() == c["after"][k], f"{where}: {k} after"
