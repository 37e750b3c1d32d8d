"""CPU: the reference's own adapter.py with this library dropped in (Option B
of INTEGRATION.md), where the reference project is present.

* The reference's loader (``_load_cuda_extension_module``,
  adapter.py:1347-1367) finds this library's module as its sibling
  ``kv_cache_adapter_cuda`` and gets every op its CUDA branch calls.
* The reference's ``KVCacheAdapter`` and ``InMemoryBlockStoreBackend``, on
  their CUDA branch with the packed slot-meta op set (computed here by the
  oracle, which the GPU tests hold the CUDA module to), reproduce the state
  the reference's strict path recorded after every step of all 60 scenarios.
* The committed call transcript that the GPU replays
  (``tests/golden/dropin_u8.json``) is what such a run records today.
"""
from __future__ import annotations

import json
import pathlib

import pytest

from dropin_reference import Recorder, import_patched_reference, make_adapter, run_step
from oracle import build_ref
from oracle_ops import OracleOps
from scenario_runner import load_scenarios

REFERENCE = build_ref.reference_dir()
pytestmark = pytest.mark.skipif(REFERENCE is None, reason="reference project not present")


@pytest.fixture(scope="module")
def ref(tmp_path_factory):
    return import_patched_reference(REFERENCE, tmp_path_factory.mktemp("reference"))


def test_reference_loader_finds_this_library(ref):
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda

    mod = ref.adapter._load_cuda_extension_module()
    assert mod is not None
    for name in Recorder.OPS:
        assert getattr(mod, name) is getattr(kv_cache_adapter_cuda, name), name


@pytest.mark.parametrize("case", range(60))
def test_reference_adapter_on_the_packed_ops_reproduces_recorded_states(ref, case):
    sc = load_scenarios()[case]
    spec = sc["spec"]
    ad, backend = make_adapter(ref, spec, OracleOps())
    for i, step in enumerate(sc["steps"]):
        where = f"case {case} step {i} {step['op']}"
        result, error = run_step(ad, step, tuple(spec["block_shape"]))
        assert (result, error) == (step["result"], step["error"]), where
        st = step["state"]
        assert ad._logical_to_physical.tolist() == st["l2p"], where
        assert ad._physical_to_logical.tolist() == st["p2l"], where
        assert ad._slot_meta.tolist() == st["slot_meta"], where
        assert int(ad._search_start[0]) == st["search_start"], where
        assert ad.actual_blocks.reshape(ad.actual_blocks.shape[0], -1).tolist() == st["actual_blocks"], where
        assert [list(x) for x in backend.operation_log] == st["operation_log"], where


def test_committed_transcript_is_current(golden_dir, ref):
    import importlib.util

    spec = importlib.util.spec_from_file_location("make_dropin", golden_dir / "make_dropin.py")
    make_dropin = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(make_dropin)
    fresh = make_dropin.record(REFERENCE)
    committed = json.loads((golden_dir / "dropin_u8.json").read_text())
    assert json.loads(json.dumps(fresh)) == committed
