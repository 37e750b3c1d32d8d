"""Generate dropin_u8.json: the calls the reference's own adapter.py makes to
its CUDA extension, with this library's module dropped in (Option B of
INTEGRATION.md), recorded on CPU with the oracle as the op set.

Usage (in a container where the reference project is mounted):

    python tests/golden/make_dropin.py --reference <reference project dir>

(or with the directory in KVCA_REFERENCE_DIR).  A scratch copy of the
reference gets the Option B edits (tests/dropin_reference.py); its
KVCacheAdapter and InMemoryBlockStoreBackend replay the first recorded
scenarios of scenarios_u8.json on their CUDA branch, and every step must end
in the state the reference's strict path recorded.  Each native call is
written with its arguments (adapter state tensors by name), its results or
error, and the adapter state before and after it, so that
tests/test_gpu_dropin.py can make the same calls on a GPU, where the
reference sources are absent.  Nothing of the reference is copied into this
repository.
"""
from __future__ import annotations

import argparse
import json
import os
import pathlib
import sys
import tempfile

HERE = pathlib.Path(__file__).resolve().parent
TESTS = HERE.parent
REPO = TESTS.parent
for p in (str(REPO), str(TESTS)):
    if p not in sys.path:
        sys.path.insert(0, p)

from dropin_reference import Recorder, import_patched_reference, make_adapter, run_step  # noqa: E402
from oracle_ops import OracleOps  # noqa: E402

SCENARIOS = 16


def record(reference: pathlib.Path, count: int = SCENARIOS) -> list[dict]:
    cases = json.loads((HERE / "scenarios_u8.json").read_text())[:count]
    out = []
    with tempfile.TemporaryDirectory() as tmp:
        ref = import_patched_reference(reference, pathlib.Path(tmp))
        for case in cases:
            spec = case["spec"]
            rec = Recorder(OracleOps())
            ad, backend = make_adapter(ref, spec, rec)
            rec.adapter = ad
            for i, step in enumerate(case["steps"]):
                result, error = run_step(ad, step, tuple(spec["block_shape"]))
                st = step["state"]
                where = f"case {spec['case']} step {i}"
                assert (result, error) == (step["result"], step["error"]), where
                assert ad._logical_to_physical.tolist() == st["l2p"], where
                assert ad._physical_to_logical.tolist() == st["p2l"], where
                assert ad._slot_meta.tolist() == st["slot_meta"], where
                assert int(ad._search_start[0]) == st["search_start"], where
                assert ad.actual_blocks.reshape(ad.actual_blocks.shape[0], -1).tolist() == st["actual_blocks"], where
            out.append({"spec": spec, "calls": rec.calls})
    return out


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--reference", default=os.environ.get("KVCA_REFERENCE_DIR"))
    ap.add_argument("--out", default=str(HERE / "dropin_u8.json"))
    args = ap.parse_args()
    if not args.reference:
        ap.error("give the reference project's directory (--reference or KVCA_REFERENCE_DIR)")
    cases = record(pathlib.Path(args.reference))
    pathlib.Path(args.out).write_text(json.dumps(cases, separators=(",", ":")) + "\n")
    print(f"{args.out}: {len(cases)} scenarios, {sum(len(c['calls']) for c in cases)} native calls")


if __name__ == "__main__":
    main()
