"""Generate the golden fixtures in this directory by running the reference.

Usage (in a container where the reference project is mounted):

    python tests/golden/make_golden.py --reference <reference project dir>

(or with the directory in the KVCA_REFERENCE_DIR environment variable).

The reference package is copied to a scratch directory under the name
``kv_cache_adapter`` and imported from there; nothing of it is copied into
this repository.  CPU tensors select the reference's strict (pure PyTorch)
path, which is the normative semantics for slot metadata and the clock sweep.

Fixtures written (JSON, small):
  * kat_metadata.json   - the six known-answer tests of the reference
                          (test_adapter_npu_kernels.py:42-194), each re-run
                          through the strict path here and checked before
                          writing;
  * pop_u8.json         - seeded random clock-sweep cases (8-bit slot meta);
  * scenarios_u8.json   - seeded random load/save/release sequences through
                          KVCacheAdapter + InMemoryBlockStoreBackend, with
                          the full adapter and backend state after every op;
  * clock_stream.json   - small clock streams (pop, refill, Zipf re-access);
  * layout.json         - _MergedKVBlockLayout shapes and
                          _physical_slot_mapping outputs;
  * program.json        - the reference demo (test_program.py) transcript.
  * kat_metadata_u16.json, pop_u16.json, scenarios_u16.json,
    clock_stream_u16.json - the same
                          with the reference's 16-bit slot meta
                          (KVCA_SLOT_META_BITS=16: 8-bit pin and usage
                          fields), made in a child process with that
                          variable set.
The reference's 16-bit mode calls index_select, index_put_ and arithmetic
on uint16 tensors, which torch 2.11 implements for conversions only on CPU;
the child installs install_uint16_shim (below), which computes those ops
through the int16 view or int64 values with uint16 results, so the
reference's own code runs unchanged.
The Zipf and scenario generators live in kv_cache_adapter_b200/workloads.py
so that the GPU tests and bench.py regenerate identical inputs.
"""
from __future__ import annotations

import argparse
import contextlib
import io
import json
import os
import pathlib
import shutil
import subprocess
import sys
import tempfile

HERE = pathlib.Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

import torch  # noqa: E402

from kv_cache_adapter_b200 import workloads  # noqa: E402


def install_uint16_shim() -> None:
    """Make the uint16 ops the reference's 16-bit mode needs run on a torch
    build whose CPU kernels lack them (torch 2.11 implements conversions for
    uint16 but not index_select, index_put_, arithmetic or comparisons).
    Each wrapped op computes the same values through a wider or same-width
    type: indexing and in-place copies on the int16 view (bit moves only),
    arithmetic on int32 with the result wrapped to 16 bits (what uint16
    arithmetic does), comparisons on int32 (exact for every uint16 value).
    Only tensors whose dtype is uint16 take the wrapped path; the reference
    code itself is unchanged."""
    u16 = torch.uint16

    def conv(x, fn):
        if isinstance(x, torch.Tensor) and x.dtype == u16:
            return fn(x)
        if isinstance(x, (tuple, list)):
            return type(x)(conv(y, fn) for y in x)
        return x

    def has_u16(a, k):
        flat = list(a) + list(k.values())
        return any(isinstance(x, torch.Tensor) and x.dtype == u16 or
                   isinstance(x, (tuple, list)) and has_u16(x, {}) for x in flat)

    i16 = lambda t: t.view(torch.int16)  # noqa: E731  same bits
    i64 = lambda t: t.to(torch.int64)  # noqa: E731  same values

    def bits(name, inplace):
        orig = getattr(torch.Tensor, name)

        def f(self, *a, **k):
            if self.dtype == u16:  # bit moves on the int16 view; other dtypes convert mod 2^16
                r = orig(i16(self), *conv(a, i16), **{kk: conv(v, i16) for kk, v in k.items()})
                if inplace:
                    return self
                return r.view(u16) if isinstance(r, torch.Tensor) and r.dtype == torch.int16 else r
            if has_u16(a, k):  # a uint16 operand into another dtype: by value
                return orig(self, *conv(a, i64), **{kk: conv(v, i64) for kk, v in k.items()})
            return orig(self, *a, **k)
        setattr(torch.Tensor, name, f)

    def arith(name, compare):
        orig = getattr(torch.Tensor, name)

        def f(self, other):
            if self.dtype != u16 and not (isinstance(other, torch.Tensor) and other.dtype == u16):
                return orig(self, other)
            rt = torch.result_type(self, other)
            r = orig(conv(self, i64), conv(other, i64))
            if compare:
                return r
            return (r & 0xFFFF).to(u16) if rt == u16 else r.to(rt)
        setattr(torch.Tensor, name, f)

    for name in ("index_select",):
        bits(name, inplace=False)
    for name in ("index_put_", "index_fill_", "index_copy_", "copy_"):
        bits(name, inplace=True)
    for name in ("__add__", "__radd__", "__sub__", "__rsub__", "__mul__", "__rmul__", "__and__", "__rand__",
                 "__or__", "__ror__", "__xor__", "__rshift__", "__lshift__"):
        arith(name, compare=False)
    for name in ("__eq__", "__ne__", "__lt__", "__le__", "__gt__", "__ge__"):
        arith(name, compare=True)


def _import_reference(scratch: pathlib.Path):
    sys.path.insert(0, str(scratch))
    import kv_cache_adapter  # noqa: F401
    from kv_cache_adapter import adapter as ref

    return ref


def _state(ad, backend) -> dict:
    storage = backend._storage
    present = backend._present_mask
    return {
        "l2p": ad._logical_to_physical.tolist(),
        "p2l": ad._physical_to_logical.tolist(),
        "slot_meta": ad._slot_meta.tolist(),
        "search_start": int(ad._search_start[0]),
        "actual_blocks": ad.actual_blocks.reshape(ad.actual_blocks.shape[0], -1).tolist(),
        "storage": None if storage is None else storage.reshape(storage.shape[0], -1).tolist(),
        "present": None if present is None else present.int().tolist(),
        "operation_log": [list(x) for x in backend.operation_log],
    }


def kat_cases(ref) -> dict:
    """The reference KATs (test_adapter_npu_kernels.py), run through the strict path."""
    pk = lambda pin, usage: int(ref._pack_slot_meta(torch.tensor([pin]), torch.tensor([usage]))[0])  # noqa: E731
    umax = ref.USAGE_COUNT_MAX
    cases = {}

    # test_adapter_npu_kernels.py:42-64 (inspect_save)
    cases["inspect_save"] = {
        "l2p": [-1, 0, 1, -1], "slot_meta": [pk(0, 2), pk(1, umax)], "ids": [0, 1, 2, 3],
        "expect": {"cur": [-1, 0, 1, -1], "existing": [0, 1, 1, 0], "usage": [1, 3, umax, 1]},
    }
    # test_adapter_npu_kernels.py:66-88 (inspect_load)
    cases["inspect_load"] = {
        "l2p": [-1, 0, 1, -1], "slot_meta": [pk(2, 2), pk(1, umax)], "ids": [0, 1, 2, 3],
        "expect": {"cur": [-1, 0, 1, -1], "resident": [0, 1, 1, 0], "pins": [0, 3, 2, 0],
                   "usage": [0, 3, umax, 0]},
    }
    # test_adapter_npu_kernels.py:91-115 (pop: threshold scan and aging)
    cases["pop"] = {
        "slot_meta": [pk(0, 1), pk(0, 0), pk(1, 0), pk(0, 0)], "search_start": 0, "blocked": [1],
        "count": 2,
        "expect": {"selected": [3, 0], "search_start": 1,
                   "slot_meta": [pk(0, 0), pk(0, 0), pk(1, 0), pk(0, 0)]},
    }
    # test_adapter_npu_kernels.py:118-145 (commit_save)
    cases["commit_save"] = {
        "l2p": [0, 1, 2, -1, -1], "p2l": [0, 1, 2], "slot_meta": [pk(0, 1), pk(0, 2), pk(0, 3)],
        "evicted": [1, 2], "ids": [3, 4], "slots": [1, 2], "final_pins": [1, 0],
        "final_usage": [1, 2],
        "expect": {"l2p": [0, -1, -1, 1, 2], "p2l": [0, 3, 4],
                   "slot_meta": [pk(0, 1), pk(1, 1), pk(0, 2)]},
    }
    # test_adapter_npu_kernels.py:148-177 (commit_load)
    cases["commit_load"] = {
        "l2p": [0, 1, 2, -1], "p2l": [0, 1, 2], "slot_meta": [pk(1, 5), pk(1, 4), pk(1, 3)],
        "evicted": [1], "miss_ids": [3], "miss_slots": [1], "hit_slots": [0], "hit_pins": [2],
        "hit_usage": [6], "miss_usage": [2],
        "expect": {"l2p": [0, -1, 2, 1], "p2l": [0, 3, 2],
                   "slot_meta": [pk(2, 6), pk(1, 2), pk(1, 3)]},
    }
    # test_adapter_npu_kernels.py:180-194 (release)
    cases["release"] = {
        "l2p": [0, 1, -1], "slot_meta": [pk(2, 5), pk(1, 3)], "ids": [0, 1],
        "expect": {"slot_meta": [pk(1, 5), pk(0, 3)]},
    }

    # Re-run each through the strict path and check the expectations hold.
    backend = ref.InMemoryBlockStoreBackend(num_logical_blocks=8)

    def adapter_with(num_slots: int, num_logical: int):
        return ref.KVCacheAdapter(num_slots, num_logical, torch.zeros((num_slots, 2)), backend)

    c = cases["inspect_save"]
    ad = adapter_with(2, 4)
    ad._logical_to_physical.copy_(torch.tensor(c["l2p"]))
    ad._slot_meta.copy_(torch.tensor(c["slot_meta"], dtype=ref.SLOT_META_DTYPE))
    cur, existing, usage = ad._inspect_save_requests(torch.tensor(c["ids"]))
    assert cur.tolist() == c["expect"]["cur"] and existing.int().tolist() == c["expect"]["existing"]
    assert usage.tolist() == c["expect"]["usage"]

    c = cases["inspect_load"]
    ad = adapter_with(2, 4)
    ad._logical_to_physical.copy_(torch.tensor(c["l2p"]))
    ad._slot_meta.copy_(torch.tensor(c["slot_meta"], dtype=ref.SLOT_META_DTYPE))
    cur, resident, pins, usage = ad._inspect_load_requests(torch.tensor(c["ids"]))
    assert cur.tolist() == c["expect"]["cur"] and resident.int().tolist() == c["expect"]["resident"]
    assert pins.tolist() == c["expect"]["pins"] and usage.tolist() == c["expect"]["usage"]

    c = cases["pop"]
    ad = adapter_with(4, 8)
    ad._slot_meta.copy_(torch.tensor(c["slot_meta"], dtype=ref.SLOT_META_DTYPE))
    sel = ad._pop_reusable_slots(c["count"], blocked_slot_ids=torch.tensor(c["blocked"]))
    assert sel.tolist() == c["expect"]["selected"]
    assert int(ad._search_start[0]) == c["expect"]["search_start"]
    assert ad._slot_meta.tolist() == c["expect"]["slot_meta"]

    c = cases["commit_save"]
    ad = adapter_with(3, 5)
    ad._logical_to_physical.copy_(torch.tensor(c["l2p"]))
    ad._physical_to_logical.copy_(torch.tensor(c["p2l"]))
    ad._slot_meta.copy_(torch.tensor(c["slot_meta"], dtype=ref.SLOT_META_DTYPE))
    ad._commit_save_metadata(
        evicted_logical_block_ids=torch.tensor(c["evicted"]), logical_block_ids=torch.tensor(c["ids"]),
        physical_slot_ids=torch.tensor(c["slots"]),
        final_pin_counts=torch.tensor(c["final_pins"], dtype=ref.SLOT_META_DTYPE),
        final_usage_counts=torch.tensor(c["final_usage"], dtype=ref.SLOT_META_DTYPE))
    assert ad._logical_to_physical.tolist() == c["expect"]["l2p"]
    assert ad._physical_to_logical.tolist() == c["expect"]["p2l"]
    assert ad._slot_meta.tolist() == c["expect"]["slot_meta"]

    c = cases["commit_load"]
    ad = adapter_with(3, 4)
    ad._logical_to_physical.copy_(torch.tensor(c["l2p"]))
    ad._physical_to_logical.copy_(torch.tensor(c["p2l"]))
    ad._slot_meta.copy_(torch.tensor(c["slot_meta"], dtype=ref.SLOT_META_DTYPE))
    ad._commit_load_metadata(
        evicted_logical_block_ids=torch.tensor(c["evicted"]),
        miss_logical_block_ids=torch.tensor(c["miss_ids"]),
        miss_physical_slot_ids=torch.tensor(c["miss_slots"]),
        hit_slot_ids=torch.tensor(c["hit_slots"]), hit_pin_counts=torch.tensor(c["hit_pins"]),
        hit_usage_counts=torch.tensor(c["hit_usage"], dtype=ref.SLOT_META_DTYPE),
        miss_usage_counts=torch.tensor(c["miss_usage"], dtype=ref.SLOT_META_DTYPE))
    assert ad._logical_to_physical.tolist() == c["expect"]["l2p"]
    assert ad._physical_to_logical.tolist() == c["expect"]["p2l"]
    assert ad._slot_meta.tolist() == c["expect"]["slot_meta"]

    c = cases["release"]
    ad = adapter_with(2, 3)
    ad._logical_to_physical.copy_(torch.tensor(c["l2p"]))
    ad._slot_meta.copy_(torch.tensor(c["slot_meta"], dtype=ref.SLOT_META_DTYPE))
    ad.release(torch.tensor(c["ids"]))
    assert ad._slot_meta.tolist() == c["expect"]["slot_meta"]
    return cases


def pop_cases(ref, count: int, seed: int) -> list[dict]:
    out = []
    backend = ref.InMemoryBlockStoreBackend(num_logical_blocks=1)
    for case in workloads.pop_case_params(count, seed, usage_max=ref.USAGE_COUNT_MAX,
                                          pin_max=ref.PIN_COUNT_MAX):
        n = len(case["usage"])
        ad = ref.KVCacheAdapter(n, n, torch.zeros((n, 1)), backend)
        ad._slot_meta.copy_(ref._pack_slot_meta(torch.tensor(case["pins"]), torch.tensor(case["usage"])))
        ad._search_start[0] = case["search_start"]
        record = dict(case)
        record["slot_meta"] = ad._slot_meta.tolist()
        try:
            sel = ad._pop_reusable_slots(case["count"], blocked_slot_ids=torch.tensor(case["blocked"], dtype=torch.int64))
            record["selected"] = sel.tolist()
            record["error"] = None
        except ref.InsufficientCapacityError:
            record["selected"] = None
            record["error"] = "InsufficientCapacityError"
        record["after_slot_meta"] = ad._slot_meta.tolist()
        record["after_search_start"] = int(ad._search_start[0])
        out.append(record)
    return out


def scenarios(ref, count: int, seed: int) -> list[dict]:
    out = []
    for spec in workloads.scenario_specs(count, seed):
        init = {int(k): torch.tensor(v, dtype=torch.float32).reshape(spec["block_shape"])
                for k, v in spec["initial"].items()}
        backend = (ref.InMemoryBlockStoreBackend(init, num_logical_blocks=spec["num_logical"])
                   if init else ref.InMemoryBlockStoreBackend(num_logical_blocks=spec["num_logical"]))
        ad = ref.KVCacheAdapter(spec["num_actual"], spec["num_logical"],
                                torch.zeros((spec["num_actual"], *spec["block_shape"])), backend)
        steps = []
        for op in workloads.scenario_ops(spec):
            ids = torch.tensor(op["ids"], dtype=torch.int64)
            step = {"op": op["op"], "ids": op["ids"], "result": None, "error": None}
            try:
                if op["op"] == "load":
                    step["result"] = ad.load(ids).tolist()
                elif op["op"] == "save":
                    data = torch.tensor(op["data"], dtype=torch.float32).reshape(len(op["ids"]), *spec["block_shape"])
                    ad.save(ids, data)
                else:
                    ad.release(ids)
            except Exception as exc:  # recorded, and the sequence goes on
                step["error"] = type(exc).__name__
            step["state"] = _state(ad, backend)
            steps.append(step)
            if op["op"] == "save":
                step["data"] = op["data"]
        out.append({"spec": spec, "steps": steps})
    return out


def clock_streams(ref) -> list[dict]:
    out = []
    backend = ref.InMemoryBlockStoreBackend(num_logical_blocks=1)
    for params in workloads.clock_stream_params_small():
        meta0 = workloads.clock_initial_meta(params, ref._pack_slot_meta)
        reaccess = workloads.zipf_reaccess(params)
        n = params["num_slots"]
        ad = ref.KVCacheAdapter(n, n, torch.zeros((n, 1)), backend)
        ad._slot_meta.copy_(meta0)
        victims: list[int] = []
        k, m = params["alloc_per_step"], params["reaccess_per_step"]
        error = None
        steps_done = 0
        for step in range(params["num_steps"]):
            try:
                v = ad._pop_reusable_slots(k, blocked_slot_ids=torch.empty(0, dtype=torch.int64))
            except ref.InsufficientCapacityError:
                error = "InsufficientCapacityError"
                break
            victims.extend(v.tolist())
            # refill the victims as a save miss: pin kept, usage 1 (adapter.py:233-242, :651)
            pins = ref._slot_meta_pin_counts(ad._slot_meta.index_select(0, v))
            ad._slot_meta.index_put_((v,), ref._pack_slot_meta(pins, torch.ones_like(v)))
            # usage bump of the re-accessed slots (adapter.py:1414-1416)
            r = reaccess[step * m:(step + 1) * m]
            cur = ad._slot_meta.index_select(0, r)
            bumped = ref._saturating_increment_usage(ref._slot_meta_usage_counts(cur))
            ad._slot_meta.index_put_((r,), ref._pack_slot_meta(ref._slot_meta_pin_counts(cur), bumped))
            steps_done += 1
        out.append({
            "params": params,
            "victims": victims,
            "steps_done": steps_done,
            "error": error,
            "final_slot_meta_sha256": workloads.sha256_of(ad._slot_meta),
            "final_search_start": int(ad._search_start[0]),
            "final_slot_meta": ad._slot_meta.tolist() if n <= 4096 else None,
        })
    return out


def layout_cases(ref) -> dict:
    cases = []
    for shape in [(16, 2, 4, 8), (2, 16, 4, 8), (16, 2, 8, 128), (2, 64, 1, 576), (4, 4), (2, 2, 2)]:
        layout = ref._MergedKVBlockLayout.detect(shape)
        rec = {"block_shape": list(shape), "detected": layout is not None}
        if layout is not None:
            rec.update({
                "transfer_shape": list(layout.transfer_shape),
                "block_size": layout.block_size,
                "hidden_dim": layout.hidden_dim,
                "token_major": layout.token_major,
            })
            fused = ref._NPUFusedBlockTransfer(block_shape=torch.Size(shape), block_dtype=torch.float16,
                                               memory_format_enum=None)
            slots = torch.tensor([3, 0, 7, 2], dtype=torch.int64)
            rec["slot_ids"] = slots.tolist()
            rec["physical_slot_mapping"] = fused._physical_slot_mapping(slots).tolist()
            rec["dense_slot_mapping"] = fused._dense_slot_mapping(3, device=torch.device("cpu")).tolist()
            rec["chunk_offsets"] = fused._chunk_offsets(3)
            rec["chunk_sizes"] = fused._chunk_sizes(3)
        cases.append(rec)
    return {"cases": cases}


def program_transcript(scratch: pathlib.Path) -> dict:
    buf = io.StringIO()
    sys.path.insert(0, str(scratch / "kv_cache_adapter"))
    import test_program  # the reference demo, run on CPU

    with contextlib.redirect_stdout(buf):
        test_program.main()
    lines = [ln for ln in buf.getvalue().splitlines() if not ln.startswith("adapter snapshot")]
    return {"stdout": lines}


POP_U16 = dict(count=200, seed=4321)
SCENARIOS_U16 = dict(count=30, seed=4321)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("KVCA_REFERENCE_DIR"),
                    help="the reference project's directory (default: $KVCA_REFERENCE_DIR)")
    ap.add_argument("--out", default=str(HERE))
    ap.add_argument("--meta16", action="store_true", help="(child) the 16-bit fixtures")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give the reference project's directory (--reference or KVCA_REFERENCE_DIR)")
    out = pathlib.Path(args.out)

    def dump(name: str, obj) -> None:
        (out / name).write_text(json.dumps(obj, separators=(",", ":")) + "\n")

    with tempfile.TemporaryDirectory() as tmp:
        scratch = pathlib.Path(tmp)
        shutil.copytree(args.reference, scratch / "kv_cache_adapter")
        if args.meta16:
            assert os.environ.get("KVCA_SLOT_META_BITS") == "16"
            install_uint16_shim()
            ref = _import_reference(scratch)
            assert ref.SLOT_META_DTYPE == torch.uint16
            dump("kat_metadata_u16.json", kat_cases(ref))
            dump("pop_u16.json", pop_cases(ref, **POP_U16))
            dump("scenarios_u16.json", scenarios(ref, **SCENARIOS_U16))
            dump("clock_stream_u16.json", clock_streams(ref))
            return
        ref = _import_reference(scratch)
        assert ref.SLOT_META_DTYPE == torch.uint8, "run with 8-bit slot meta"

        dump("kat_metadata.json", kat_cases(ref))
        dump("pop_u8.json", pop_cases(ref, 400, seed=1234))
        dump("scenarios_u8.json", scenarios(ref, 60, seed=1234))
        dump("clock_stream.json", clock_streams(ref))
        dump("layout.json", layout_cases(ref))
        dump("program.json", program_transcript(scratch))
    env = dict(os.environ, KVCA_SLOT_META_BITS="16")
    subprocess.run([sys.executable, __file__, "--reference", args.reference, "--out", str(out), "--meta16"],
                   env=env, check=True)


if __name__ == "__main__":
    main()
