"""The reference's own ``adapter.py`` with this library dropped in (test helper).

INTEGRATION.md's "Option B" keeps the reference's adapter and replaces its
CUDA extension with ``kv_cache_adapter_b200.kv_cache_adapter_cuda``.  This
module makes those edits on a scratch copy of the reference project, never in
this repository:

1. the six native branches (``release``, ``_inspect_load_requests``,
   ``_inspect_save_requests``, ``_pop_reusable_slots``,
   ``_commit_load_metadata``, ``_commit_save_metadata``; adapter.py:317,
   :398, :438, :478, :558, :616) take the packed slot-meta signatures on CUDA
   as they do on NPU;
2. the eviction gather (adapter.py:543) and the block scatter
   (adapter.py:656) call the row mover on CUDA;
3. a sibling ``kv_cache_adapter_cuda.py`` re-exports this library's module,
   where ``_load_cuda_extension_module`` (adapter.py:1347-1367) looks first.

``Recorder`` wraps an op set and records every call the reference adapter
makes (arguments, results, the adapter state before and after), so the same
calls can be replayed through the CUDA module on a GPU, where the reference
sources are not available.
"""
from __future__ import annotations

import importlib
import pathlib
import shutil
import sys

import torch

NATIVE_BRANCH = 'if self._platform == "npu":'
NATIVE_BRANCH_CUDA = 'if self._platform in ("npu", "cuda"):'
GATHER_LINE = "eviction_payloads = self.actual_blocks.index_select(0, eviction_slot_ids)"
GATHER_CUDA = ("eviction_payloads = (self._native_ext.gather_blocks(self.actual_blocks, eviction_slot_ids)\n"
               "                             if self._platform == \"cuda\" else "
               "self.actual_blocks.index_select(0, eviction_slot_ids))")
SCATTER_LINE = "self.actual_blocks.index_copy_(0, physical_slot_ids, block_data)"
SCATTER_CUDA = ("if self._platform == \"cuda\":\n"
                "            self._native_ext.scatter_blocks(self.actual_blocks, physical_slot_ids, "
                "block_data.contiguous())\n"
                "            return\n"
                "        self.actual_blocks.index_copy_(0, physical_slot_ids, block_data)")
SHIM = ('"""This library in place of the reference\'s CUDA extension."""\n'
        "from kv_cache_adapter_b200.kv_cache_adapter_cuda import *  # noqa: F401,F403\n")


def patch_adapter_source(text: str) -> str:
    """The Option B edits on the text of the reference's adapter.py."""
    assert text.count(NATIVE_BRANCH) == 6, "expected the six native branches"
    assert text.count(GATHER_LINE) == 1 and text.count(SCATTER_LINE) == 1
    text = text.replace(NATIVE_BRANCH, NATIVE_BRANCH_CUDA)
    text = text.replace(GATHER_LINE, GATHER_CUDA)
    return text.replace(SCATTER_LINE, SCATTER_CUDA)


def import_patched_reference(reference: pathlib.Path, scratch: pathlib.Path):
    """Copy the reference project to ``scratch/kv_cache_adapter``, apply the
    edits, add the sibling shim, import it as package ``kv_cache_adapter``."""
    pkg = scratch / "kv_cache_adapter"
    shutil.copytree(reference, pkg, ignore=shutil.ignore_patterns("csrc", "*.so", "build"))
    adapter = pkg / "adapter.py"
    adapter.write_text(patch_adapter_source(adapter.read_text()))
    (pkg / "kv_cache_adapter_cuda.py").write_text(SHIM)
    for name in [m for m in sys.modules if m == "kv_cache_adapter" or m.startswith("kv_cache_adapter.")]:
        del sys.modules[name]
    sys.path.insert(0, str(scratch))
    try:
        return importlib.import_module("kv_cache_adapter")
    finally:
        sys.path.remove(str(scratch))


STATE = ("l2p", "p2l", "slot_meta", "search_start", "actual_blocks")


def adapter_state(ad) -> dict:
    return {"l2p": ad._logical_to_physical, "p2l": ad._physical_to_logical, "slot_meta": ad._slot_meta,
            "search_start": ad._search_start, "actual_blocks": ad.actual_blocks}


def _values(t: torch.Tensor) -> dict:
    return {"t": t.detach().cpu().reshape(-1).tolist(), "dtype": str(t.dtype).replace("torch.", ""),
            "shape": list(t.shape)}


class Recorder:
    """Forwards the reference adapter's native calls to ``ops`` and records them."""

    OPS = ("inspect_load_requests", "inspect_save_requests", "pop_reusable_slots", "commit_load_metadata",
           "commit_save_metadata", "release_metadata", "gather_blocks", "scatter_blocks")

    def __init__(self, ops) -> None:
        self.ops = ops
        self.adapter = None
        self.calls: list[dict] = []

    def _arg(self, a):
        if isinstance(a, torch.Tensor):
            for name, t in adapter_state(self.adapter).items():
                if a.numel() and a.data_ptr() == t.data_ptr() and a.shape == t.shape:
                    return {"state": name}
            return _values(a)
        return a

    def _snapshot(self) -> dict:
        return {k: v.detach().cpu().reshape(-1).tolist() for k, v in adapter_state(self.adapter).items()}

    def __getattr__(self, name):
        if name not in self.OPS:
            raise AttributeError(name)
        fn = getattr(self.ops, name)

        def call(*args):
            rec = {"op": name, "args": [self._arg(a) for a in args], "before": self._snapshot()}
            try:
                out = fn(*args)
                rec["error"] = None
            except Exception as exc:  # recorded by type name, re-raised for the adapter
                rec["error"] = type(exc).__name__
                rec["out"] = None
                rec["after"] = self._snapshot()
                self.calls.append(rec)
                raise
            if isinstance(out, (tuple, list)):
                rec["out"] = [_values(o) for o in out]
            elif isinstance(out, torch.Tensor):
                rec["out"] = _values(out)
            else:
                rec["out"] = None
            rec["after"] = self._snapshot()
            self.calls.append(rec)
            return out

        return call


def make_adapter(ref, spec: dict, native_ext, device=torch.device("cpu")):
    """The reference's KVCacheAdapter and InMemoryBlockStoreBackend for a
    recorded scenario, with ``native_ext`` on its CUDA branch.  On CPU tensors
    the adapter would choose its strict path, so the platform and extension
    are set after construction, as the constructor sets them for CUDA tensors
    (adapter.py:167, :369-381)."""
    shape = tuple(spec["block_shape"])
    init = {int(k): torch.tensor(v, dtype=torch.float32, device=device).reshape(shape)
            for k, v in spec["initial"].items()}
    kwargs = {"num_logical_blocks": spec["num_logical"]}
    backend = ref.InMemoryBlockStoreBackend(init, **kwargs) if init else ref.InMemoryBlockStoreBackend(**kwargs)
    ad = ref.KVCacheAdapter(spec["num_actual"], spec["num_logical"],
                            torch.zeros((spec["num_actual"], *shape), dtype=torch.float32, device=device), backend)
    ad._native_ext = native_ext
    ad._platform = "cuda"
    ad.runtime_path = "cuda_ext_meta"
    return ad, backend


def run_step(ad, step: dict, shape: tuple, device=torch.device("cpu")):
    """One recorded load / save / release through the adapter: (result, error name)."""
    ids = torch.tensor(step["ids"], dtype=torch.int64, device=device)
    try:
        if step["op"] == "load":
            return ad.load(ids).tolist(), None
        if step["op"] == "save":
            data = torch.tensor(step["data"], dtype=torch.float32, device=device).reshape(len(step["ids"]), *shape)
            ad.save(ids, data)
        else:
            ad.release(ids)
        return None, None
    except Exception as exc:
        return None, type(exc).__name__
