"""Recipe: compile the reference's own CUDA extension into oracle/_ref/ -- TEST
INFRASTRUCTURE ONLY.

    python -m oracle.build_ref [--reference DIR] [--force]

The reference ships its metadata kernels as a torch extension
(``csrc/kv_adapter_cuda.cu`` + ``csrc/binding.cpp``, module
``kv_cache_adapter_cuda``, bound at ``csrc/binding.cpp:64-99``).  This recipe
compiles those two files unchanged, from where they lie in the reference
project, with torch's extension builder (the torch headers and libraries of
this image; no reference build system is run).  Flags follow the reference's
``setup.py:252-265`` (``-O3 --use_fast_math``) plus the sm_100a target that
its flags lack.  Every output (objects, ninja file, the module
``kvca_reference_cuda.so``) goes to ``oracle/_ref/``, which git ignores and
which travels with the repository snapshot to a GPU machine, where
``load()`` imports the prebuilt module without needing the reference sources.

The module is the checker for the prefix-order clock sweep
(``pop_reusable_slots_kernel``, ``csrc/kv_adapter_cuda.cu:64-237``, host side
``:406-450``) and the per-call pop timing of the reference's CUDA arm.  The
product never loads it.

The reference project is looked up in ``--reference``, else the
``KVCA_REFERENCE_DIR`` environment variable, else the standard read-only
mount ``/root/reference``; when none exists the recipe does nothing.
"""
from __future__ import annotations

import argparse
import importlib.machinery
import importlib.util
import os
import pathlib
import sys
from types import ModuleType

HERE = pathlib.Path(__file__).resolve().parent
OUT = HERE / "_ref"
NAME = "kvca_reference_cuda"
MODULE = OUT / f"{NAME}.so"
SOURCES = ("csrc/binding.cpp", "csrc/kv_adapter_cuda.cu")
DEFAULT_REFERENCE = "/root/reference"


def reference_dir(explicit: str | None = None) -> pathlib.Path | None:
    for cand in (explicit, os.environ.get("KVCA_REFERENCE_DIR"), DEFAULT_REFERENCE):
        if cand and (pathlib.Path(cand) / SOURCES[1]).exists():
            return pathlib.Path(cand)
    return None


def build(reference: str | None = None, force: bool = False) -> pathlib.Path | None:
    """Compile the reference extension; None when the reference is absent."""
    ref = reference_dir(reference)
    if ref is None:
        return None
    srcs = [ref / s for s in SOURCES]
    if MODULE.exists() and not force and all(s.stat().st_mtime <= MODULE.stat().st_mtime for s in srcs):
        return MODULE
    OUT.mkdir(exist_ok=True)
    from torch.utils import cpp_extension

    cpp_extension.load(
        name=NAME,
        sources=[str(s) for s in srcs],
        build_directory=str(OUT),
        extra_cflags=["-O3"],
        extra_cuda_cflags=["-O3", "--use_fast_math", "-gencode", "arch=compute_100a,code=sm_100a"],
        with_cuda=True,
        verbose=False,
    )
    if not MODULE.exists():
        raise RuntimeError(f"reference extension build left no {MODULE}")
    return MODULE


_mod: ModuleType | None = None


def available() -> bool:
    return MODULE.exists()


def load() -> ModuleType:
    """Import the prebuilt reference module (after torch, whose libraries it links)."""
    global _mod
    if _mod is None:
        import torch  # noqa: F401  (loads libtorch / libc10 first)

        if not MODULE.exists():
            raise FileNotFoundError(f"{MODULE} is not built (python -m oracle.build_ref)")
        loader = importlib.machinery.ExtensionFileLoader(NAME, str(MODULE))
        spec = importlib.util.spec_from_file_location(NAME, str(MODULE), loader=loader)
        mod = importlib.util.module_from_spec(spec)
        loader.exec_module(mod)
        _mod = mod
    return _mod


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--reference", default=None)
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args(argv)
    print(build(args.reference, force=args.force) or "reference project not found: nothing built")


if __name__ == "__main__":
    main(sys.argv[1:])
