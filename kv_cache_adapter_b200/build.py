"""Build recipe for libkvca_b200.so (sm_100a only).

    python -m kv_cache_adapter_b200.build [--force] [--ptxas-verbose]

Compiles csrc/kv_adapter_cuda.cu (kernels), csrc/row_ceiling.cu (the
random-row roofline reference) and csrc/binding.cpp (the C ABI of
include/kvca.h) with nvcc into a shared library next to this file, with
the CUDA runtime linked statically so the library has no runtime dependency
beyond the driver.
"""
from __future__ import annotations

import argparse
import os
import pathlib
import shutil
import subprocess
import sys

PKG = pathlib.Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = REPO / "include"
SOURCES = [CSRC / "kv_adapter_cuda.cu", CSRC / "row_ceiling.cu", CSRC / "binding.cpp"]
HEADERS = [CSRC / "kvca_launch.h", INCLUDE / "kvca.h"]
TARGET = PKG / "libkvca_b200.so"
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and pathlib.Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the sm_100a library cannot be built")


def stale() -> bool:
    if not TARGET.exists():
        return True
    t = TARGET.stat().st_mtime
    return any(p.stat().st_mtime > t for p in SOURCES + HEADERS)


def build(force: bool = False, ptxas_verbose: bool = False) -> pathlib.Path:
    if not force and not stale():
        return TARGET
    cmd = [
        nvcc(), *ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
        "-cudart", "static", f"-I{INCLUDE}", f"-I{CSRC}",
        *(["-Xptxas", "-v"] if ptxas_verbose else []),
        *[str(s) for s in SOURCES], "-o", str(TARGET) + ".tmp",
    ]
    subprocess.run(cmd, check=True)
    os.replace(str(TARGET) + ".tmp", TARGET)
    return TARGET


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    args = ap.parse_args(argv)
    print(build(force=args.force, ptxas_verbose=args.ptxas_verbose))


if __name__ == "__main__":
    main(sys.argv[1:])
