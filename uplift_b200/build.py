"""Build the sm_100a Local Attender library in-tree with nvcc.

    python -m uplift_b200.build          # -> uplift_b200/lib/libuplift_la.so

The library is plain CUDA C++ behind a C ABI (include/uplift_la.h): no torch
headers, cudart linked statically, so any host language can bind it.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
INCLUDE = ROOT / "include"
CSRC = PKG / "csrc"
LIB_DIR = PKG / "lib"
LIB_NAME = "libuplift_la.so"
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the Local Attender library needs the CUDA 12.8+ toolkit")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def lib_path() -> Path:
    return LIB_DIR / LIB_NAME


def is_stale() -> bool:
    lib = lib_path()
    if not lib.exists():
        return True
    t = lib.stat().st_mtime
    deps = sources() + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every .cu under uplift_b200/csrc (one nvcc per file, in
    parallel) and link them into one shared library."""
    if not force and not is_stale():
        return lib_path()
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    obj_dir = LIB_DIR / "obj"
    obj_dir.mkdir(exist_ok=True)
    nvcc = nvcc_path()
    common = [*ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", f"-I{INCLUDE}", f"-I{CSRC}"]
    if verbose:
        common.append("-Xptxas=-v")
    procs, objs = [], []
    for src in sources():
        obj = obj_dir / (src.stem + ".o")
        cmd = [nvcc, *common, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        procs.append((src, subprocess.Popen(cmd)))
        objs.append(obj)
    failed = [src.name for src, proc in procs if proc.wait() != 0]
    if failed:
        raise RuntimeError(f"nvcc failed on {', '.join(failed)}")
    tmp = lib_path().with_suffix(".so.tmp")
    subprocess.run([nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)], check=True)
    os.replace(tmp, lib_path())
    return lib_path()


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
