"""Builds libddtree_b200.so (the C-ABI library) in-tree with nvcc for sm_100a.

    python -m ddtree_eagle3_patch_b200.build [--force]

The library links the CUDA runtime statically and exports only the
``extern "C"`` entry points declared in include/ddtree_b200.h.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libddtree_b200.so"
SOURCES = ["capi.cu", "tree_build.cu", "accept.cu", "attention.cu", "attention_f32.cu", "cache.cu", "fused.cu",
           "mask.cu", "sample.cu", "wgemm.cu"]
HEADERS = ["common.cuh", "sm100.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the B200 library cannot be built")


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + [CSRC / h for h in HEADERS] + [ROOT / "include" / "ddtree_b200.h"]
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not _stale():
        return LIB
    out_dir = PKG / "_build"
    out_dir.mkdir(exist_ok=True)
    objs = []
    common = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler",
              "-fvisibility=hidden", f"-I{ROOT / 'include'}", "-DDDT_BUILD"]
    for src in SOURCES:
        obj = out_dir / (Path(src).stem + ".o")
        cmd = common + ["-c", str(CSRC / src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = LIB.with_suffix(f".so.tmp{os.getpid()}")
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *objs, "-cudart", "static"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
