"""Builds libhkv.so (the engine: host C++ + sm_100a kernels) in-tree.

Usage: python higgs-audio.cpp_b200/hkv_build.py [--force]

The library is a plain C-ABI shared object (include/hkv.h); nothing here
depends on torch.  The output lands in higgs-audio.cpp_b200/lib/ so it
travels with the source tree.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "lib"
LIB = LIB_DIR / "libhkv.so"
SOURCES = [CSRC / "hkv_kernels.cu", CSRC / "hkv_engine.cpp", CSRC / "hkv_noalloc.cu",
           CSRC / "hkv_backbone.cu"]
HEADERS = [CSRC / "hkv_internal.h", CSRC / "hkv_plan.h", CSRC / "hkv_device.cuh",
           REPO / "include" / "hkv.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC,-O3,-Wall",
    "-shared",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the engine needs the CUDA 12.9 toolchain")


def host_compiler() -> str:
    # nvcc's host compiler: the system g++ (an inherited CXX may lack parts of
    # the runtime).
    return shutil.which("g++", path="/usr/bin:/bin") or "g++"


def stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not stale():
        return LIB
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), "-ccbin", host_compiler(), *NVCC_FLAGS,
           *[str(s) for s in SOURCES], "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"building {LIB.name} failed (exit {res.returncode})")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=True))
