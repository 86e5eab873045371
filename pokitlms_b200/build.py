"""Builds pokitlms_b200/libpokit_cuda.so (the C-ABI library) for sm_100a.

nvcc cross-compiles without a GPU, so this runs on any machine with the CUDA
12.9 toolkit.  The library links the CUDA runtime statically and exposes only
the plain-C entry points declared in include/pokit_cuda.h; it has no torch
dependency.

Usage:  python -m pokitlms_b200.build [--force] [--verbose]
"""
from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libpokit_cuda.so"

SOURCES = ["pokit_linear.cu", "pokit_moe.cu", "pokit_grouped.cu", "pokit_synth.cu", "pokit_backend.cpp",
           "pokit_static_scratch.cu", "pokit_decoder.cu", "pokit_deltanet.cu",
           "pokit_deltablock.cu"]
HEADERS = ["pokit_common.cuh", "pokit_quant.cuh", "pokit_mma.cuh", "pokit_tc.cuh", "pokit_attention.cuh", "pokit_deltablock.cuh", "pokit_kernels.h",
           "pokit_types.h"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-Wall",
                f"-I{ROOT / 'include'}", f"-I{CSRC}"]


def nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    cand = Path("/usr/local/cuda/bin/nvcc")
    if cand.exists():
        return str(cand)
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libpokit_cuda.so")


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, obj: Path, verbose: bool) -> None:
    cmd = [nvcc(), *ARCH_FLAGS, *COMMON_FLAGS, "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cu":
        cmd.insert(1, "-Xptxas=-v" if verbose else "-Xptxas=-O3")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, file=sys.stderr)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compiles every CUDA/C++ source for sm_100a and links the shared library."""
    BUILD.mkdir(exist_ok=True)
    headers = [CSRC / h for h in HEADERS] + [ROOT / "include" / "pokit_cuda.h"]
    jobs = []
    objs = []
    for name in SOURCES:
        src = CSRC / name
        obj = BUILD / (name + ".o")
        objs.append(obj)
        if force or _stale(obj, [src, *headers]):
            jobs.append((src, obj))
    if jobs:
        workers = min(len(jobs), os.cpu_count() or 1)
        with concurrent.futures.ThreadPoolExecutor(max_workers=workers) as pool:
            list(pool.map(lambda j: _compile(j[0], j[1], verbose), jobs))
    if force or jobs or _stale(LIB, objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp),
               *[str(o) for o in objs], "-Xcompiler", "-fPIC"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
