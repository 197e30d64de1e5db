#!/usr/bin/env python3
"""Builds libmathplus_cuda.so (sm_100a) in-tree, next to this file, with nvcc.

    python math-plus_b200/build.py [--force] [--jobs N]

Every .cu file under csrc/ is compiled for ``-gencode arch=compute_100a,code=sm_100a`` into
``lib/libmathplus_cuda.so``; objects are cached under ``_build/`` and rebuilt when a source or
header is newer. The library links only the CUDA runtime (statically) and libdl.
"""
from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "lib")
LIB = os.path.join(OUT_DIR, "libmathplus_cuda.so")
OBJ_DIR = os.path.join(ROOT, "_build", "mathplus_cuda")


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def host_cxx() -> list[str]:
    # /usr/bin/g++ is the system compiler nvcc supports; prefer it over other g++ on PATH.
    return ["-ccbin", "/usr/bin/g++"] if os.path.exists("/usr/bin/g++") else []


FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-Xptxas", "-warn-spills",
    "-I", os.path.join(ROOT, "include"),
]


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def headers() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
                  + glob.glob(os.path.join(ROOT, "include", "*.h")))


def _compile(src: str, force: bool, verbose: bool) -> str:
    obj = os.path.join(OBJ_DIR, os.path.basename(src) + ".o")
    newest_dep = max([os.path.getmtime(src)] + [os.path.getmtime(h) for h in headers()])
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= newest_dep:
        return obj
    cmd = [nvcc(), *host_cxx(), *FLAGS, "-c", src, "-o", obj]
    if verbose:
        cmd.insert(-4, "-Xptxas")
        cmd.insert(-4, "-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout or r.stderr):
        sys.stderr.write(r.stdout + r.stderr)
    return obj


def build(force: bool = False, jobs: int = 8, verbose: bool = False) -> str:
    os.makedirs(OBJ_DIR, exist_ok=True)
    os.makedirs(OUT_DIR, exist_ok=True)
    with ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, verbose), sources()))
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= max(os.path.getmtime(o) for o in objs):
        return LIB
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *host_cxx(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", tmp, *objs,
           "-cudart", "static", "-ldl", "-lpthread"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=8)
    ap.add_argument("-v", "--verbose", action="store_true", help="print ptxas register / spill report")
    a = ap.parse_args()
    print(build(a.force, a.jobs, a.verbose))


if __name__ == "__main__":
    main()
