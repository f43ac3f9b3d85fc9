"""Build the sm_100a shared library ``lib/libagillm_moe.so`` with nvcc.

Usage: ``python agillm4.1_b200/build.py [--force] [-v]`` or ``build()`` from
Python. Every ``csrc/*.cu`` is compiled for ``-gencode
arch=compute_100a,code=sm_100a`` with ``-lineinfo`` (objects in ``_build/``,
compiled in parallel) and linked into one position-independent shared
library whose exported symbols are the ``extern "C"`` entry points declared
in ``include/agillm_moe.h``. The CUDA runtime is linked statically and the
driver entry point for tensor-map encoding is resolved at run time, so the
library needs no libcuda at link time and loads on a host without a GPU.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(REPO, "include")
LIB_DIR = os.path.join(PKG_DIR, "lib")
LIB_PATH = os.path.join(LIB_DIR, "libagillm_moe.so")
BUILD_DIR = os.path.join(REPO, "_build")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put /usr/local/cuda/bin on PATH)")


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) +
                  glob.glob(os.path.join(INCLUDE, "*.h")))


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, extra_flags=None) -> str:
    """Compile (if stale) and return the path of the shared library."""
    nvcc = nvcc_path()
    os.makedirs(BUILD_DIR, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    hdrs = headers()
    flags = ARCH_FLAGS + NVCC_FLAGS + ["-I", INCLUDE, "-I", CSRC] + list(extra_flags or [])
    jobs = []
    objs = []
    for src in sources():
        obj = os.path.join(BUILD_DIR, os.path.basename(src) + ".o")
        objs.append(obj)
        if force or _stale(obj, [src, __file__] + hdrs):
            jobs.append([nvcc] + flags + ["-c", src, "-o", obj])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed ({r.returncode}):\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout + r.stderr, flush=True)
        return r

    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            list(ex.map(run, jobs))
    if force or jobs or _stale(LIB_PATH, objs):
        tmp = LIB_PATH + ".tmp"
        run([nvcc] + ARCH_FLAGS + ["-shared", "-o", tmp] + objs + ["-cudart", "static"])
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers/spills/smem per kernel")
    args = ap.parse_args(argv)
    extra = ["-Xptxas", "-v"] if args.ptxas_info else []
    path = build(force=args.force or args.ptxas_info, verbose=args.verbose or args.ptxas_info, extra_flags=extra)
    print(path)


if __name__ == "__main__":
    sys.exit(main())
