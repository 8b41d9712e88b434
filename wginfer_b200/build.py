"""Builds wginfer_b200/libwginfer_b200.so from wginfer_b200/csrc for sm_100a.

Every translation unit is compiled by nvcc with
``-gencode arch=compute_100a,code=sm_100a`` (tcgen05/TMA need the arch-specific
target) and linked into one shared library with the CUDA runtime linked
statically, so the library loads on a machine without a GPU driver (the
driver is only needed at the first CUDA call). The driver API entry points
used for TMA descriptors are fetched at run time through
cudaGetDriverEntryPoint, never linked.

Usage: python -m wginfer_b200.build [--force] [-j N]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libwginfer_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include"), "-I", CSRC,
         "-DWGB_BUILDING_LIBRARY"]


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def _headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) +
                  glob.glob(os.path.join(ROOT, "include", "*.h")))


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, extra, verbose):
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    if not _stale(obj, [src] + _headers() + [__file__]):
        return obj
    cmd = [NVCC] + ARCH + FLAGS + extra + ["-c", src, "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr.strip():
        print(r.stderr, flush=True)
    return obj


def build(force: bool = False, jobs: int | None = None, verbose: bool = False, ptxas_info: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    if force:
        for f in glob.glob(os.path.join(BUILD, "*.o")):
            os.remove(f)
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra, verbose or ptxas_info), srcs))
    if _stale(LIB, objs) or force:
        cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs + ["-cudart", "static", "-ldl", "-lpthread", "-lrt"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.check_call(cmd)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("-v", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.j, a.v, a.ptxas_info))
    sys.exit(0)
