"""Build libbramha_cuda.so and libbramha_cuda.a in-tree with nvcc for sm_100a.

    python -m bramha_b200.build [--force] [-v]

Every .cu file under csrc/ is compiled with
``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3`` and linked into one
shared library next to this file (the C ABI of include/bramha_cuda.h), and
archived into a static library of the same objects.  No
fast-math: the packers must round exactly like the reference, and the GEMV's
int4/int8 decode relies on subnormal floats (no flush-to-zero).
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libbramha_cuda.so")
STATIC_LIB = os.path.join(HERE, "libbramha_cuda.a")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3,-fvisibility=hidden",
    "--expt-relaxed-constexpr", "-ftz=false", "-prec-div=true", "-prec-sqrt=true",
    "-I", os.path.join(ROOT, "include"), "-I", CSRC,
]


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h")))


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, verbose):
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    if not _stale(obj, [src] + _headers()):
        return obj, ""
    cmd = [NVCC] + FLAGS + (["-Xptxas", "-v"] if verbose else []) + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = _sources()
    if force:
        for o in glob.glob(os.path.join(BUILD, "*.o")):
            os.remove(o)
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        results = list(ex.map(lambda s: _compile(s, verbose), srcs))
    objs = [o for o, _ in results]
    if verbose:
        for _, log in results:
            if log:
                sys.stderr.write(log)
    if force or _stale(LIB, objs):
        cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcudart_static", "-lrt", "-ldl", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if force or _stale(STATIC_LIB, objs):
        # the same objects as a static archive, for a host program (e.g. a Rust
        # crate's build step) that links the plane into its own binary; the
        # final link adds -lcudart_static (or -lcudart) -lrt -ldl -lpthread -lstdc++
        if os.path.exists(STATIC_LIB):
            os.remove(STATIC_LIB)
        cmd = [NVCC] + ARCH + ["-lib", "-o", STATIC_LIB] + objs
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"archive failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
