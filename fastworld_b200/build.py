"""Build ``libfastworld_b200.so`` in-tree with nvcc for sm_100a (no JIT cache, no torch extension).

    python -m fastworld_b200.build [--verbose]

Each ``csrc/*.cu`` is compiled to an object in ``_build/`` (in parallel, skipped when up to
date) and linked into ``fastworld_b200/libfastworld_b200.so`` with the static CUDA runtime.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(HERE, "libfastworld_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I", os.path.join(ROOT, "include")]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _deps() -> list:
    return [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))] + \
        [os.path.join(ROOT, "include", f) for f in os.listdir(os.path.join(ROOT, "include"))]


def _compile(src: str, obj: str, verbose: bool) -> str:
    cmd = [nvcc(), *ARCH, *FLAGS, "-c", src, "-o", obj]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{r.stderr}")
    return r.stderr


def build(verbose: bool = False, force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))
    dep_t = max(os.path.getmtime(d) for d in _deps())
    jobs, objs = [], []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if force or verbose or not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s), dep_t):
            jobs.append((s, o))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        for (s, _), log in zip(jobs, ex.map(lambda j: _compile(j[0], j[1], verbose), jobs)):
            if verbose and log:
                print(f"== {os.path.basename(s)}\n{log}", file=sys.stderr)
    if jobs or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        tmp = LIB + ".tmp"
        r = subprocess.run([nvcc(), *ARCH, "-shared", "-o", tmp, *objs], capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(a.verbose, a.force))
