"""Builds libb2moe.so (all CUDA sources in csrc/) for sm_100a, in-tree.

    python mlxfast-challenge_senpai_b200/build.py [--force] [--jobs N]

Objects go to _build/ next to this file, the library to lib/libb2moe.so and
the C-ABI end-to-end timer (capi_decode_e2e.cpp) to lib/capi_decode_e2e.
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
LIBDIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIBDIR, "libb2moe.so")
CAPI_E2E = os.path.join(LIBDIR, "capi_decode_e2e")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    f"-I{os.path.join(ROOT, 'include')}", f"-I{CSRC}",
]


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h")))


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, force: bool, verbose_ptxas: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    if force or _stale(obj, [src] + _headers()):
        cmd = [NVCC, *ARCH, *FLAGS, "-c", src, "-o", obj]
        if verbose_ptxas:
            cmd[1:1] = ["-Xptxas", "-v"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if verbose_ptxas:
            sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, jobs: int = 0, verbose_ptxas: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    srcs = _sources()
    jobs = jobs or min(len(srcs), os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, verbose_ptxas), srcs))
    if force or _stale(LIB, objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-cudart", "static"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    # the C-ABI end-to-end timer (host code linked against the library)
    src = os.path.join(HERE, "capi_decode_e2e.cpp")
    if force or _stale(CAPI_E2E, [src, LIB] + _headers()):
        cmd = [NVCC, "-O2", "-std=c++17", f"-I{os.path.join(ROOT, 'include')}", src, "-o", CAPI_E2E,
               f"-L{LIBDIR}", "-lb2moe", "-Xlinker", "-rpath", "-Xlinker", "$ORIGIN"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"capi_decode_e2e build failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=0)
    ap.add_argument("--ptxas-v", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.jobs, a.ptxas_v))
