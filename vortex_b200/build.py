"""Build libvxb.so (all CUDA sources of vortex_b200/csrc) for sm_100a.

Usage: python -m vortex_b200.build [--force]

Objects go to vortex_b200/_build/, the shared library to
vortex_b200/_lib/libvxb.so (in-tree, so it travels with the repository
snapshot). The CUDA runtime is linked statically; NCCL is opened at run time.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIBDIR = os.path.join(HERE, "_lib")
LIB = os.path.join(LIBDIR, "libvxb.so")
ROOT = os.path.dirname(HERE)

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-std=c++17", "-lineinfo",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-Xcompiler", "-Wall", "-Xptxas", "-warn-spills",
    f"-I{os.path.join(ROOT, 'include')}",
]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build vortex_b200")


def _newer(src_list, target) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in src_list)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    cus = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = sorted(glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(ROOT, "include", "*.h")))
    nv = nvcc()
    jobs = []
    objs = []
    for cu in cus:
        obj = os.path.join(BUILD, os.path.basename(cu)[:-3] + ".o")
        objs.append(obj)
        if force or _newer([cu] + headers, obj):
            jobs.append([nv] + NVCC_FLAGS + ["-c", cu, "-o", obj])

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        return cmd, r

    failed = []
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        for cmd, r in ex.map(run, jobs):
            if verbose or r.returncode:
                sys.stderr.write(r.stdout + r.stderr)
            if r.returncode:
                failed.append(cmd[-3])
    if failed:
        raise RuntimeError(f"nvcc failed for: {failed}")
    if force or jobs or _newer(objs, LIB):
        link = [nv] + ARCH + ["-shared", "-cudart=static", "-o", LIB] + objs + ["-ldl", "-lpthread"]
        r = subprocess.run(link, capture_output=True, text=True)
        if r.returncode:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("link of libvxb.so failed")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))
